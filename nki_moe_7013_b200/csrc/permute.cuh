// K2: expert-grouped permutation.
//
// Replaces the NxDI blockwise preparation whose outputs the reference's
// prefill kernels consume (token_position_to_id / block_to_expert,
// qwen_with_nki.py:5872-5881; padding row qwen_with_nki.py:5466-5470).  Instead
// of fixed 512-row blocks with padding slots, every expert gets one contiguous
// range of rows (no padding rows at all) cut into 128-row tiles for the
// grouped GEMMs.
//
//   scan kernel    (1 CTA per expert): per-chunk histogram column ->
//                  per-chunk exclusive prefix and the expert's row count.
//   scatter kernel (1 CTA per router chunk): expert offsets by a block scan
//                  of the counts (CTA 0 also publishes offsets and the tile
//                  list); the rank of a (token, slot) pair
//                  inside its expert is the number of earlier tokens of the
//                  chunk that chose the same expert (popcount of a bitmask)
//                  plus the chunk prefix, so rows inside an expert follow
//                  ascending token id -- deterministic and bit-exact.  The CTA
//                  then gathers its tokens' activation rows into x_perm and
//                  zero-fills their rows of the fp32 combine accumulator.
#pragma once

#include "common.cuh"
#include "router.cuh"

namespace qmoe {

constexpr int kTileRows = 128;  // rows per grouped-GEMM tile
constexpr int kScanThreads = 256;
constexpr int kScatterThreads = 256;

// Exclusive block-wide scan of one int per thread (blockDim.x == 256).
__device__ __forceinline__ int block_exclusive_scan_256(int v, int* total, int* warp_sums) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int ws = lane < 8 ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) {
      const int n = __shfl_up_sync(0xFFFFFFFFu, ws, off);
      if (lane >= off) ws += n;
    }
    if (lane < 8) warp_sums[lane] = ws;  // inclusive
  }
  __syncthreads();
  const int base = warp > 0 ? warp_sums[warp - 1] : 0;
  *total = warp_sums[7];
  __syncthreads();
  return base + incl - v;
}

// Column scan: CTA e turns chunk_hist[:, e] into its exclusive prefix over
// chunks and writes counts[e].
__global__ void __launch_bounds__(kScanThreads)
    permute_scan_kernel(int32_t* __restrict__ chunk_hist, int nchunks, int E,
                        int32_t* __restrict__ counts) {
  __shared__ int warp_sums[8];
  const int e = blockIdx.x;
  if (threadIdx.x == 0) QMOE_TRACE_AT(4, 0);
  griddep_wait();
  griddep_launch_dependents();
  const int per = (nchunks + kScanThreads - 1) / kScanThreads;
  const int c0 = min(nchunks, int(threadIdx.x) * per);
  const int c1 = min(nchunks, c0 + per);
  int local = 0;
  for (int c = c0; c < c1; ++c) local += chunk_hist[size_t(c) * E + e];
  int total = 0;
  int run = block_exclusive_scan_256(local, &total, warp_sums);
  for (int c = c0; c < c1; ++c) {
    const int v = chunk_hist[size_t(c) * E + e];
    chunk_hist[size_t(c) * E + e] = run;
    run += v;
  }
  if (threadIdx.x == 0) counts[e] = total;
  if (threadIdx.x == 0) QMOE_TRACE_AT(4, 3);
}

// One CTA per router chunk (8 tokens); gridDim.y CTAs share the row gather.
__global__ void __launch_bounds__(kScatterThreads)
    permute_scatter_kernel(const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
                           const int32_t* __restrict__ chunk_prefix,
                           const int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                           const __nv_bfloat16* __restrict__ x, int T, int H, int E, int k,
                           int32_t* __restrict__ row_token, float* __restrict__ row_w,
                           int32_t* __restrict__ slot_row, __nv_bfloat16* __restrict__ x_perm,
                           float* __restrict__ acc_zero, int32_t* __restrict__ tiles, int max_tiles,
                           int32_t* __restrict__ zero_words, int n_zero_words) {
  __shared__ unsigned mask[256];
  __shared__ int off_s[256];
  __shared__ int pos_s[kScatterThreads];
  __shared__ int warp_sums[8];
  const int c = blockIdx.x;
  const int part = blockIdx.y;
  const int t0 = c * kRouterChunk;
  const int nt = min(kRouterChunk, T - t0);
  const int npairs = nt * k;
  const int tid = threadIdx.x;
  if (threadIdx.x == 0 && blockIdx.y == 0) QMOE_TRACE_AT(5, 0);
  griddep_wait();
  griddep_launch_dependents();

  // Expert offsets: exclusive scan of counts (E <= 256).
  const int cnt = tid < E ? counts[tid] : 0;
  int total = 0;
  const int off = block_exclusive_scan_256(cnt, &total, warp_sums);
  if (tid < E) off_s[tid] = off;
  if (c == 0 && part == 0) {
    // Also publish offsets and the 128-row tile list (expert order).
    int tot_tiles = 0;
    const int nt_e = (cnt + kTileRows - 1) / kTileRows;
    const int tbase = block_exclusive_scan_256(nt_e, &tot_tiles, warp_sums);
    if (tid < E) {
      offsets[tid] = off;
      int32_t* t_exp = tiles + 1;
      int32_t* t_row0 = t_exp + max_tiles;
      int32_t* t_rows = t_row0 + max_tiles;
      for (int i = 0; i < nt_e; ++i) {
        const int ti = tbase + i;
        if (ti < max_tiles) {
          t_exp[ti] = tid;
          t_row0[ti] = off + i * kTileRows;
          t_rows[ti] = min(kTileRows, cnt - i * kTileRows);
        }
      }
    }
    if (tid == 0) {
      offsets[E] = total;
      tiles[0] = min(tot_tiles, max_tiles);
    }
  }
  if (c == 0 && part == 0)
    for (int i = tid; i < n_zero_words; i += kScatterThreads) zero_words[i] = 0;
  for (int i = tid; i < E; i += kScatterThreads) mask[i] = 0u;
  __syncthreads();
  int e = -1;
  if (tid < npairs) {
    e = topk_idx[size_t(t0) * k + tid];
    if (e < 0 || e >= E) {
      record_device_error(kDevErrBadIndex);
      e = -1;
    } else {
      atomicOr(&mask[e], 1u << (tid / k));
    }
  }
  __syncthreads();
  if (tid < npairs) {
    int pos = -1;
    if (e >= 0) {
      const int tl = tid / k;
      const int rank = __popc(mask[e] & ((1u << tl) - 1u));
      pos = off_s[e] + chunk_prefix[size_t(c) * E + e] + rank;
      if (part == 0) {
        row_token[pos] = t0 + tl;
        row_w[pos] = topk_w[size_t(t0) * k + tid];
      }
    }
    if (part == 0) slot_row[size_t(t0) * k + tid] = pos;
    pos_s[tid] = pos;
  }
  __syncthreads();
  if (x_perm) {
    // rows of this chunk split across gridDim.y CTAs; 4 independent 16-byte
    // copies in flight per thread
    const int vec_per_row = H / 8;
    const int total_v = npairs * vec_per_row;
    const int stride = kScatterThreads * gridDim.y;
    for (int v0 = part * kScatterThreads + tid; v0 < total_v; v0 += 4 * stride) {
      uint4 val[4];
      int dst[4], col[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int v = v0 + u * stride;
        dst[u] = -1;
        if (v < total_v) {
          const int p = v / vec_per_row;
          col[u] = (v - p * vec_per_row) * 8;
          dst[u] = pos_s[p];
          if (dst[u] >= 0)
            val[u] = *reinterpret_cast<const uint4*>(x + size_t(t0 + p / k) * H + col[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (dst[u] >= 0) *reinterpret_cast<uint4*>(x_perm + size_t(dst[u]) * H + col[u]) = val[u];
    }
  }
  if (acc_zero) {
    // the chunk's accumulator rows, split across the chunk's CTAs
    const int vec_per_row = H / 4;
    const int total_v = nt * vec_per_row;
    for (int v = part * kScatterThreads + tid; v < total_v; v += kScatterThreads * gridDim.y) {
      const int tl = v / vec_per_row;
      const int cc = (v % vec_per_row) * 4;
      *reinterpret_cast<float4*>(acc_zero + size_t(t0 + tl) * H + cc) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if (threadIdx.x == 0 && blockIdx.y == 0) QMOE_TRACE_AT(5, 3);
}

}  // namespace qmoe
