// K2: expert-grouped permutation.
//
// Replaces the NxDI blockwise preparation whose outputs the reference's
// prefill kernels consume (token_position_to_id / block_to_expert,
// qwen_with_nki.py:5872-5881; padding row qwen_with_nki.py:5466-5470).  Instead
// of fixed 512-row blocks with padding slots, every expert gets one contiguous
// range of rows (no padding rows at all) cut into 128-row tiles for the
// grouped GEMMs.
//
//   scan kernel    (1 CTA): per-chunk histograms -> per-chunk exclusive
//                  prefixes, expert counts / offsets, and the tile list.
//   scatter kernel (1 CTA per router chunk): the rank of a (token, slot) pair
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
constexpr int kScanThreads = 1024;
constexpr int kScatterThreads = 256;

__global__ void __launch_bounds__(kScanThreads, 1)
    permute_scan_kernel(int32_t* __restrict__ chunk_hist, int nchunks, int E,
                        int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                        int32_t* __restrict__ tiles, int max_tiles) {
  __shared__ int part_sum[kScanThreads];  // [part][E]
  __shared__ int tot[1024];
  __shared__ int off_s[1025];
  __shared__ int tile_base[1025];
  const int tid = threadIdx.x;
  const int parts = kScanThreads / E;
  const int e = tid % E;
  const int part = tid / E;
  const bool active = part < parts;
  const int cpp = (nchunks + parts - 1) / parts;
  const int c0 = min(nchunks, part * cpp);
  const int c1 = min(nchunks, c0 + cpp);

  int local = 0;
  if (active)
    for (int c = c0; c < c1; ++c) local += chunk_hist[size_t(c) * E + e];
  part_sum[tid] = local;
  __syncthreads();
  if (active) {
    int run = 0;
    for (int p = 0; p < part; ++p) run += part_sum[p * E + e];
    for (int c = c0; c < c1; ++c) {
      const int v = chunk_hist[size_t(c) * E + e];
      chunk_hist[size_t(c) * E + e] = run;
      run += v;
    }
    if (part == 0) {
      int total = 0;
      for (int p = 0; p < parts; ++p) total += part_sum[p * E + e];
      tot[e] = total;
    }
  }
  __syncthreads();
  if (tid == 0) {
    int o = 0, tb = 0;
    for (int i = 0; i < E; ++i) {
      off_s[i] = o;
      tile_base[i] = tb;
      o += tot[i];
      tb += (tot[i] + kTileRows - 1) / kTileRows;
    }
    off_s[E] = o;
    tile_base[E] = tb;
    offsets[E] = o;
    tiles[0] = min(tb, max_tiles);
  }
  __syncthreads();
  if (tid < E) {
    counts[tid] = tot[tid];
    offsets[tid] = off_s[tid];
    const int n = tot[tid];
    int32_t* t_exp = tiles + 1;
    int32_t* t_row0 = t_exp + max_tiles;
    int32_t* t_rows = t_row0 + max_tiles;
    for (int i = 0; i * kTileRows < n; ++i) {
      const int ti = tile_base[tid] + i;
      if (ti < max_tiles) {
        t_exp[ti] = tid;
        t_row0[ti] = off_s[tid] + i * kTileRows;
        t_rows[ti] = min(kTileRows, n - i * kTileRows);
      }
    }
  }
}

__global__ void __launch_bounds__(kScatterThreads)
    permute_scatter_kernel(const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
                           const int32_t* __restrict__ chunk_prefix,
                           const int32_t* __restrict__ offsets,
                           const __nv_bfloat16* __restrict__ x, int T, int H, int E, int k,
                           int32_t* __restrict__ row_token, float* __restrict__ row_w,
                           int32_t* __restrict__ slot_row, __nv_bfloat16* __restrict__ x_perm,
                           float* __restrict__ acc_zero) {
  __shared__ unsigned mask[256];
  __shared__ int pos_s[kScatterThreads];
  const int c = blockIdx.x;
  const int t0 = c * kRouterChunk;
  const int nt = min(kRouterChunk, T - t0);
  const int npairs = nt * k;
  for (int i = threadIdx.x; i < E; i += kScatterThreads) mask[i] = 0u;
  __syncthreads();
  const int i = threadIdx.x;
  int e = -1;
  if (i < npairs) {
    e = topk_idx[size_t(t0) * k + i];
    if (e < 0 || e >= E) {
      record_device_error(kDevErrBadIndex);
      e = -1;
    } else {
      atomicOr(&mask[e], 1u << (i / k));
    }
  }
  __syncthreads();
  if (i < npairs) {
    int pos = -1;
    if (e >= 0) {
      const int tl = i / k;
      const int rank = __popc(mask[e] & ((1u << tl) - 1u));
      pos = offsets[e] + chunk_prefix[size_t(c) * E + e] + rank;
      row_token[pos] = t0 + tl;
      row_w[pos] = topk_w[size_t(t0) * k + i];
    }
    slot_row[size_t(t0) * k + i] = pos;
    pos_s[i] = pos;
  }
  __syncthreads();
  if (x_perm) {
    const int vec_per_row = H / 8;  // 16-byte vectors
    const int total = npairs * vec_per_row;
    for (int v = threadIdx.x; v < total; v += kScatterThreads) {
      const int p = v / vec_per_row;
      const int col = (v % vec_per_row) * 8;
      const int dst = pos_s[p];
      if (dst < 0) continue;
      const int tok = t0 + p / k;
      const uint4 val = *reinterpret_cast<const uint4*>(x + size_t(tok) * H + col);
      *reinterpret_cast<uint4*>(x_perm + size_t(dst) * H + col) = val;
    }
  }
  if (acc_zero) {
    const int vec_per_row = H / 4;
    const int total = nt * vec_per_row;
    for (int v = threadIdx.x; v < total; v += kScatterThreads) {
      const int tl = v / vec_per_row;
      const int col = (v % vec_per_row) * 4;
      *reinterpret_cast<float4*>(acc_zero + size_t(t0 + tl) * H + col) =
          make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

}  // namespace qmoe
