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
//                  then copies its tokens' activation rows into x_perm (TMA
//                  bulk loads of the chunk's 8 token rows into shared memory,
//                  one bulk store per (token, slot) row) and zero-fills their
//                  rows of the fp32 combine accumulator.
//   route_permute kernel (batches of at most one chunk per SM): the router
//                  and both kernels above in one launch -- every CTA routes
//                  its chunk, publishes the chunk histogram, waits at one
//                  grid-wide barrier (all CTAs are resident), then sums the
//                  published histograms into the counts and its own chunk
//                  prefix and does its chunk's scatter.  Same outputs, bit
//                  for bit, as router_topk + scan + scatter.  The chunk's
//                  token rows are bulk-loaded into shared memory while the
//                  CTA routes; each permuted row is one bulk store.
#pragma once

#include "common.cuh"
#include "router.cuh"

namespace qmoe {

constexpr int kTileRows = 128;  // rows per grouped-GEMM tile
constexpr int kScanThreads = 256;
constexpr int kScatterThreads = 256;

// Exclusive block-wide scan of one int per thread (blockDim.x a multiple of
// 32, at most 1024); *total = the block sum.  warp_sums: 32 ints of shared
// memory.
__device__ __forceinline__ int block_exclusive_scan(int v, int* total, int* warp_sums) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int ws = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(0xFFFFFFFFu, ws, off);
      if (lane >= off) ws += n;
    }
    if (lane < nw) warp_sums[lane] = ws;  // inclusive
  }
  __syncthreads();
  const int base = warp > 0 ? warp_sums[warp - 1] : 0;
  *total = warp_sums[nw - 1];
  __syncthreads();
  return base + incl - v;
}

// Column scan: CTA e turns chunk_hist[:, e] into its exclusive prefix over
// chunks and writes counts[e].
__global__ void __launch_bounds__(kScanThreads)
    permute_scan_kernel(int32_t* __restrict__ chunk_hist, int nchunks, int E,
                        int32_t* __restrict__ counts) {
  __shared__ int warp_sums[32];
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
  int run = block_exclusive_scan(local, &total, warp_sums);
  for (int c = c0; c < c1; ++c) {
    const int v = chunk_hist[size_t(c) * E + e];
    chunk_hist[size_t(c) * E + e] = run;
    run += v;
  }
  if (threadIdx.x == 0) counts[e] = total;
  if (threadIdx.x == 0) QMOE_TRACE_AT(4, 3);
}

// Expert offsets from the counts (thread e < E passes counts[e] as cnt, the
// others 0): off_s[e] = exclusive prefix.  With `publish` the CTA also
// writes offsets (E+1), the 128-row tile list and (if given) counts.  All
// threads of the block take part.
__device__ __forceinline__ void permute_offsets(int cnt, int E, bool publish, int* off_s, int* warp_sums,
                                                int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                                                int32_t* __restrict__ tiles, int max_tiles) {
  const int tid = threadIdx.x;
  int total = 0;
  const int off = block_exclusive_scan(cnt, &total, warp_sums);
  if (tid < E) off_s[tid] = off;
  if (publish) {
    int tot_tiles = 0;
    const int nt_e = (cnt + kTileRows - 1) / kTileRows;
    const int tbase = block_exclusive_scan(nt_e, &tot_tiles, warp_sums);
    if (tid < E) {
      if (counts) counts[tid] = cnt;
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
  __syncthreads();
}

// One chunk's rows: rank of each (token, slot) pair inside its expert, its
// permuted row (offsets + chunk prefix + rank), and with write_rows the
// row_token / row_w / slot_row outputs.  pos_s[p] (shared, one per pair of
// the chunk) receives the permuted row of pair p or -1.  pre(e) is the
// chunk's prefix of expert e.  mask: E unsigned of shared memory.
template <typename Prefix>
__device__ __forceinline__ void permute_chunk_rows(int c, int T, int E, int k, const int32_t* __restrict__ topk_idx,
                                                   const float* __restrict__ topk_w, const int* off_s, Prefix pre,
                                                   bool write_rows, int32_t* __restrict__ row_token,
                                                   float* __restrict__ row_w, int32_t* __restrict__ slot_row,
                                                   unsigned* mask, int* pos_s) {
  const int tid = threadIdx.x;
  const int t0 = c * kRouterChunk;
  const int npairs = min(kRouterChunk, T - t0) * k;
  for (int i = tid; i < E; i += blockDim.x) mask[i] = 0u;
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
      pos = off_s[e] + pre(e) + rank;
      if (write_rows) {
        row_token[pos] = t0 + tl;
        row_w[pos] = topk_w[size_t(t0) * k + tid];
      }
    }
    if (write_rows) slot_row[size_t(t0) * k + tid] = pos;
    pos_s[tid] = pos;
  }
  __syncthreads();
}

// The chunk's rows of the combine accumulator zero-filled; this CTA takes
// share `part` of `nparts`.
__device__ __forceinline__ void permute_chunk_zero_acc(int c, int part, int nparts, int T, int H,
                                                       float* __restrict__ acc_zero) {
  if (!acc_zero) return;
  const int t0 = c * kRouterChunk;
  const int nt = min(kRouterChunk, T - t0);
  const int vec_per_row = H / 4;
  const int total_v = nt * vec_per_row;
  for (int v = part * blockDim.x + threadIdx.x; v < total_v; v += blockDim.x * nparts) {
    const int tl = v / vec_per_row;
    const int cc = (v % vec_per_row) * 4;
    *reinterpret_cast<float4*>(acc_zero + size_t(t0 + tl) * H + cc) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// The chunk's (token, slot) rows of this CTA's share into x_perm with one
// bulk store each, from the token rows (rows_s, bf16, loaded on rows_bar);
// every thread that issued waits until its store has read shared memory (the
// writes complete on their own; the next grid sees them).  Thread 0 also
// waits for the row loads when it issues nothing, so no load outlives the
// CTA.  (The copy is bound by the aggregate write rate, ~5.6 TB/s for the
// 1,024-token layer's 33.5 MB: 16-byte stores from every thread were slower.)
__device__ __forceinline__ void permute_chunk_bulk_rows(int c, int part, int nparts, int T, int H, int k,
                                                        const int* pos_s, const __nv_bfloat16* rows_s,
                                                        uint64_t* rows_bar, int* rows_abort,
                                                        __nv_bfloat16* __restrict__ x_perm) {
  const int tid = threadIdx.x;
  const int npairs = min(kRouterChunk, T - c * kRouterChunk) * k;
  const bool mine = tid < npairs && tid % nparts == part;
  if (mine || tid == 0) {
    const bool rows_in = mbar_wait_bounded(rows_bar, 0, rows_abort, kDevErrWaitTimeoutProducer);
    const int pos = mine ? pos_s[tid] : -1;
    if (rows_in && pos >= 0) {
      bulk_store(x_perm + size_t(pos) * H, rows_s + (tid / k) * H, H * 2);
      bulk_commit_group();
      bulk_wait_read_all();
    }
  }
}

// Thread 0: bulk loads of the chunk's token rows into rows_s (bf16) on
// rows_bar (initialised here).
__device__ __forceinline__ void permute_chunk_load_rows(int c, int T, int H, const __nv_bfloat16* __restrict__ x,
                                                        __nv_bfloat16* rows_s, uint64_t* rows_bar, int* rows_abort) {
  const int nt = min(kRouterChunk, T - c * kRouterChunk);
  *rows_abort = 0;
  mbar_init(rows_bar, 1);
  fence_mbarrier_init();
  mbar_arrive_expect_tx(rows_bar, uint32_t(nt) * H * 2);
  for (int t = 0; t < nt; ++t) bulk_load(rows_s + t * H, x + size_t(c * kRouterChunk + t) * H, H * 2, rows_bar);
}

// One CTA per router chunk (8 tokens); gridDim.y CTAs share the row copy.
// Dynamic shared memory: kRouterChunk * H bf16 when x_perm is set.
__global__ void __launch_bounds__(kScatterThreads)
    permute_scatter_kernel(const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
                           const int32_t* __restrict__ chunk_prefix,
                           const int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                           const __nv_bfloat16* __restrict__ x, int T, int H, int E, int k,
                           int32_t* __restrict__ row_token, float* __restrict__ row_w,
                           int32_t* __restrict__ slot_row, __nv_bfloat16* __restrict__ x_perm,
                           float* __restrict__ acc_zero, int32_t* __restrict__ tiles, int max_tiles,
                           int32_t* __restrict__ zero_words, int n_zero_words) {
  extern __shared__ __align__(16) __nv_bfloat16 scatter_rows_s[];
  __shared__ unsigned mask[256];
  __shared__ int off_s[256];
  __shared__ int pos_s[kScatterThreads];
  __shared__ int warp_sums[32];
  __shared__ __align__(8) uint64_t rows_bar;
  __shared__ int rows_abort;
  const int c = blockIdx.x;
  const int part = blockIdx.y;
  const int tid = threadIdx.x;
  if (threadIdx.x == 0 && blockIdx.y == 0) QMOE_TRACE_AT(5, 0);
  griddep_wait();
  griddep_launch_dependents();
  // x is an input of the layer, not of the router: its rows can be in flight
  // while the offsets and ranks are worked out
  if (x_perm && tid == 0) permute_chunk_load_rows(c, T, H, x, scatter_rows_s, &rows_bar, &rows_abort);

  const bool lead = c == 0 && part == 0;
  permute_offsets(tid < E ? counts[tid] : 0, E, lead, off_s, warp_sums, nullptr, offsets, tiles, max_tiles);
  if (lead)
    for (int i = tid; i < n_zero_words; i += kScatterThreads) zero_words[i] = 0;
  const int32_t* pre_row = chunk_prefix + size_t(c) * E;
  permute_chunk_rows(
      c, T, E, k, topk_idx, topk_w, off_s, [&](int e) { return pre_row[e]; }, part == 0, row_token, row_w,
      slot_row, mask, pos_s);
  permute_chunk_zero_acc(c, part, gridDim.y, T, H, acc_zero);
  if (x_perm)
    permute_chunk_bulk_rows(c, part, gridDim.y, T, H, k, pos_s, scatter_rows_s, &rows_bar, &rows_abort, x_perm);
  if (threadIdx.x == 0 && blockIdx.y == 0) QMOE_TRACE_AT(5, 3);
}

// Dynamic shared memory of route_permute_kernel: the router's staging (or
// the histogram partials, <= 32 B per thread, that reuse it), then the
// chunk's token rows in bf16.
__host__ __device__ constexpr int route_permute_stage_bytes(int H, int E, int threads) {
  return ((4 * kRouterChunk * (H + E) > 32 * threads ? 4 * kRouterChunk * (H + E) : 32 * threads) + 15) / 16 * 16;
}
__host__ __device__ constexpr int route_permute_smem_bytes(int H, int E, int threads) {
  return route_permute_stage_bytes(H, E, threads) + 2 * kRouterChunk * H;
}

// Router + permutation in one launch for nchunks <= SMs (see the header
// comment).  chunk_hist (nchunks, E) int32 scratch receives the raw chunk
// histograms; barrier: two int32 (arrivals, departures of the grid-wide
// barrier), zero on entry -- the last CTA through resets both, so a launch
// that completes leaves them zero for the next.  Writes what router_topk +
// scan + scatter write except the per-chunk prefixes (chunk_hist keeps the
// histograms).
template <int G>
__global__ void __launch_bounds__(router_warps<G>() * 32, 1)
    route_permute_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                         const float* __restrict__ bias, int T, int E, int k, int normalize,
                         int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, int32_t* __restrict__ chunk_hist,
                         int32_t* __restrict__ counts, int32_t* __restrict__ offsets, int32_t* __restrict__ row_token,
                         float* __restrict__ row_w, int32_t* __restrict__ slot_row, __nv_bfloat16* __restrict__ x_perm,
                         float* __restrict__ acc_zero, int32_t* __restrict__ tiles, int max_tiles,
                         int32_t* __restrict__ zero_words, int n_zero_words, int* __restrict__ barrier) {
  constexpr int kWarps = router_warps<G>();
  constexpr int kThreads = kWarps * 32;
  constexpr int H = G * 256;
  extern __shared__ __align__(16) float router_smem[];
  __shared__ int hist[256];
  __shared__ unsigned mask[256];
  __shared__ int pre_s[256];
  __shared__ int off_s[256];
  __shared__ int pos_s[kThreads];
  __shared__ int warp_sums[32];
  __shared__ __align__(8) uint64_t rows_bar;
  __shared__ int rows_abort;
  const int c = blockIdx.x;
  const int tid = threadIdx.x;
  __nv_bfloat16* rows_s = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(router_smem) +
                                                           route_permute_stage_bytes(H, E, kThreads));
  if (tid == 0) QMOE_TRACE_AT(0, 0);
  griddep_wait();
  griddep_launch_dependents();
  const bool copy_rows = x_perm != nullptr;
  if (tid == 0) QMOE_TRACE_AT(0, 1);
  // the chunk's token rows, bf16, for the bulk stores after the barrier
  if (copy_rows && tid == 0) permute_chunk_load_rows(c, T, H, x, rows_s, &rows_bar, &rows_abort);
  router_chunk<G, kWarps>(c, x, w, bias, T, E, k, normalize, nullptr, topk_idx, topk_w, router_smem,
                          router_smem + kRouterChunk * H, hist);
  for (int e = tid; e < E; e += kThreads) chunk_hist[size_t(c) * E + e] = hist[e];
  if (!grid_barrier_once(barrier, kDevErrWaitTimeoutProducer)) {
    // the row loads land before the CTA leaves
    if (copy_rows && tid == 0) mbar_wait_bounded(&rows_bar, 0, &rows_abort, kDevErrWaitTimeoutProducer);
    return;
  }
  // every CTA has passed the wait once its departure is counted: the last one
  // clears the barrier for the next launch
  if (tid == 0) {
    QMOE_TRACE_AT(0, 2);
    if (atomicAdd(barrier + 1, 1) == int(gridDim.x) - 1) {
      barrier[0] = 0;
      barrier[1] = 0;
    }
  }

  // Every chunk's histogram is out: this chunk's prefix and the counts.  A
  // thread sums 4 experts over a strided subset of the chunks (16-byte loads
  // through L2: the rows were written by other SMs); the row groups' partials
  // meet in shared memory (the staging area, free after the router).
  const int E4 = E / 4;
  const int n_rg = kThreads / E4;
  int* part_tot = reinterpret_cast<int*>(router_smem);  // [n_rg][E]
  int* part_pre = part_tot + n_rg * E;                  // [n_rg][E]
  if (tid < n_rg * E4) {
    const int col4 = tid % E4;
    const int rg = tid / E4;
    int4 tot = make_int4(0, 0, 0, 0), pre = tot;
    // eight rows' loads in flight at a time
    for (int r0 = rg; r0 < int(gridDim.x); r0 += 8 * n_rg) {
      int4 h[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int r = r0 + u * n_rg;
        h[u] = r < int(gridDim.x) ? __ldcg(reinterpret_cast<const int4*>(chunk_hist + size_t(r) * E) + col4)
                                  : make_int4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int r = r0 + u * n_rg;
        tot.x += h[u].x;
        tot.y += h[u].y;
        tot.z += h[u].z;
        tot.w += h[u].w;
        if (r < c) {
          pre.x += h[u].x;
          pre.y += h[u].y;
          pre.z += h[u].z;
          pre.w += h[u].w;
        }
      }
    }
    reinterpret_cast<int4*>(part_tot + rg * E)[col4] = tot;
    reinterpret_cast<int4*>(part_pre + rg * E)[col4] = pre;
  }
  __syncthreads();
  if (tid == 0) QMOE_TRACE_AT(0, 4);
  int cnt = 0;
  if (tid < E) {
    int p = 0;
    for (int rg = 0; rg < n_rg; ++rg) {
      cnt += part_tot[rg * E + tid];
      p += part_pre[rg * E + tid];
    }
    pre_s[tid] = p;
  }
  const bool lead = c == 0;
  permute_offsets(cnt, E, lead, off_s, warp_sums, counts, offsets, tiles, max_tiles);
  if (tid == 0) QMOE_TRACE_AT(0, 5);
  if (lead)
    for (int i = tid; i < n_zero_words; i += kThreads) zero_words[i] = 0;
  permute_chunk_rows(
      c, T, E, k, topk_idx, topk_w, off_s, [&](int e) { return pre_s[e]; }, true, row_token, row_w, slot_row, mask,
      pos_s);
  if (tid == 0) QMOE_TRACE_AT(0, 6);
  permute_chunk_zero_acc(c, 0, 1, T, H, acc_zero);
  if (tid == 0) QMOE_TRACE_AT(0, 7);
  if (copy_rows) permute_chunk_bulk_rows(c, 0, 1, T, H, k, pos_s, rows_s, &rows_bar, &rows_abort, x_perm);
  if (tid == 0) QMOE_TRACE_AT(0, 3);
}

}  // namespace qmoe
