// Expert-parallel plumbing around the NCCL all-to-alls.
//
// The reference's EP variant (qwen_with_nki.py:8148-8271) computes only local
// experts on every rank and combines with a world all-reduce of masked
// partials.  Here rank r owns experts [r*E_local, (r+1)*E_local) and the
// (token, slot) rows travel to their owner and back:
//
//   routing_hist  per-chunk expert histogram of caller-given routing (the
//                 permutation's input when routing does not come from K1)
//   ep_dest_hist  per-chunk histogram of destination ranks
//   (column scan: permute_scan_kernel over ranks)
//   ep_pack       rows grouped by destination rank, (token, slot) order kept:
//                 send_x (rows of x), send_expert (expert id local to the
//                 destination), send_w (routing weight), pair_pos (row of
//                 each (token, slot) in the send buffer)
//   ep_unpack     out[t] = bf16(residual[t] + sum_j y_back[pair_pos[t, j]]),
//                 the k weighted expert outputs summed in fp32 in slot order
#pragma once

#include "common.cuh"
#include "router.cuh"

namespace qmoe {

constexpr int kEpThreads = 256;

// chunk_hist[c][e] = #pairs of tokens [8c, 8c+8) routed to expert e.
__global__ void __launch_bounds__(kEpThreads)
    routing_hist_kernel(const int32_t* __restrict__ topk_idx, int T, int k, int E,
                        int32_t* __restrict__ chunk_hist) {
  __shared__ int h[256];
  const int c = blockIdx.x;
  for (int i = threadIdx.x; i < E; i += kEpThreads) h[i] = 0;
  __syncthreads();
  const int t0 = c * kRouterChunk;
  const int npairs = min(kRouterChunk, T - t0) * k;
  for (int i = threadIdx.x; i < npairs; i += kEpThreads) {
    const int e = topk_idx[size_t(t0) * k + i];
    if (e >= 0 && e < E) atomicAdd(&h[e], 1);
    else record_device_error(kDevErrBadIndex);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += kEpThreads) chunk_hist[size_t(c) * E + i] = h[i];
}

// chunk_hist[c][d] = #pairs of tokens [8c, 8c+8) whose expert lives on rank d.
__global__ void __launch_bounds__(kEpThreads)
    ep_dest_hist_kernel(const int32_t* __restrict__ topk_idx, int T, int k, int e_local, int n_ranks,
                        int32_t* __restrict__ chunk_hist) {
  __shared__ int h[256];
  const int c = blockIdx.x;
  for (int i = threadIdx.x; i < n_ranks; i += kEpThreads) h[i] = 0;
  __syncthreads();
  const int t0 = c * kRouterChunk;
  const int npairs = min(kRouterChunk, T - t0) * k;
  for (int i = threadIdx.x; i < npairs; i += kEpThreads) {
    const int d = topk_idx[size_t(t0) * k + i] / e_local;
    if (d >= 0 && d < n_ranks) atomicAdd(&h[d], 1);
    else record_device_error(kDevErrBadIndex);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n_ranks; i += kEpThreads) chunk_hist[size_t(c) * n_ranks + i] = h[i];
}

// One CTA per chunk of 8 tokens (<= 256 pairs); rows of one destination rank
// follow (token, slot) order.  counts (n_ranks) comes from the column scan.
__global__ void __launch_bounds__(kEpThreads)
    ep_pack_kernel(const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w,
                   const __nv_bfloat16* __restrict__ x, const int32_t* __restrict__ chunk_prefix,
                   const int32_t* __restrict__ counts, int T, int H, int k, int e_local, int n_ranks,
                   __nv_bfloat16* __restrict__ send_x, int32_t* __restrict__ send_expert,
                   float* __restrict__ send_w, int32_t* __restrict__ pair_pos) {
  __shared__ int dest[kEpThreads];
  __shared__ int pos_s[kEpThreads];
  __shared__ int off[257];
  const int c = blockIdx.x;
  const int t0 = c * kRouterChunk;
  const int npairs = min(kRouterChunk, T - t0) * k;
  const int tid = threadIdx.x;
  if (tid == 0) {
    int o = 0;
    for (int d = 0; d < n_ranks; ++d) {
      off[d] = o;
      o += counts[d];
    }
  }
  int e = -1, d = -1;
  if (tid < npairs) {
    e = topk_idx[size_t(t0) * k + tid];
    d = e / e_local;
    if (e < 0 || d >= n_ranks) d = -1;
  }
  dest[tid] = d;
  __syncthreads();
  if (tid < npairs) {
    int pos = -1;
    if (d >= 0) {
      int rank = 0;
      for (int i = 0; i < tid; ++i) rank += dest[i] == d;
      pos = off[d] + chunk_prefix[size_t(c) * n_ranks + d] + rank;
      send_expert[pos] = e - d * e_local;
      send_w[pos] = topk_w[size_t(t0) * k + tid];
    }
    pair_pos[size_t(t0) * k + tid] = pos;
    pos_s[tid] = pos;
  }
  __syncthreads();
  const int vec_per_row = H / 8;
  const int total = npairs * vec_per_row;
  for (int v0 = tid; v0 < total; v0 += 4 * kEpThreads) {
    uint4 val[4];
    int dst[4], col[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = v0 + u * kEpThreads;
      dst[u] = -1;
      if (v < total) {
        const int p = v / vec_per_row;
        col[u] = (v - p * vec_per_row) * 8;
        dst[u] = pos_s[p];
        if (dst[u] >= 0) val[u] = *reinterpret_cast<const uint4*>(x + size_t(t0 + p / k) * H + col[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (dst[u] >= 0) *reinterpret_cast<uint4*>(send_x + size_t(dst[u]) * H + col[u]) = val[u];
  }
}

// One warp per (token, 256-column slab): fp32 sum of the k returned rows.
__global__ void __launch_bounds__(kEpThreads)
    ep_unpack_kernel(const __nv_bfloat16* __restrict__ y_back, const int32_t* __restrict__ pair_pos,
                     const __nv_bfloat16* __restrict__ residual, int T, int H, int k, int n_back,
                     __nv_bfloat16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int slabs = H / 256;
  const int gw = blockIdx.x * (kEpThreads / 32) + (threadIdx.x >> 5);
  if (gw >= T * slabs) return;
  const int t = gw / slabs;
  const int col = (gw - t * slabs) * 256 + lane * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < k; ++j) {
    const int r = pair_pos ? pair_pos[size_t(t) * k + j] : t * k + j;
    if (r < 0 || r >= n_back) {
      if (r >= n_back) record_device_error(kDevErrBadIndex);
      continue;
    }
    const uint4 v = *reinterpret_cast<const uint4*>(y_back + size_t(r) * H + col);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc[2 * q] += bf16lo_to_f32(w[q]);
      acc[2 * q + 1] += bf16hi_to_f32(w[q]);
    }
  }
  if (residual) {
    const uint4 v = *reinterpret_cast<const uint4*>(residual + size_t(t) * H + col);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc[2 * q] += bf16lo_to_f32(w[q]);
      acc[2 * q + 1] += bf16hi_to_f32(w[q]);
    }
  }
  uint4 o;
  uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
    ow[q] = *reinterpret_cast<const uint32_t*>(&p);
  }
  *reinterpret_cast<uint4*>(out + size_t(t) * H + col) = o;
}

}  // namespace qmoe
