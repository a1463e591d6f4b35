// Decode-sized batches: router and permutation in ONE launch.
//
// At a few tokens the separate router (logits + selection) and permutation
// (scan + scatter) kernels are four launches of mostly latency.  Here one
// thread-block cluster of kRouteSmallCtas CTAs does all of it:
//
//   every CTA   stages the T token rows (bf16) in shared memory, computes the
//               fp32 logits of its E / kRouteSmallCtas experts (one warp per
//               expert, all tokens) in the canonical order of the fused router
//               (lane l owns elements [8l, 8l+8) of each 256-element group,
//               group-major FMA from +0, xor butterfly 16..1), writes them to
//               `logits` and into CTA 0's shared memory (distributed shared
//               memory of the cluster), and zeroes its slice of the combine
//               accumulator;
//   cluster barrier (release / acquire);
//   CTA 0       softmax + top-k + renorm per token (select_topk_warp, as the
//               other router kernels), then the stable expert-grouped
//               permutation (rows of an expert in ascending token order),
//               expert offsets and the 128-row tile list.
//
// Outputs match router_topk + moe_permute bit for bit (routing, rows, tiles);
// the per-chunk histogram is not produced.
#pragma once

#include "common.cuh"
#include "router.cuh"

namespace qmoe {

constexpr int kRouteSmallCtas = 8;    // one cluster (portable size)
constexpr int kRouteSmallMaxT = 16;   // tokens per launch
constexpr int kRouteSmallMaxE = 128;  // experts: one warp each, E/8 warps per CTA
constexpr int kRouteSmallTileRows = 128;

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Exclusive scan of v[0..n) (n <= 256, n % 32 == 0) by one warp, in place;
// returns the total.
__device__ __forceinline__ int warp_exclusive_scan_smem(int* v, int n, int lane) {
  const int per = n / 32;
  int local = 0;
  for (int i = 0; i < per; ++i) local += v[lane * per + i];
  int incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += o;
  }
  int run = incl - local;
  for (int i = 0; i < per; ++i) {
    const int c = v[lane * per + i];
    v[lane * per + i] = run;
    run += c;
  }
  return __shfl_sync(0xFFFFFFFFu, incl, 31);
}

template <int G>  // G = H / 256
__global__ void __launch_bounds__(kRouteSmallMaxE / kRouteSmallCtas * 32, 1)
    route_small_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                       const float* __restrict__ bias, int T, int E, int k, int normalize,
                       float* __restrict__ logits, int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
                       int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                       int32_t* __restrict__ row_token, float* __restrict__ row_w,
                       int32_t* __restrict__ slot_row, int32_t* __restrict__ tiles, int max_tiles,
                       float* __restrict__ acc_zero, int32_t* __restrict__ zero_words, int n_zero_words) {
  constexpr int H = G * 256;
  extern __shared__ __align__(16) uint8_t route_small_smem[];
  // [Tpad][H] bf16 token rows | [T][E] fp32 logits (CTA 0's copy is filled by
  // every CTA) | [T*k] picks | [T*k] weights
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(route_small_smem);
  float* ls = reinterpret_cast<float*>(route_small_smem + 2 * size_t((T + 3) & ~3) * (G * 256));
  int* idx_s = reinterpret_cast<int*>(ls + T * E);
  float* w_s = reinterpret_cast<float*>(idx_s + T * k);
  __shared__ int hist[256];
  __shared__ int off_s[256];
  __shared__ int tile_s[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;  // the grid is one cluster
  const int e_per = E / kRouteSmallCtas;
  const int Tpad = (T + 3) & ~3;
  if (threadIdx.x == 0) QMOE_TRACE_AT(0, 0);
  // this warp's expert: its canonical weight slice, one load per group.  The
  // router weights (and bias) are not produced by the kernels in front of
  // this one, so their loads are in flight before the dependency wait and
  // overlap the preceding kernel's tail; everything this kernel writes, and
  // every read of x, comes after the wait.
  const int e = cta * e_per + warp;
  uint4 wv[G];
#pragma unroll
  for (int g = 0; g < G; ++g)
    wv[g] = __ldg(reinterpret_cast<const uint4*>(w + size_t(e) * H + 256 * g + 8 * lane));
  const float be = bias ? __ldg(bias + e) : 0.f;
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x == 0) QMOE_TRACE_AT(0, 1);
  {
    const uint4* src = reinterpret_cast<const uint4*>(x);
    uint4* dst = reinterpret_cast<uint4*>(xs);
    const int n = T * (H / 8), npad = Tpad * (H / 8);
    for (int i = threadIdx.x; i < npad; i += blockDim.x) dst[i] = i < n ? src[i] : make_uint4(0u, 0u, 0u, 0u);
  }
  if (cta == kRouteSmallCtas - 1)
    for (int i = threadIdx.x; i < n_zero_words; i += blockDim.x) zero_words[i] = 0;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  uint32_t ls_cta0;  // CTA 0's logits array in the cluster's shared window
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ls_cta0) : "r"(smem_u32(ls)), "r"(0));
  if (acc_zero) {
    const int n4 = T * (H / 4);
    for (int i = cta * blockDim.x + threadIdx.x; i < n4; i += kRouteSmallCtas * blockDim.x)
      reinterpret_cast<float4*>(acc_zero)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();

  // logits: 4 tokens' chains interleaved
  for (int t0 = 0; t0 < T; t0 += 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float wf[8] = {bf16lo_to_f32(wv[g].x), bf16hi_to_f32(wv[g].x), bf16lo_to_f32(wv[g].y),
                           bf16hi_to_f32(wv[g].y), bf16lo_to_f32(wv[g].z), bf16hi_to_f32(wv[g].z),
                           bf16lo_to_f32(wv[g].w), bf16hi_to_f32(wv[g].w)};
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xs + size_t(t0 + tt) * H + 256 * g + 8 * lane);
        acc[tt] = fmaf(bf16lo_to_f32(xv.x), wf[0], acc[tt]);
        acc[tt] = fmaf(bf16hi_to_f32(xv.x), wf[1], acc[tt]);
        acc[tt] = fmaf(bf16lo_to_f32(xv.y), wf[2], acc[tt]);
        acc[tt] = fmaf(bf16hi_to_f32(xv.y), wf[3], acc[tt]);
        acc[tt] = fmaf(bf16lo_to_f32(xv.z), wf[4], acc[tt]);
        acc[tt] = fmaf(bf16hi_to_f32(xv.z), wf[5], acc[tt]);
        acc[tt] = fmaf(bf16lo_to_f32(xv.w), wf[6], acc[tt]);
        acc[tt] = fmaf(bf16hi_to_f32(xv.w), wf[7], acc[tt]);
      }
    }
#pragma unroll
    for (int tt = 0; tt < 4; ++tt) {
      float v = acc[tt];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
      if (lane == 0 && t0 + tt < T) {
        const float lg = bias ? __fadd_rn(v, be) : v;
        logits[size_t(t0 + tt) * E + e] = lg;
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ls_cta0 + 4u * uint32_t((t0 + tt) * E + e)), "f"(lg)
                     : "memory");
      }
    }
  }
  __threadfence();
  cluster_sync_all();
  if (threadIdx.x == 0) QMOE_TRACE_AT(0, 2);
  if (cta != 0) return;

  // ---- CTA 0: selection (the logits are in its shared memory now) ----
  const int nwarps = blockDim.x >> 5;
  for (int t = warp; t < T; t += nwarps) select_topk_warp(ls + t * E, t, E, k, normalize, lane, nullptr, idx_s, w_s, hist);
  __syncthreads();

  // ---- expert offsets and tiles (warp 0), outputs of the selection ----
  const int R = T * k;
  for (int i = threadIdx.x; i < R; i += blockDim.x) {
    topk_idx[i] = idx_s[i];
    topk_w[i] = w_s[i];
  }
  if (warp == 0) {
    for (int i = lane; i < E; i += 32) {
      off_s[i] = hist[i];
      tile_s[i] = (hist[i] + kRouteSmallTileRows - 1) / kRouteSmallTileRows;
    }
    __syncwarp();
    const int total = warp_exclusive_scan_smem(off_s, E, lane);
    const int ntiles = warp_exclusive_scan_smem(tile_s, E, lane);
    __syncwarp();
    int32_t* t_exp = tiles + 1;
    int32_t* t_row0 = t_exp + max_tiles;
    int32_t* t_rows = t_row0 + max_tiles;
    for (int i = lane; i < E; i += 32) {
      counts[i] = hist[i];
      offsets[i] = off_s[i];
      const int nt_e = (hist[i] + kRouteSmallTileRows - 1) / kRouteSmallTileRows;
      for (int j = 0; j < nt_e; ++j) {
        const int ti = tile_s[i] + j;
        if (ti < max_tiles) {
          t_exp[ti] = i;
          t_row0[ti] = off_s[i] + j * kRouteSmallTileRows;
          t_rows[ti] = min(kRouteSmallTileRows, hist[i] - j * kRouteSmallTileRows);
        }
      }
    }
    if (lane == 0) {
      offsets[E] = total;
      tiles[0] = min(ntiles, max_tiles);
    }
  }
  __syncthreads();

  // ---- rows: stable by token inside each expert ----
  for (int p = threadIdx.x; p < R; p += blockDim.x) {
    const int ep = idx_s[p];
    int rank = 0;
    for (int q = 0; q < p; ++q) rank += idx_s[q] == ep;
    const int pos = off_s[ep] + rank;
    row_token[pos] = p / k;
    row_w[pos] = w_s[p];
    slot_row[p] = pos;
  }
  if (threadIdx.x == 0) QMOE_TRACE_AT(0, 3);
}

}  // namespace qmoe
