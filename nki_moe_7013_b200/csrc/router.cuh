// K1: fused router -- fp32 logits in a fixed reduction order, softmax,
// warp-shuffle top-k (ties -> lower expert index), L1 renormalisation, and the
// per-chunk expert histogram that the permutation consumes.
//
// Reference semantics: qwen.py:260-269 (fp32 router, softmax,
// normalize_top_k_affinities), qwen_with_nki.py:2398-2405 (affinity gather,
// F.normalize(p=1)).
//
// Canonical logit order (restated exactly by the CPU oracle, so logits and
// expert indices are bit-exact): H is cut into 256-element groups; lane l of a
// warp owns elements [8l, 8l+8) of every group and accumulates them
// group-major from +0.0f with fmaf (bf16*bf16 products are exact in fp32, so
// each step rounds once); the 32 lane sums are folded by an xor butterfly
// (16, 8, 4, 2, 1).
#pragma once

#include "common.cuh"

namespace qmoe {

constexpr int kRouterChunk = QMOE_ROUTER_CHUNK;  // tokens per CTA (= histogram chunk)
constexpr int kRouterTE = 4;                       // experts per register tile
// Warps per router CTA: 16 (two 4-expert tiles each for E=128) keeps enough
// warps resident to hide the L2 latency of the weight stream; H = 4096 uses 8
// so its larger register footprint fits.  Batches of more chunks than SMs
// use 8-warp CTAs, two per SM: one CTA's staging and top-k phases (half its
// warps idle) then overlap the other's logit FMAs.
template <int G>
constexpr int router_warps() { return G >= 16 ? 8 : 16; }
template <int G, int kWarps>
constexpr int router_ctas_per_sm() { return (G < 16 && kWarps == 8) ? 2 : 1; }
static_assert(kRouterChunk * kRouterTE == 32, "one reduced chain per lane");

// Sums v[0..31] of every lane across the warp; returns in lane l the total of
// chain l.  Step s exchanges half of the remaining chains with lane ^ (16>>s).
__device__ __forceinline__ float warp_reduce_32_chains(const float* v, int lane) {
  float a[16];
  {
    const bool hi = lane & 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float keep = hi ? v[i + 16] : v[i];
      const float send = hi ? v[i] : v[i + 16];
      a[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, 16);
    }
  }
  {
    const bool hi = lane & 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float keep = hi ? a[i + 8] : a[i];
      const float send = hi ? a[i] : a[i + 8];
      a[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, 8);
    }
  }
  {
    const bool hi = lane & 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float keep = hi ? a[i + 4] : a[i];
      const float send = hi ? a[i] : a[i + 4];
      a[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, 4);
    }
  }
  {
    const bool hi = lane & 2;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float keep = hi ? a[i + 2] : a[i];
      const float send = hi ? a[i] : a[i + 2];
      a[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, 2);
    }
  }
  const bool hi = lane & 1;
  const float keep = hi ? a[1] : a[0];
  const float send = hi ? a[0] : a[1];
  return keep + __shfl_xor_sync(0xFFFFFFFFu, send, 1);
}
// Softmax over one token's E logits (`row`), top-k by logit (ties -> lower
// expert index), L1 renormalisation of the picked probabilities; one warp.
// Writes topk_idx/topk_w of token `tok`, optional logits, and counts the picks
// into the shared histogram `hist`.
// Order-preserving map of a finite float to an unsigned key (larger float ->
// larger key; -0.0 maps like +0.0, as the float comparison treats them).
__device__ __forceinline__ unsigned int float_order_key(float f) {
  unsigned int u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float float_from_order_key(unsigned int key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

__device__ __forceinline__ void select_topk_warp(const float* row, int tok, int E, int k, int normalize,
                                                 int lane, float* __restrict__ logits_out,
                                                 int32_t* __restrict__ topk_idx,
                                                 float* __restrict__ topk_w, int* hist) {
  const int per_lane = E / 32;  // <= 8
  float lv[8];
  unsigned int key[8];  // 0: no expert in this slot (below every finite logit's key)
  unsigned int kmax = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    lv[i] = (i < per_lane) ? row[lane + 32 * i] : -INFINITY;
    key[i] = (i < per_lane) ? float_order_key(lv[i]) : 0u;
    kmax = max(kmax, key[i]);
  }
  const float m = float_from_order_key(__reduce_max_sync(0xFFFFFFFFu, kmax));
  float ex[8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ex[i] = (i < per_lane) ? expf(lv[i] - m) : 0.f;
    s += ex[i];
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, off);
  const float inv_s = 1.0f / s;
  if (logits_out) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < per_lane) logits_out[size_t(tok) * E + lane + 32 * i] = lv[i];
  }
  // k rounds: the largest remaining logit (warp max of the keys), then the
  // lowest expert index holding it (warp min) -- ties go to the lower index.
  // A chosen expert's key is cleared to 0.
  float chosen_p = 0.f;  // lane j (< k) keeps the probability of pick j
  int chosen_e = 0;
  for (int j = 0; j < k; ++j) {
    unsigned int lk = 0u;
#pragma unroll
    for (int i = 0; i < 8; ++i) lk = max(lk, key[i]);
    const unsigned int bk = __reduce_max_sync(0xFFFFFFFFu, lk);
    int li = 0x7FFFFFFF;
#pragma unroll
    for (int i = 7; i >= 0; --i)
      if (key[i] == bk && bk != 0u) li = lane + 32 * i;
    const int be = __reduce_min_sync(0xFFFFFFFFu, li);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (lane + 32 * i == be) key[i] = 0u;
    const int owner = be & 31;
    float mine = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (lane + 32 * i == be) mine = ex[i] * inv_s;
    const float p = __shfl_sync(0xFFFFFFFFu, mine, owner);
    if (lane == j) {
      chosen_p = p;
      chosen_e = be;
    }
  }
  float denom = 0.f;
  for (int j = 0; j < k; ++j) denom += __shfl_sync(0xFFFFFFFFu, chosen_p, j);
  if (lane < k) {
    const float wv = normalize ? chosen_p / fmaxf(denom, 1e-12f) : chosen_p;
    topk_idx[size_t(tok) * k + lane] = chosen_e;
    topk_w[size_t(tok) * k + lane] = wv;
    atomicAdd(&hist[chosen_e], 1);
  }
}

// The router for one chunk of kRouterChunk tokens (kWarps warps): fp32
// logits in the canonical order, softmax, top-k, renormalisation; writes
// topk_idx / topk_w (and logits_out) of its tokens and leaves the chunk's
// expert histogram in hist[0, E) (shared), synchronised.  xs: kRouterChunk*H
// floats and ls: kRouterChunk*E floats of shared memory.
template <int G, int kWarps>
__device__ __forceinline__ void router_chunk(int chunk, const __nv_bfloat16* __restrict__ x,
                                             const __nv_bfloat16* __restrict__ w, const float* __restrict__ bias,
                                             int T, int E, int k, int normalize, float* __restrict__ logits_out,
                                             int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, float* xs,
                                             float* ls, int* hist) {
  constexpr int H = G * 256;
  constexpr int kThreads = kWarps * 32;
  static_assert(kRouterChunk <= kWarps, "one warp per token in the top-k phase");
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int t0 = chunk * kRouterChunk;
  const int nt = min(kRouterChunk, T - t0);

  // Stage the chunk's activations in shared memory as fp32.  Inside each
  // 256-element group, element 8l+q is stored at (q/4)*128 + 4l + q%4 so the
  // two float4 reads of a lane's slice are conflict-free across the warp.
  for (int i = threadIdx.x; i < kRouterChunk * (H / 8); i += kThreads) {
    const int t = i / (H / 8);
    const int c = (i % (H / 8)) * 8;
    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
    if (t < nt) {
      const uint4 v = *reinterpret_cast<const uint4*>(x + size_t(t0 + t) * H + c);
      lo = make_float4(bf16lo_to_f32(v.x), bf16hi_to_f32(v.x), bf16lo_to_f32(v.y),
                       bf16hi_to_f32(v.y));
      hi = make_float4(bf16lo_to_f32(v.z), bf16hi_to_f32(v.z), bf16lo_to_f32(v.w),
                       bf16hi_to_f32(v.w));
    }
    const int gbase = t * H + (c & ~255);
    const int sl = (c & 255) >> 3;  // lane slot inside the group
    *reinterpret_cast<float4*>(xs + gbase + 4 * sl) = lo;
    *reinterpret_cast<float4*>(xs + gbase + 128 + 4 * sl) = hi;
  }
  for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
  __syncthreads();

  // Logits.  Experts are taken four at a time (tile i = experts 4i..4i+3,
  // tiles dealt round-robin to the warps) for all 8 tokens of the chunk: 32
  // independent fp32 chains per lane (token t x expert j), each accumulating
  // the lane's canonical slice group-major.  Weights stream from L2 one group
  // ahead; activations come from shared memory.
  for (int tile = warp; tile < E / kRouterTE; tile += kWarps) {
    const int e0 = tile * kRouterTE;
    const __nv_bfloat16* wp = w + size_t(e0) * H + 8 * lane;
    float acc[kRouterChunk][kRouterTE];
#pragma unroll
    for (int t = 0; t < kRouterChunk; ++t)
#pragma unroll
      for (int j = 0; j < kRouterTE; ++j) acc[t][j] = 0.f;
    uint4 wv[kRouterTE];
#pragma unroll
    for (int j = 0; j < kRouterTE; ++j)
      wv[j] = __ldg(reinterpret_cast<const uint4*>(wp + size_t(j) * H));
#pragma unroll
    for (int g = 0; g < G; ++g) {
      uint4 wn[kRouterTE];
      if (g + 1 < G) {
#pragma unroll
        for (int j = 0; j < kRouterTE; ++j)
          wn[j] = __ldg(reinterpret_cast<const uint4*>(wp + size_t(j) * H + 256 * (g + 1)));
      }
      float wf[kRouterTE][8];
#pragma unroll
      for (int j = 0; j < kRouterTE; ++j) {
        wf[j][0] = bf16lo_to_f32(wv[j].x);
        wf[j][1] = bf16hi_to_f32(wv[j].x);
        wf[j][2] = bf16lo_to_f32(wv[j].y);
        wf[j][3] = bf16hi_to_f32(wv[j].y);
        wf[j][4] = bf16lo_to_f32(wv[j].z);
        wf[j][5] = bf16hi_to_f32(wv[j].z);
        wf[j][6] = bf16lo_to_f32(wv[j].w);
        wf[j][7] = bf16hi_to_f32(wv[j].w);
      }
#pragma unroll
      for (int t = 0; t < kRouterChunk; ++t) {
        const float* xr = xs + t * H + 256 * g + 4 * lane;
        const float4 a = *reinterpret_cast<const float4*>(xr);
        const float4 b = *reinterpret_cast<const float4*>(xr + 128);
        const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int q = 0; q < 8; ++q)
#pragma unroll
          for (int j = 0; j < kRouterTE; ++j) acc[t][j] = fmaf(xv[q], wf[j][q], acc[t][j]);
      }
      if (g + 1 < G) {
#pragma unroll
        for (int j = 0; j < kRouterTE; ++j) wv[j] = wn[j];
      }
    }
    // Cross-lane sum of the 32 chains by recursive halving.  Every partial
    // sum formed here is the same pairwise sum the xor butterfly forms (fp32
    // addition commutes), so the result is bit-identical to the butterfly;
    // it ends with chain index v = lane in lane `lane`.
    const float v = warp_reduce_32_chains(&acc[0][0], lane);
    const int t = lane / kRouterTE;
    const int e = e0 + lane % kRouterTE;
    if (t < nt) ls[t * E + e] = bias ? __fadd_rn(v, bias[e]) : v;
  }
  __syncthreads();

  // Softmax + top-k: one warp per token.
  const int t = warp;
  if (t < nt) select_topk_warp(ls + t * E, t0 + t, E, k, normalize, lane, logits_out, topk_idx, topk_w, hist);
  __syncthreads();
}

template <int G, int kWarps = router_warps<G>()>  // G = H / 256
__global__ void __launch_bounds__(kWarps * 32, router_ctas_per_sm<G, kWarps>())
    router_topk_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                       const float* __restrict__ bias, int T, int E, int k, int normalize,
                       float* __restrict__ logits_out, int32_t* __restrict__ topk_idx,
                       float* __restrict__ topk_w, int32_t* __restrict__ chunk_hist) {
  extern __shared__ __align__(16) float router_smem[];
  __shared__ int hist[256];
  if (threadIdx.x == 0) QMOE_TRACE_AT(0, 0);
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x == 0) QMOE_TRACE_AT(0, 1);
  router_chunk<G, kWarps>(blockIdx.x, x, w, bias, T, E, k, normalize, logits_out, topk_idx, topk_w, router_smem,
                          router_smem + kRouterChunk * G * 256, hist);
  if (chunk_hist)
    for (int e = threadIdx.x; e < E; e += kWarps * 32) chunk_hist[size_t(blockIdx.x) * E + e] = hist[e];
  if (threadIdx.x == 0) QMOE_TRACE_AT(0, 3);
}

// ---------------------------------------------------------------------------
// Small batches (decode): the fused kernel above would run on ceil(T/8) CTAs
// only.  Here each warp owns ONE expert for a chunk of 8 tokens: the lane's
// whole canonical weight slice is loaded at once (one L2 round trip), the 8
// token chains run interleaved, and the logits go to global memory; grid =
// (E/8 expert groups, ceil(T/8) chunks).  router_select_kernel then applies
// softmax / top-k / renormalisation per token.  Same reduction order as the
// fused kernel, so the logits are bit-identical.
// ---------------------------------------------------------------------------
constexpr int kRouterSmallWarps = 8;

template <int G>
__global__ void __launch_bounds__(kRouterSmallWarps * 32)
    router_logits_small_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                               const float* __restrict__ bias, int T, int E, float* __restrict__ logits) {
  constexpr int H = G * 256;
  extern __shared__ __align__(16) float router_small_smem[];
  float* xs = router_small_smem;  // [8][H], interleaved like the fused kernel
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.y * kRouterChunk;
  const int nt = min(kRouterChunk, T - t0);
  const int e = blockIdx.x * kRouterSmallWarps + warp;
  griddep_wait();
  griddep_launch_dependents();
  // weight slice first: its loads overlap the activation staging
  uint4 wv[G];
  if (e < E) {
#pragma unroll
    for (int g = 0; g < G; ++g)
      wv[g] = __ldg(reinterpret_cast<const uint4*>(w + size_t(e) * H + 256 * g + 8 * lane));
  }
  for (int i = threadIdx.x; i < kRouterChunk * (H / 8); i += kRouterSmallWarps * 32) {
    const int t = i / (H / 8);
    const int c = (i % (H / 8)) * 8;
    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
    if (t < nt) {
      const uint4 v = *reinterpret_cast<const uint4*>(x + size_t(t0 + t) * H + c);
      lo = make_float4(bf16lo_to_f32(v.x), bf16hi_to_f32(v.x), bf16lo_to_f32(v.y), bf16hi_to_f32(v.y));
      hi = make_float4(bf16lo_to_f32(v.z), bf16hi_to_f32(v.z), bf16lo_to_f32(v.w), bf16hi_to_f32(v.w));
    }
    const int gbase = t * H + (c & ~255);
    const int sl = (c & 255) >> 3;
    *reinterpret_cast<float4*>(xs + gbase + 4 * sl) = lo;
    *reinterpret_cast<float4*>(xs + gbase + 128 + 4 * sl) = hi;
  }
  __syncthreads();
  if (e >= E) return;
  float acc[kRouterChunk];
#pragma unroll
  for (int t = 0; t < kRouterChunk; ++t) acc[t] = 0.f;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float wf[8] = {bf16lo_to_f32(wv[g].x), bf16hi_to_f32(wv[g].x), bf16lo_to_f32(wv[g].y),
                         bf16hi_to_f32(wv[g].y), bf16lo_to_f32(wv[g].z), bf16hi_to_f32(wv[g].z),
                         bf16lo_to_f32(wv[g].w), bf16hi_to_f32(wv[g].w)};
#pragma unroll
    for (int t = 0; t < kRouterChunk; ++t) {
      const float* xr = xs + t * H + 256 * g + 4 * lane;
      const float4 a = *reinterpret_cast<const float4*>(xr);
      const float4 b = *reinterpret_cast<const float4*>(xr + 128);
      acc[t] = fmaf(a.x, wf[0], acc[t]);
      acc[t] = fmaf(a.y, wf[1], acc[t]);
      acc[t] = fmaf(a.z, wf[2], acc[t]);
      acc[t] = fmaf(a.w, wf[3], acc[t]);
      acc[t] = fmaf(b.x, wf[4], acc[t]);
      acc[t] = fmaf(b.y, wf[5], acc[t]);
      acc[t] = fmaf(b.z, wf[6], acc[t]);
      acc[t] = fmaf(b.w, wf[7], acc[t]);
    }
  }
  const float be = bias ? bias[e] : 0.f;
#pragma unroll
  for (int t = 0; t < kRouterChunk; ++t) {
    float v = acc[t];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
    if (lane == 0 && t < nt) logits[size_t(t0 + t) * E + e] = bias ? __fadd_rn(v, be) : v;
  }
}

// Softmax / top-k / renorm / chunk histogram from precomputed logits; one CTA
// per chunk of 8 tokens, one warp per token.
__global__ void __launch_bounds__(kRouterChunk * 32)
    router_select_kernel(const float* __restrict__ logits, int T, int E, int k, int normalize,
                         int32_t* __restrict__ topk_idx, float* __restrict__ topk_w,
                         int32_t* __restrict__ chunk_hist) {
  __shared__ int hist[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
  griddep_wait();
  griddep_launch_dependents();
  __syncthreads();
  const int t0 = blockIdx.x * kRouterChunk;
  const int t = t0 + warp;
  if (t < T) select_topk_warp(logits + size_t(t) * E, t, E, k, normalize, lane, nullptr, topk_idx, topk_w, hist);
  if (chunk_hist) {
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_hist[size_t(blockIdx.x) * E + e] = hist[e];
  }
}

}  // namespace qmoe
