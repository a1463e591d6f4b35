// Decode-row dense projections on the CUDA cores: out (T, N) = x (T, K) . w^T
// for T <= kGemvMaxT token rows.
//
// At a few rows a projection is a matrix-vector product: every weight byte
// is used T times, so the bound is the HBM stream (and, at 16-32 MB per
// projection, its latency), not the tensor cores.  One warp owns one output
// feature n: lane l loads 16-byte pieces l, l+32, l+64, ... of weight row n
// (all KC of them in flight at once, K = 256 * KC) BEFORE the programmatic-
// launch wait -- the weights are not written by the previous kernel, so
// their stream overlaps that kernel's tail -- then stages the T token rows
// (written by the previous kernel) in shared memory, accumulates T fp32 dot
// products (piece order i = 0..KC-1, 8 fused multiply-adds per piece), and
// reduces each over the warp with an xor butterfly (16..1).  The order is
// fixed, so results are run-to-run identical.
//
// Replaces, for decode rows, the tensor-core projection of the QKV and O
// projections (qwen.py:313-341); the LM head (622 MB) stays on the
// tensor-core kernel, which already streams at the HBM rate.
#pragma once

#include "common.cuh"

namespace qmoe {

constexpr int kGemvWarps = 8;  // output features per CTA
// Up to 4 rows: each warp re-reads the staged rows from shared memory for
// every weight piece, so that traffic grows with T; at 8 rows it made the
// projection slower than the tensor-core kernel (+1.9 us each), at 1 row
// 4.9 us faster.
constexpr int kGemvMaxT = 4;

template <int KC, int TT>  // K = 256 * KC; TT = token rows rounded up to 1, 2 or 4
__global__ void __launch_bounds__(kGemvWarps * 32)
    linear_rows_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w, int T, int N,
                       __nv_bfloat16* __restrict__ out) {
  constexpr int K = KC * 256;
  extern __shared__ __align__(16) uint8_t gemv_smem[];
  uint4* xs = reinterpret_cast<uint4*>(gemv_smem);  // [TT][K / 8], rows >= T zero
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * kGemvWarps + warp;
  uint4 wv[KC];
  if (n < N) {
    const uint4* wr = reinterpret_cast<const uint4*>(w + size_t(n) * K);
#pragma unroll
    for (int i = 0; i < KC; ++i) wv[i] = __ldg(wr + lane + 32 * i);
  }
  griddep_wait();
  griddep_launch_dependents();
  {
    const uint4* src = reinterpret_cast<const uint4*>(x);
    const int nv = T * (K / 8);
    for (int i = threadIdx.x; i < TT * (K / 8); i += blockDim.x) xs[i] = i < nv ? src[i] : make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
  if (n >= N) return;
  float acc[TT];
#pragma unroll
  for (int t = 0; t < TT; ++t) acc[t] = 0.f;
#pragma unroll
  for (int i = 0; i < KC; ++i) {
    const float wf[8] = {bf16lo_to_f32(wv[i].x), bf16hi_to_f32(wv[i].x), bf16lo_to_f32(wv[i].y),
                         bf16hi_to_f32(wv[i].y), bf16lo_to_f32(wv[i].z), bf16hi_to_f32(wv[i].z),
                         bf16lo_to_f32(wv[i].w), bf16hi_to_f32(wv[i].w)};
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      const uint4 xv = xs[t * (K / 8) + lane + 32 * i];
      acc[t] = fmaf(bf16lo_to_f32(xv.x), wf[0], acc[t]);
      acc[t] = fmaf(bf16hi_to_f32(xv.x), wf[1], acc[t]);
      acc[t] = fmaf(bf16lo_to_f32(xv.y), wf[2], acc[t]);
      acc[t] = fmaf(bf16hi_to_f32(xv.y), wf[3], acc[t]);
      acc[t] = fmaf(bf16lo_to_f32(xv.z), wf[4], acc[t]);
      acc[t] = fmaf(bf16hi_to_f32(xv.z), wf[5], acc[t]);
      acc[t] = fmaf(bf16lo_to_f32(xv.w), wf[6], acc[t]);
      acc[t] = fmaf(bf16hi_to_f32(xv.w), wf[7], acc[t]);
    }
  }
  float mine = 0.f;  // lane t keeps row t's sum
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    float v = acc[t];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
    if (lane == t) mine = v;
  }
  if (lane < T) out[size_t(lane) * N + n] = __float2bfloat16_rn(mine);
}

// ---------------------------------------------------------------------------
// Expert GEMMs of a 1-2 token decode step on the CUDA cores.
//
// At one or two tokens each routed expert sees one or two rows, so its
// gate/up and down projections are matrix-vector products: 75 MB of weights
// (8 experts at Qwen3-30B-A3B shapes) read once.  The routing kernels'
// 128-row tile list (expert, first permuted row, rows) drives both kernels;
// an expert gets at most T rows, so a tile holds at most kExpertRowsMaxT.
// Both kernels are persistent (two CTAs per SM): a CTA stages the tile list,
// the rows' tokens and weights, and the token or activation rows in shared
// memory once, then each warp walks its work items, so the only memory
// round trip left per item is its weight stream.
//
//   gate/up  item = (tile, intermediate feature i): the gate and up rows i
//            of the tile's expert; act[row][i] = bf16(silu(g) * u) with
//            silu(g) = g / (1 + exp(-g)) as in the tensor-core epilogue
//            (the SwiGLU of qwen_with_nki.py:5341-5369).
//   down     item = output feature h: for each token, the sum over tiles in
//            tile order (ascending expert) of row_w * (w_down[e][h] . act),
//            plus the residual, written as bf16 -- the weighted combine and
//            its finalisation (qwen_with_nki.py:4967-5040, qwen.py:430)
//            without an fp32 accumulator or atomics, so the result is
//            run-to-run identical.
// Tiles whose expert, rows, first row or tokens fall outside their limits
// are skipped and recorded as device error kDevErrBadIndex.
// ---------------------------------------------------------------------------
constexpr int kExpertRowsMaxT = 2;
constexpr int kExpertRowsMaxR = 64;       // permuted rows (T * k)
constexpr int kExpertRowsMaxTiles = 64;   // every tile has a row: at most R tiles
// tiles whose weight rows a warp loads together (register budget of two
// CTAs per SM)
__host__ __device__ constexpr int down_tile_group(int IC) { return IC >= 3 ? 4 : 8; }

__device__ __forceinline__ float dot8_bf16(const uint4 a, const uint4 b, float acc) {
  acc = fmaf(bf16lo_to_f32(a.x), bf16lo_to_f32(b.x), acc);
  acc = fmaf(bf16hi_to_f32(a.x), bf16hi_to_f32(b.x), acc);
  acc = fmaf(bf16lo_to_f32(a.y), bf16lo_to_f32(b.y), acc);
  acc = fmaf(bf16hi_to_f32(a.y), bf16hi_to_f32(b.y), acc);
  acc = fmaf(bf16lo_to_f32(a.z), bf16lo_to_f32(b.z), acc);
  acc = fmaf(bf16hi_to_f32(a.z), bf16hi_to_f32(b.z), acc);
  acc = fmaf(bf16lo_to_f32(a.w), bf16lo_to_f32(b.w), acc);
  acc = fmaf(bf16hi_to_f32(a.w), bf16hi_to_f32(b.w), acc);
  return acc;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
  return v;
}

// The tile list, rows' tokens and rows' weights in shared memory, checked:
// meta[t] = {expert, first row, rows (0: skip), 0}; tok[r] in [0, T) or -1.
// Returns the tile count.  All threads of the CTA take part; ends with a
// CTA barrier.
__device__ __forceinline__ int stage_expert_tiles(const int32_t* __restrict__ tiles, int max_tiles,
                                                  const int32_t* __restrict__ row_token,
                                                  const float* __restrict__ row_w, int R, int E, int T,
                                                  int4* meta, int* tok, float* rw) {
  const int nt = min(min(tiles[0], max_tiles), kExpertRowsMaxTiles);
  for (int t = threadIdx.x; t < nt; t += blockDim.x) {
    int4 m = make_int4(tiles[1 + t], tiles[1 + max_tiles + t], tiles[1 + 2 * max_tiles + t], 0);
    if (m.x < 0 || m.x >= E || m.z < 1 || m.z > kExpertRowsMaxT || m.y < 0 || m.y > R - m.z) {
      record_device_error(kDevErrBadIndex);
      m.z = 0;
    }
    meta[t] = m;
  }
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const int tk = row_token[r];
    tok[r] = (tk >= 0 && tk < T) ? tk : -1;
    if (rw) rw[r] = row_w[r];
  }
  __syncthreads();
  return nt;
}

template <int KC>  // H = 256 * KC
__global__ void __launch_bounds__(kGemvWarps * 32, 2)
    expert_gateup_rows_kernel(const __nv_bfloat16* __restrict__ x, const int32_t* __restrict__ row_token,
                              const __nv_bfloat16* __restrict__ w_gate_up, const int32_t* __restrict__ tiles,
                              int max_tiles, int R, int I, int E, int T, __nv_bfloat16* __restrict__ act) {
  constexpr int H = KC * 256;
  __shared__ uint4 xs[kExpertRowsMaxT * (H / 8)];
  __shared__ int4 meta[kExpertRowsMaxTiles];
  __shared__ int tok[kExpertRowsMaxR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_wait();
  griddep_launch_dependents();
  for (int v = threadIdx.x; v < T * (H / 8); v += blockDim.x) xs[v] = reinterpret_cast<const uint4*>(x)[v];
  const int nt = stage_expert_tiles(tiles, max_tiles, row_token, nullptr, R, E, T, meta, tok, nullptr);
  const int items = nt * I;
  const int stride = gridDim.x * kGemvWarps;
  for (int u = blockIdx.x * kGemvWarps + warp; u < items; u += stride) {
    const int t = u / I, i = u - t * I;
    const int4 m = meta[t];
    if (m.z == 0) continue;
    const uint4* gr = reinterpret_cast<const uint4*>(w_gate_up + (size_t(m.x) * 2 * I + i) * H);
    const uint4* ur = reinterpret_cast<const uint4*>(w_gate_up + (size_t(m.x) * 2 * I + I + i) * H);
    uint4 gv[KC], uv[KC];
#pragma unroll
    for (int k = 0; k < KC; ++k) {
      gv[k] = __ldg(gr + lane + 32 * k);
      uv[k] = __ldg(ur + lane + 32 * k);
    }
    // the tile's (at most two) rows side by side, piece by piece
    const int tk0 = tok[m.y];
    const int tk1 = m.z > 1 ? tok[m.y + 1] : -1;
    const uint4* x0 = xs + max(tk0, 0) * (H / 8) + lane;
    const uint4* x1 = xs + max(tk1, 0) * (H / 8) + lane;
    float g0 = 0.f, u0 = 0.f, g1 = 0.f, u1 = 0.f;
#pragma unroll
    for (int k = 0; k < KC; ++k) {
      const uint4 xa = x0[32 * k];
      g0 = dot8_bf16(gv[k], xa, g0);
      u0 = dot8_bf16(uv[k], xa, u0);
      if (m.z > 1) {
        const uint4 xb = x1[32 * k];
        g1 = dot8_bf16(gv[k], xb, g1);
        u1 = dot8_bf16(uv[k], xb, u1);
      }
    }
    g0 = warp_sum(g0);
    u0 = warp_sum(u0);
    if (lane == 0 && tk0 >= 0) act[size_t(m.y) * I + i] = __float2bfloat16_rn(g0 / (1.0f + __expf(-g0)) * u0);
    if (m.z > 1) {
      g1 = warp_sum(g1);
      u1 = warp_sum(u1);
      if (lane == 0 && tk1 >= 0) act[size_t(m.y + 1) * I + i] = __float2bfloat16_rn(g1 / (1.0f + __expf(-g1)) * u1);
    }
  }
}

template <int IC>  // I = 256 * IC
__global__ void __launch_bounds__(kGemvWarps * 32, 2)
    expert_down_rows_kernel(const __nv_bfloat16* __restrict__ act, const __nv_bfloat16* __restrict__ w_down,
                            const int32_t* __restrict__ tiles, int max_tiles, const int32_t* __restrict__ row_token,
                            const float* __restrict__ row_w, int R, int H, int E, int T,
                            const __nv_bfloat16* __restrict__ residual, __nv_bfloat16* __restrict__ out) {
  constexpr int I = IC * 256;
  extern __shared__ __align__(16) uint8_t down_rows_smem[];
  uint4* as = reinterpret_cast<uint4*>(down_rows_smem);  // [R][I / 8]
  __shared__ int4 meta[kExpertRowsMaxTiles];
  __shared__ int tok[kExpertRowsMaxR];
  __shared__ float rw[kExpertRowsMaxR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_wait();
  griddep_launch_dependents();
  for (int v = threadIdx.x; v < R * (I / 8); v += blockDim.x) as[v] = reinterpret_cast<const uint4*>(act)[v];
  const int nt = stage_expert_tiles(tiles, max_tiles, row_token, row_w, R, E, T, meta, tok, rw);
  for (int h = blockIdx.x * kGemvWarps + warp; h < H; h += gridDim.x * kGemvWarps) {
    float s0 = 0.f, s1 = 0.f;  // tokens 0 and 1
    constexpr int kGroup = down_tile_group(IC);
    for (int t0 = 0; t0 < nt; t0 += kGroup) {
      uint4 wv[kGroup][IC];
#pragma unroll
      for (int j = 0; j < kGroup; ++j) {
        if (t0 + j < nt && meta[t0 + j].z) {
          const uint4* wr = reinterpret_cast<const uint4*>(w_down + (size_t(meta[t0 + j].x) * H + h) * I);
#pragma unroll
          for (int k = 0; k < IC; ++k) wv[j][k] = __ldg(wr + lane + 32 * k);
        }
      }
#pragma unroll
      for (int j = 0; j < kGroup; ++j) {
        if (t0 + j >= nt) break;
        const int4 m = meta[t0 + j];
        for (int r = 0; r < m.z; ++r) {
          const int row = m.y + r;
          float d = 0.f;
#pragma unroll
          for (int k = 0; k < IC; ++k) d = dot8_bf16(wv[j][k], as[row * (I / 8) + lane + 32 * k], d);
          d = warp_sum(d);
          const float c = rw[row] * d;
          if (tok[row] == 0) s0 += c;
          else if (tok[row] == 1) s1 += c;
        }
      }
    }
    if (lane < T) {
      float v = lane == 0 ? s0 : s1;
      if (residual) v += __bfloat162float(residual[size_t(lane) * H + h]);
      out[size_t(lane) * H + h] = __float2bfloat16_rn(v);
    }
  }
}

}  // namespace qmoe
