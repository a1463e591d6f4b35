// K4: RMSNorm (with the decoder layer's residual add fused in) and the fused
// per-head QK-RMSNorm + RoPE + KV-cache append.
//
// Reference semantics:
//   RMSNorm  y = x * rsqrt(mean(x^2) + eps) * w, fp32 math, one output cast
//            (qwen_with_nki.py:1286-1342; NxDI CustomRMSNorm, qwen.py:236-240).
//   residual the decoder layer adds the sub-layer output to the residual in
//            the activation dtype before the next norm (qwen.py:423, 428).
//   QK-norm  per-head RMSNorm over head_dim on q and k, before RoPE
//            (qwen.py:333-335).
//   RoPE     rotate-half form with theta 1e6 (qwen.py:315-319):
//            out[d]      = x[d]*cos(p*f_d) - x[d+D/2]*sin(p*f_d)
//            out[d+D/2]  = x[d+D/2]*cos(p*f_d) + x[d]*sin(p*f_d),  d < D/2,
//            f_d = inv_freq[d] supplied by the caller in fp32.
#pragma once

#include "common.cuh"

namespace qmoe {

constexpr int kNormThreads = 256;  // 8 rows per CTA, one warp per row

// x (rows, H) bf16 or fp32; residual (rows, H) bf16 or null.  With a
// residual, s = bf16(x + residual) is written to residual_out and normalised.
// One warp per row; lane l handles elements [128c + 4l, 128c + 4l + 4) for
// c < kChunks (kChunks * 128 >= H), all loaded before any is used so a row
// costs one memory round trip; the values stay in registers for the scaling.
template <typename Tin, typename Tout, int kChunks>
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_kernel(const Tin* __restrict__ x, const __nv_bfloat16* __restrict__ residual,
                   const float* __restrict__ w, int rows, int H, float eps, Tout* __restrict__ y,
                   __nv_bfloat16* __restrict__ residual_out) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // the norm weight is a parameter, not written by the previous kernel: its
  // loads go out before the programmatic-launch wait
  float4 wq[kChunks];
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = i * 128 + lane * 4;
    wq[i] = c < H ? *reinterpret_cast<const float4*>(w + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  griddep_wait();
  griddep_launch_dependents();
  const int row = blockIdx.x * (kNormThreads / 32) + warp;
  if (row >= rows) return;
  const Tin* xr = x + size_t(row) * H;
  float v[kChunks][4];
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = i * 128 + lane * 4;
    v[i][0] = v[i][1] = v[i][2] = v[i][3] = 0.f;
    if (c < H) {
      if constexpr (sizeof(Tin) == 4) {
        const float4 a = *reinterpret_cast<const float4*>(xr + c);
        v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
      } else {
        const uint2 a = *reinterpret_cast<const uint2*>(xr + c);
        v[i][0] = bf16lo_to_f32(a.x); v[i][1] = bf16hi_to_f32(a.x);
        v[i][2] = bf16lo_to_f32(a.y); v[i][3] = bf16hi_to_f32(a.y);
      }
    }
  }
  if (residual) {
    uint2 rr[kChunks];
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int c = i * 128 + lane * 4;
      if (c < H) rr[i] = *reinterpret_cast<const uint2*>(residual + size_t(row) * H + c);
    }
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int c = i * 128 + lane * 4;
      if (c < H) {
        const __nv_bfloat162 s0 = __floats2bfloat162_rn(v[i][0] + bf16lo_to_f32(rr[i].x),
                                                        v[i][1] + bf16hi_to_f32(rr[i].x));
        const __nv_bfloat162 s1 = __floats2bfloat162_rn(v[i][2] + bf16lo_to_f32(rr[i].y),
                                                        v[i][3] + bf16hi_to_f32(rr[i].y));
        uint2 o;
        o.x = *reinterpret_cast<const uint32_t*>(&s0);
        o.y = *reinterpret_cast<const uint32_t*>(&s1);
        *reinterpret_cast<uint2*>(residual_out + size_t(row) * H + c) = o;
        v[i][0] = bf16lo_to_f32(o.x); v[i][1] = bf16hi_to_f32(o.x);
        v[i][2] = bf16lo_to_f32(o.y); v[i][3] = bf16hi_to_f32(o.y);
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kChunks; ++i) ss = sumsq4(ss, v[i][0], v[i][1], v[i][2], v[i][3]);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
  const float r = rsqrtf(ss / float(H) + eps);
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = i * 128 + lane * 4;
    if (c >= H) continue;
    const float4 wv = wq[i];
    const float o0 = __fmul_rn(__fmul_rn(v[i][0], r), wv.x), o1 = __fmul_rn(__fmul_rn(v[i][1], r), wv.y),
                o2 = __fmul_rn(__fmul_rn(v[i][2], r), wv.z), o3 = __fmul_rn(__fmul_rn(v[i][3], r), wv.w);
    if constexpr (sizeof(Tout) == 4) {
      *reinterpret_cast<float4*>(y + size_t(row) * H + c) = make_float4(o0, o1, o2, o3);
    } else {
      const __nv_bfloat162 a = __floats2bfloat162_rn(o0, o1);
      const __nv_bfloat162 b = __floats2bfloat162_rn(o2, o3);
      uint2 o;
      o.x = *reinterpret_cast<const uint32_t*>(&a);
      o.y = *reinterpret_cast<const uint32_t*>(&b);
      *reinterpret_cast<uint2*>(y + size_t(row) * H + c) = o;
    }
  }
}

// The same RMSNorm for bf16 rows at prefill sizes (more rows than one
// wave of the kernel above keeps resident): the row stays in registers as
// packed bf16 (its values are bf16 either way, so every sum and product is
// the same as above) and the norm weight is read at use (L1), which keeps
// the kernel near 60 registers -- several CTAs per SM, several rows per
// warp scheduler in flight -- instead of ~190 and one CTA per SM.
template <typename Tout, int kChunks>
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_rows_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ residual,
                        const float* __restrict__ w, int rows, int H, float eps, Tout* __restrict__ y,
                        __nv_bfloat16* __restrict__ residual_out) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  griddep_wait();
  griddep_launch_dependents();
  const int row = blockIdx.x * (kNormThreads / 32) + warp;
  if (row >= rows) return;
  uint2 pv[kChunks];
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = i * 128 + lane * 4;
    pv[i] = c < H ? *reinterpret_cast<const uint2*>(x + size_t(row) * H + c) : make_uint2(0u, 0u);
  }
  if (residual) {
    uint2 rr[kChunks];
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int c = i * 128 + lane * 4;
      if (c < H) rr[i] = *reinterpret_cast<const uint2*>(residual + size_t(row) * H + c);
    }
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int c = i * 128 + lane * 4;
      if (c < H) {
        const __nv_bfloat162 s0 = __floats2bfloat162_rn(bf16lo_to_f32(pv[i].x) + bf16lo_to_f32(rr[i].x),
                                                        bf16hi_to_f32(pv[i].x) + bf16hi_to_f32(rr[i].x));
        const __nv_bfloat162 s1 = __floats2bfloat162_rn(bf16lo_to_f32(pv[i].y) + bf16lo_to_f32(rr[i].y),
                                                        bf16hi_to_f32(pv[i].y) + bf16hi_to_f32(rr[i].y));
        pv[i].x = *reinterpret_cast<const uint32_t*>(&s0);
        pv[i].y = *reinterpret_cast<const uint32_t*>(&s1);
        *reinterpret_cast<uint2*>(residual_out + size_t(row) * H + c) = pv[i];
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kChunks; ++i)
    ss = sumsq4(ss, bf16lo_to_f32(pv[i].x), bf16hi_to_f32(pv[i].x), bf16lo_to_f32(pv[i].y), bf16hi_to_f32(pv[i].y));
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
  const float r = rsqrtf(ss / float(H) + eps);
#pragma unroll
  for (int i = 0; i < kChunks; ++i) {
    const int c = i * 128 + lane * 4;
    if (c >= H) continue;
    const float4 wv = *reinterpret_cast<const float4*>(w + c);
    const float o0 = __fmul_rn(__fmul_rn(bf16lo_to_f32(pv[i].x), r), wv.x),
                o1 = __fmul_rn(__fmul_rn(bf16hi_to_f32(pv[i].x), r), wv.y),
                o2 = __fmul_rn(__fmul_rn(bf16lo_to_f32(pv[i].y), r), wv.z),
                o3 = __fmul_rn(__fmul_rn(bf16hi_to_f32(pv[i].y), r), wv.w);
    if constexpr (sizeof(Tout) == 4) {
      *reinterpret_cast<float4*>(y + size_t(row) * H + c) = make_float4(o0, o1, o2, o3);
    } else {
      const __nv_bfloat162 a = __floats2bfloat162_rn(o0, o1);
      const __nv_bfloat162 b = __floats2bfloat162_rn(o2, o3);
      uint2 o;
      o.x = *reinterpret_cast<const uint32_t*>(&a);
      o.y = *reinterpret_cast<const uint32_t*>(&b);
      *reinterpret_cast<uint2*>(y + size_t(row) * H + c) = o;
    }
    // at most four chunks' weight loads in flight (registers, not latency,
    // bound this kernel's occupancy)
    if ((i & 3) == 3) asm volatile("" ::: "memory");
  }
}

// One CTA of kQkWarps warps per token; warp w takes heads w, w + kQkWarps,
// ... and issues the loads of all of them before any arithmetic (a head row
// is only 256 bytes, so one per warp in flight left the kernel latency-
// bound at prefill sizes).  Heads [0, nh) are query heads, [nh, nh+nkv) key
// heads, [nh+nkv, nh+2nkv) value heads of the fused QKV projection row.
// head_dim is 128: lane l holds dims [4l, 4l+4); the RoPE partner dims
// d +- 64 live in lane l ^ 16.  The token's 64 rotary angles are the same for
// every head, so the CTA's first 64 threads take their sines and cosines once
// into shared memory.
constexpr int kQkHeadDim = 128;
constexpr int kQkWarps = 8;
constexpr int kQkMaxHeadsPerWarp = 16;  // nh + 2 * nkv <= 128

__global__ void __launch_bounds__(256)
    qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ qkv, const int32_t* __restrict__ positions,
                        const int32_t* __restrict__ cache_slot, const float* __restrict__ q_w,
                        const float* __restrict__ k_w, const float* __restrict__ inv_freq, int T, int nh,
                        int nkv, float eps, __nv_bfloat16* __restrict__ q_out,
                        __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                        int max_seq, int n_slots) {
  __shared__ float rope_cos[kQkHeadDim / 2], rope_sin[kQkHeadDim / 2];
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nheads = nh + 2 * nkv;
  const int t = blockIdx.x;
  const int pos = positions[t];
  const int slot = cache_slot ? cache_slot[t] : 0;
  const int row_len = nheads * kQkHeadDim;
  // this warp's head rows, all loads issued first
  uint2 raw[kQkMaxHeadsPerWarp];
#pragma unroll
  for (int j = 0; j < kQkMaxHeadsPerWarp; ++j) {
    const int head = warp + j * kQkWarps;
    if (head < nheads)
      raw[j] = *reinterpret_cast<const uint2*>(qkv + size_t(t) * row_len + head * kQkHeadDim + lane * 4);
  }
  if (threadIdx.x < kQkHeadDim / 2)
    sincosf(float(pos) * inv_freq[threadIdx.x], &rope_sin[threadIdx.x], &rope_cos[threadIdx.x]);
  __syncthreads();
  const bool cache_ok = slot >= 0 && slot < n_slots && pos >= 0 && pos < max_seq;
  if (!cache_ok && threadIdx.x == 0) record_device_error(kDevErrBadIndex);
#pragma unroll
  for (int j = 0; j < kQkMaxHeadsPerWarp; ++j) {
    const int head = warp + j * kQkWarps;
    if (head >= nheads) break;
    float v[4] = {bf16lo_to_f32(raw[j].x), bf16hi_to_f32(raw[j].x), bf16lo_to_f32(raw[j].y),
                  bf16hi_to_f32(raw[j].y)};
    const bool is_v = head >= nh + nkv;
    if (!is_v) {
      const float* nw = head < nh ? q_w : k_w;
      float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
      const float r = rsqrtf(ss / float(kQkHeadDim) + eps);
      const float4 wv = *reinterpret_cast<const float4*>(nw + lane * 4);
      v[0] = v[0] * r * wv.x;
      v[1] = v[1] * r * wv.y;
      v[2] = v[2] * r * wv.z;
      v[3] = v[3] * r * wv.w;
      const bool lower = lane < 16;
      const int fbase = (lane & 15) * 4;  // frequency index of this lane's dims
      float o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float partner = __shfl_xor_sync(0xFFFFFFFFu, v[i], 16);
        const float sn = rope_sin[fbase + i], cs = rope_cos[fbase + i];
        o[i] = lower ? v[i] * cs - partner * sn : v[i] * cs + partner * sn;
      }
      v[0] = o[0]; v[1] = o[1]; v[2] = o[2]; v[3] = o[3];
    }
    const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 out;
    out.x = *reinterpret_cast<const uint32_t*>(&a);
    out.y = *reinterpret_cast<const uint32_t*>(&b);
    if (head < nh) {
      *reinterpret_cast<uint2*>(q_out + (size_t(t) * nh + head) * kQkHeadDim + lane * 4) = out;
    } else if (cache_ok) {
      const int kvh = is_v ? head - nh - nkv : head - nh;
      __nv_bfloat16* cache = is_v ? v_cache : k_cache;
      *reinterpret_cast<uint2*>(cache + ((size_t(slot) * nkv + kvh) * max_seq + pos) * kQkHeadDim + lane * 4) =
          out;
    }
  }
}

}  // namespace qmoe
