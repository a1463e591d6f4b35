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

// One warp per (token, head).  Heads [0, nh) are query heads, [nh, nh+nkv)
// key heads, [nh+nkv, nh+2nkv) value heads of the fused QKV projection row.
// head_dim is 128: lane l holds dims [4l, 4l+4); the RoPE partner dims
// d +- 64 live in lane l ^ 16.
constexpr int kQkHeadDim = 128;

__global__ void __launch_bounds__(256)
    qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ qkv, const int32_t* __restrict__ positions,
                        const int32_t* __restrict__ cache_slot, const float* __restrict__ q_w,
                        const float* __restrict__ k_w, const float* __restrict__ inv_freq, int T, int nh,
                        int nkv, float eps, __nv_bfloat16* __restrict__ q_out,
                        __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                        int max_seq, int n_slots) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int nheads = nh + 2 * nkv;
  if (gw >= T * nheads) return;
  const int t = gw / nheads;
  const int head = gw - t * nheads;
  const int row_len = nheads * kQkHeadDim;
  const uint2 raw = *reinterpret_cast<const uint2*>(qkv + size_t(t) * row_len + head * kQkHeadDim + lane * 4);
  float v[4] = {bf16lo_to_f32(raw.x), bf16hi_to_f32(raw.x), bf16lo_to_f32(raw.y), bf16hi_to_f32(raw.y)};
  const int pos = positions[t];
  const int slot = cache_slot ? cache_slot[t] : 0;
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
      float sn, cs;
      sincosf(float(pos) * inv_freq[fbase + i], &sn, &cs);
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
  } else {
    const int kvh = is_v ? head - nh - nkv : head - nh;
    if (slot < 0 || slot >= n_slots || pos < 0 || pos >= max_seq) {
      record_device_error(kDevErrBadIndex);
      return;
    }
    __nv_bfloat16* cache = is_v ? v_cache : k_cache;
    *reinterpret_cast<uint2*>(cache + ((size_t(slot) * nkv + kvh) * max_seq + pos) * kQkHeadDim + lane * 4) = out;
  }
}

}  // namespace qmoe
