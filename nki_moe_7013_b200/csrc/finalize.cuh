// Combine finalisation: out = bf16(acc [+ residual]).  The residual add of the
// decoder layer (qwen.py:430) is folded in so the layer writes its output once.
#pragma once

#include "common.cuh"

namespace qmoe {

__global__ void __launch_bounds__(256)
    combine_finalize_kernel(const float* __restrict__ acc, const __nv_bfloat16* __restrict__ residual,
                            __nv_bfloat16* __restrict__ out, long long n_vec8) {
  if (threadIdx.x == 0) QMOE_TRACE_AT(3, 0);
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x == 0) QMOE_TRACE_AT(3, 1);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_vec8;
       i += (long long)gridDim.x * blockDim.x)
    finalize_vec8(acc, residual, out, i);
  if (threadIdx.x == 0) QMOE_TRACE_AT(3, 2);
}

// Masked residual add of the decoder layer's MoE output (qwen.py:429-430 with
// the block's padding_mask): out[t] = bf16(residual[t] + mask[t] * y[t]),
// computed in fp32 and rounded once; mask NULL = 1, residual NULL = 0.
__global__ void __launch_bounds__(256)
    masked_residual_kernel(const uint4* __restrict__ y, const float* __restrict__ mask,
                           const uint4* __restrict__ residual, uint4* __restrict__ out, int T, int vec_per_row) {
  griddep_wait();
  griddep_launch_dependents();
  const long long total = (long long)T * vec_per_row;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int t = int(i / vec_per_row);
    const float m = mask ? mask[t] : 1.f;
    const uint4 v = y[i];
    const uint32_t yv[4] = {v.x, v.y, v.z, v.w};
    uint32_t rv[4] = {0u, 0u, 0u, 0u};
    if (residual) {
      const uint4 r = residual[i];
      rv[0] = r.x;
      rv[1] = r.y;
      rv[2] = r.z;
      rv[3] = r.w;
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      // multiply, then add, each rounded (no fused multiply-add): the same
      // fp32 value as residual.float() + y.float() * mask
      const float lo = __fadd_rn(bf16lo_to_f32(rv[q]), __fmul_rn(m, bf16lo_to_f32(yv[q])));
      const float hi = __fadd_rn(bf16hi_to_f32(rv[q]), __fmul_rn(m, bf16hi_to_f32(yv[q])));
      const __nv_bfloat162 b2 = __floats2bfloat162_rn(lo, hi);
      ow[q] = *reinterpret_cast<const uint32_t*>(&b2);
    }
    out[i] = o;
  }
}

// Chosen expert affinities of the ExpertMLPs seam (qwen_with_nki.py:2398-2405):
// w[t, j] = affinities[t, idx[t, j]], then (normalize) divided by
// max(sum_j |w[t, j]|, 1e-12) -- F.normalize(p=1) -- summed in slot order.
// One thread per token; an index outside [0, E) gives weight 0 and device
// error 4.
__global__ void __launch_bounds__(256)
    select_affinities_kernel(const float* __restrict__ aff, const int32_t* __restrict__ idx, int T, int E, int k,
                             int normalize, float* __restrict__ w) {
  griddep_wait();
  griddep_launch_dependents();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  float v[32];
  float s = 0.f;
  for (int j = 0; j < k; ++j) {
    const int e = idx[size_t(t) * k + j];
    float a = 0.f;
    if (e < 0 || e >= E)
      record_device_error(kDevErrBadIndex);
    else
      a = aff[size_t(t) * E + e];
    v[j] = a;
    s += fabsf(a);
  }
  const float d = normalize ? fmaxf(s, 1e-12f) : 1.f;
  for (int j = 0; j < k; ++j) w[size_t(t) * k + j] = normalize ? v[j] / d : v[j];
}

// Greedy pick of a decode step (the argmax of the logits the reference's
// generation loop compares, main.py:576, 611): tokens[b] = the first index of
// the largest of logits[b, :] (NaN counts as larger than every number, as
// torch.argmax propagates it), then positions[b] += 1 and lengths[b] += 1
// when given -- the step's bookkeeping in the same launch.  One CTA per row.
__device__ __forceinline__ unsigned long long greedy_key(float f, int v) {
  unsigned int u = __float_as_uint(f);
  unsigned int key;
  if (f != f)
    key = 0xFFFFFFFFu;
  else {
    if (u == 0x80000000u) u = 0u;  // -0 ranks as +0
    key = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  // larger value first, then lower index
  return (static_cast<unsigned long long>(key) << 32) | (0xFFFFFFFFu - static_cast<unsigned int>(v));
}

__global__ void __launch_bounds__(1024)
    greedy_pick_kernel(const __nv_bfloat16* __restrict__ logits, int V, int32_t* __restrict__ tokens,
                       int32_t* __restrict__ positions, int32_t* __restrict__ lengths) {
  __shared__ unsigned long long warp_best[32];
  griddep_wait();
  griddep_launch_dependents();
  const int b = blockIdx.x;
  const __nv_bfloat16* row = logits + size_t(b) * V;
  unsigned long long best = 0ull;
  const bool vec = (V % 8) == 0;
  if (vec) {
    const uint4* r4 = reinterpret_cast<const uint4*>(row);
    for (int i = threadIdx.x; i < V / 8; i += blockDim.x) {
      const uint4 q = r4[i];
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        best = max(best, greedy_key(bf16lo_to_f32(w[j]), 8 * i + 2 * j));
        best = max(best, greedy_key(bf16hi_to_f32(w[j]), 8 * i + 2 * j + 1));
      }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) best = max(best, greedy_key(__bfloat162float(row[i]), i));
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, off));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) warp_best[warp] = best;
  __syncthreads();
  if (warp == 0) {
    best = lane < int(blockDim.x >> 5) ? warp_best[lane] : 0ull;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, off));
    if (lane == 0) {
      tokens[b] = int32_t(0xFFFFFFFFu - static_cast<unsigned int>(best & 0xFFFFFFFFull));
      if (positions) positions[b] += 1;
      if (lengths) lengths[b] += 1;
    }
  }
}

}  // namespace qmoe

namespace qmoe {

// Token embedding lookup (the model's first op; replaces the reference's
// embedding kernel, qwen_with_nki.py:1541-1578): out[i] = table[ids[i]],
// bf16 rows moved as 16-byte vectors.  An id outside [0, V) gives a zero row
// and device error 4.
__global__ void __launch_bounds__(256)
    embedding_gather_kernel(const uint4* __restrict__ table, const int32_t* __restrict__ ids, int n, int V,
                            int vec_per_row, uint4* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  const long long total = (long long)n * vec_per_row;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = int(i / vec_per_row);
    const int c = int(i - (long long)r * vec_per_row);
    const int id = ids[r];
    if (id < 0 || id >= V) {
      if (c == 0) record_device_error(kDevErrBadIndex);
      out[i] = make_uint4(0u, 0u, 0u, 0u);
    } else {
      out[i] = table[(long long)id * vec_per_row + c];
    }
  }
}

}  // namespace qmoe
