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
