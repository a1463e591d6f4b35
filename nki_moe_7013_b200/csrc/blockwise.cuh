// NxDI blockwise seam: turns (token_position_to_id, block_to_expert) blocks
// into the row description the grouped GEMMs consume.
//
// Reference semantics (qwen_with_nki.py:5440-5502, 5656-5667): block b holds
// block_size token positions for expert block_to_expert[b]; a position whose
// token id is outside [0, T) is padding (the reference points it at an
// appended zero row); if a token occurs more than once in a block only its
// last occurrence is written by the scatter-add, so it contributes once.  The
// affinity of a position is expert_affinities_masked[token, expert].
#pragma once

#include "common.cuh"

namespace qmoe {

constexpr int kBlockwiseThreads = 512;

__global__ void __launch_bounds__(kBlockwiseThreads)
    blockwise_prepare_kernel(const int32_t* __restrict__ tpi, const int32_t* __restrict__ b2e,
                             const float* __restrict__ aff, int aff_rows,
                             const __nv_bfloat16* __restrict__ x, int T, int H, int E, int B,
                             __nv_bfloat16* __restrict__ x_perm, int32_t* __restrict__ row_dst,
                             float* __restrict__ row_w, int32_t* __restrict__ tiles, int max_tiles) {
  extern __shared__ int bw_smem[];
  int* toks = bw_smem;      // [B]
  int* src = bw_smem + B;   // [B]: gather source token or -1
  const int blk = blockIdx.x;
  const int e = b2e[blk];
  const bool valid_e = e >= 0 && e < E;
  for (int p = threadIdx.x; p < B; p += blockDim.x) toks[p] = tpi[size_t(blk) * B + p];
  __syncthreads();
  for (int p = threadIdx.x; p < B; p += blockDim.x) {
    const int tok = toks[p];
    const bool valid = tok >= 0 && tok < T;
    bool dup = false;
    if (valid)
      for (int q = p + 1; q < B; ++q)
        if (toks[q] == tok) {
          dup = true;
          break;
        }
    const size_t r = size_t(blk) * B + p;
    row_dst[r] = (valid && valid_e && !dup) ? tok : -1;
    row_w[r] = (valid && valid_e && tok < aff_rows) ? aff[size_t(tok) * E + e] : 0.f;
    src[p] = valid ? tok : -1;
  }
  __syncthreads();
  const int vec_per_row = H / 8;
  for (int v = threadIdx.x; v < B * vec_per_row; v += blockDim.x) {
    const int p = v / vec_per_row;
    const int col = (v % vec_per_row) * 8;
    const int tok = src[p];
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (tok >= 0) val = *reinterpret_cast<const uint4*>(x + size_t(tok) * H + col);
    *reinterpret_cast<uint4*>(x_perm + (size_t(blk) * B + p) * H + col) = val;
  }
  const int tpb = (B + 127) / 128;
  if (threadIdx.x < tpb) {
    const int ti = blk * tpb + threadIdx.x;
    if (ti < max_tiles) {
      tiles[1 + ti] = valid_e ? e : 0;
      tiles[1 + max_tiles + ti] = blk * B + threadIdx.x * 128;
      tiles[1 + 2 * max_tiles + ti] = min(128, B - int(threadIdx.x) * 128);
    }
  }
  if (blk == 0 && threadIdx.x == 0) tiles[0] = min(int(gridDim.x) * tpb, max_tiles);
}

}  // namespace qmoe
