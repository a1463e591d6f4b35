// K5 decode: split-KV flash-decode GQA attention over a KV cache, head_dim
// 128, bf16 in / fp32 softmax and accumulation.  (The prefill kernel is the
// tcgen05 one in flash_prefill.cuh.)
//
// Reference semantics: NxDI NeuronAttentionBase with GQA (qwen.py:313-341),
// i.e. out_h = softmax(q_h K_g^T / sqrt(D)) V_g, g = h / (nh / nkv), over
// cache positions kv_start[b] .. kv_len[b]-1 of sequence b (kv_start: left
// padding, 0 without it).
//
// Decode reads each cache byte once and is bound by HBM: the warp-level bf16
// MMA (m16n8k16, fp32 accumulate) on tiles staged in shared memory with
// cp.async and read with ldmatrix is enough for its 8 query rows per KV
// head; rows are padded to 136 elements so ldmatrix is bank-conflict free.
//
// KV cache layout: (slots, nkv, max_seq, 128) bf16 for K and for V.
#pragma once

#include "common.cuh"

namespace qmoe {

constexpr int kAttnD = 128;
constexpr int kAttnPad = kAttnD + 8;   // smem row stride in elements (272 B)
constexpr int kAttnThreads = 128;      // 4 warps
constexpr int kAttnBK = 64;            // keys per smem tile

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* smem_row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(smem_row)));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* smem_row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(smem_row)));
}

// 16-byte async copy; copies zeros when !valid (the source address is only
// used when valid).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16u : 0u)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Stage rows [key0, key0+64) of one (slot, kv head) of a cache into smem;
// rows >= n_valid are zero-filled.
__device__ __forceinline__ void load_kv_tile(__nv_bfloat16* dst, const __nv_bfloat16* src_head, int key0,
                                             int n_valid) {
  // 64 rows x 16 chunks of 16 bytes = 1024 copies, 8 per thread
  for (int i = threadIdx.x; i < kAttnBK * 16; i += kAttnThreads) {
    const int r = i >> 4;
    const int c = (i & 15) * 8;
    const int key = key0 + r;
    const bool ok = key < n_valid;
    cp_async16(dst + r * kAttnPad + c, src_head + size_t(ok ? key : 0) * kAttnD + c, ok);
  }
}

// Online-softmax update of one warp's 16 rows with a new S tile (already
// scaled to log2 units and masked with -inf).  Rows g and g+8 of the lane.
__device__ __forceinline__ void softmax_update(float (&s)[8][4], float (&m)[2], float (&l)[2],
                                               float (&o)[16][4]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) mx = fmaxf(mx, fmaxf(s[nt][2 * h], s[nt][2 * h + 1]));
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
    const float m_new = fmaxf(m[h], mx);
    const float base = m_new == -INFINITY ? 0.f : m_new;
    const float alpha = exp2f(m[h] - base);  // m[h] == -inf -> 0
    l[h] *= alpha;
#pragma unroll
    for (int dn = 0; dn < 16; ++dn) {
      o[dn][2 * h] *= alpha;
      o[dn][2 * h + 1] *= alpha;
    }
    float sum = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][2 * h] = exp2f(s[nt][2 * h] - base);
      s[nt][2 * h + 1] = exp2f(s[nt][2 * h + 1] - base);
      sum += s[nt][2 * h] + s[nt][2 * h + 1];
    }
    l[h] += sum;
    m[h] = m_new;
  }
}

// ---------------------------------------------------------------------------
// Decode, split-KV: grid (nsplit, nkv, B); each CTA takes the 8 query heads
// of one KV head (MMA rows 0..7; rows 8..15 are zero) over keys
// [split*chunk, (split+1)*chunk) of that sequence.  Each warp handles 16-key
// slices of each 64-key smem tile; the four warps are merged in shared
// memory, and the partial (m, l, O) of the split goes to global memory for
// attn_decode_combine_kernel.
// ---------------------------------------------------------------------------
constexpr int kDecodeGroup = 8;  // query heads per KV head handled per CTA (nh / nkv)

__device__ __forceinline__ void qk_slice16(float (&s)[2][4], const uint32_t (&qa)[8][4],
                                           const __nv_bfloat16* ks16, int lane) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) s[nt][i] = 0.f;
  const int mi = lane >> 3, r = lane & 7;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int kk = 0; kk < 8; kk += 2) {
      uint32_t b[4];
      ldsm_x4(b, ks16 + (nt * 8 + r) * kAttnPad + kk * 16 + mi * 8);
      mma_bf16_16816(s[nt], qa[kk], b[0], b[1]);
      mma_bf16_16816(s[nt], qa[kk + 1], b[2], b[3]);
    }
}

__global__ void __launch_bounds__(kAttnThreads)
    attn_decode_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_cache,
                       const __nv_bfloat16* __restrict__ v_cache, const int32_t* __restrict__ kv_len,
                       const int32_t* __restrict__ cache_slot, const int32_t* __restrict__ kv_start, int nh,
                       int nkv, int max_seq, int n_slots, int chunk, float scale_log2,
                       float* __restrict__ part_o, float* __restrict__ part_ml) {
  extern __shared__ __align__(16) uint8_t attn_smem[];
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(attn_smem);  // [2][64][136]
  __nv_bfloat16* vs = ks + 2 * kAttnBK * kAttnPad;                   // [2][64][136]
  float* red = reinterpret_cast<float*>(vs + 2 * kAttnBK * kAttnPad); // [4 warps][8][128 + 2]
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int nsplit = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  griddep_wait();
  griddep_launch_dependents();
  int L = kv_len[b];
  const int slot_raw = cache_slot ? cache_slot[b] : b;
  const bool bad = L < 0 || L > max_seq || slot_raw < 0 || slot_raw >= n_slots;  // block-uniform
  if (bad) {
    if (threadIdx.x == 0) record_device_error(kDevErrBadIndex);
    L = 0;  // still write an empty partial so the combine stays defined
  }
  const int slot = bad ? 0 : slot_raw;
  const int kv0 = kv_start ? kv_start[b] : 0;  // keys before it are padding
  const int k_begin = split * chunk;
  const int k_end = min(L, k_begin + chunk);
  const __nv_bfloat16* kh = k_cache + (size_t(slot) * nkv + kvh) * max_seq * kAttnD;
  const __nv_bfloat16* vh = v_cache + (size_t(slot) * nkv + kvh) * max_seq * kAttnD;

  // Q fragments straight from global: row g = head kvh*8 + g, rows 8..15 = 0.
  uint32_t qa[8][4];
  const __nv_bfloat16* qrow = q + (size_t(b) * nh + kvh * kDecodeGroup + g) * kAttnD;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    qa[kk][0] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * tq);
    qa[kk][1] = 0u;
    qa[kk][2] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8 + 2 * tq);
    qa[kk][3] = 0u;
  }
  float o[16][4];
#pragma unroll
  for (int dn = 0; dn < 16; ++dn)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[dn][i] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

  const int n_tiles = k_end > k_begin ? (k_end - k_begin + kAttnBK - 1) / kAttnBK : 0;
  if (n_tiles > 0) {
    load_kv_tile(ks, kh, k_begin, k_end);
    load_kv_tile(vs, vh, k_begin, k_end);
    cp_async_commit();
  }
  for (int j = 0; j < n_tiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_tiles) {
      load_kv_tile(ks + (buf ^ 1) * kAttnBK * kAttnPad, kh, k_begin + (j + 1) * kAttnBK, k_end);
      load_kv_tile(vs + (buf ^ 1) * kAttnBK * kAttnPad, vh, k_begin + (j + 1) * kAttnBK, k_end);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int key0 = k_begin + j * kAttnBK + warp * 16;  // this warp's 16-key slice
    if (key0 < k_end) {
      const __nv_bfloat16* ks16 = ks + buf * kAttnBK * kAttnPad + warp * 16 * kAttnPad;
      const __nv_bfloat16* vs16 = vs + buf * kAttnBK * kAttnPad + warp * 16 * kAttnPad;
      float s2[2][4];
      qk_slice16(s2, qa, ks16, lane);
      // reuse the 64-key softmax helper on a zero-padded 16-key slice
      float s[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int key = key0 + nt * 8 + 2 * tq + (i & 1);
          s[nt][i] = (nt < 2 && key < k_end && key >= kv0) ? s2[nt][i] * scale_log2 : -INFINITY;
        }
      softmax_update(s, m, l, o);
      // P . V over this slice's 16 keys (one k-step)
      uint32_t a[4];
      a[0] = pack_bf16x2(s[0][0], s[0][1]);
      a[1] = pack_bf16x2(s[0][2], s[0][3]);
      a[2] = pack_bf16x2(s[1][0], s[1][1]);
      a[3] = pack_bf16x2(s[1][2], s[1][3]);
      const int mi = lane >> 3, r = lane & 7;
#pragma unroll
      for (int dn = 0; dn < 16; dn += 2) {
        uint32_t bb[4];
        ldsm_x4_trans(bb, vs16 + ((mi & 1) * 8 + r) * kAttnPad + (dn + (mi >> 1)) * 8);
        mma_bf16_16816(o[dn], a, bb[0], bb[1]);
        mma_bf16_16816(o[dn + 1], a, bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
  // row sums across the 4 lanes of a row
  l[0] += __shfl_xor_sync(0xFFFFFFFFu, l[0], 1);
  l[0] += __shfl_xor_sync(0xFFFFFFFFu, l[0], 2);
  // merge the four warps (rows g = query heads; rows 8..15 are padding)
  constexpr int kRedStride = kAttnD + 2;
  float* wr = red + (warp * kDecodeGroup + g) * kRedStride;
#pragma unroll
  for (int dn = 0; dn < 16; ++dn) {
    wr[dn * 8 + 2 * tq] = o[dn][0];
    wr[dn * 8 + 2 * tq + 1] = o[dn][1];
  }
  if (tq == 0) {
    wr[kAttnD] = m[0];
    wr[kAttnD + 1] = l[0];
  }
  __syncthreads();
  // thread -> (head hh, dims d0..d0+7)
  const int hh = threadIdx.x >> 4;
  const int d0 = (threadIdx.x & 15) * 8;
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < 4; ++w) M = fmaxf(M, red[(w * kDecodeGroup + hh) * kRedStride + kAttnD]);
  const float base = M == -INFINITY ? 0.f : M;
  float Ls = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float* rw = red + (w * kDecodeGroup + hh) * kRedStride;
    const float sc = exp2f(rw[kAttnD] - base);
    Ls += rw[kAttnD + 1] * sc;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += rw[d0 + i] * sc;
  }
  const int head = kvh * kDecodeGroup + hh;
  const size_t pidx = (size_t(b) * nh + head) * nsplit + split;
  float* po = part_o + pidx * kAttnD + d0;
#pragma unroll
  for (int i = 0; i < 8; i += 4) *reinterpret_cast<float4*>(po + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
  if (d0 == 0) {
    part_ml[pidx * 2] = M;
    part_ml[pidx * 2 + 1] = Ls;
  }
}

// out (B, nh*128) bf16 = merge of the nsplit partials; one warp per (b, head).
__global__ void __launch_bounds__(256)
    attn_decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                               int B, int nh, int nsplit, __nv_bfloat16* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (gw >= B * nh) return;
  const size_t base_idx = size_t(gw) * nsplit;
  if (nsplit <= 64) {
    // lane s holds splits s and s + 32: their maxima and sums in one round
    // trip, the scales kept in registers; then the partial outputs 16 splits
    // at a time with every load in flight.  Same sums in the same order as
    // the general loop below.
    float m0 = -INFINITY, l0 = 0.f, m1 = -INFINITY, l1 = 0.f;
    if (lane < nsplit) {
      const float2 ml = *reinterpret_cast<const float2*>(part_ml + (base_idx + lane) * 2);
      m0 = ml.x;
      l0 = ml.y;
    }
    if (lane + 32 < nsplit) {
      const float2 ml = *reinterpret_cast<const float2*>(part_ml + (base_idx + lane + 32) * 2);
      m1 = ml.x;
      l1 = ml.y;
    }
    float M = fmaxf(m0, m1);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, off));
    const float mb = M == -INFINITY ? 0.f : M;
    const float sc0 = lane < nsplit ? exp2f(m0 - mb) : 0.f;
    const float sc1 = lane + 32 < nsplit ? exp2f(m1 - mb) : 0.f;
    float L = 0.f;
    if (lane < nsplit) L += l0 * sc0;
    if (lane + 32 < nsplit) L += l1 * sc1;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) L += __shfl_xor_sync(0xFFFFFFFFu, L, off);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < nsplit; s0 += 16) {
      float4 v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (s0 + j < nsplit) v[j] = *reinterpret_cast<const float4*>(part_o + (base_idx + s0 + j) * kAttnD + lane * 4);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int sj = s0 + j;
        if (sj >= nsplit) break;
        const float sc = __shfl_sync(0xFFFFFFFFu, sj < 32 ? sc0 : sc1, sj & 31);
        acc[0] += v[j].x * sc;
        acc[1] += v[j].y * sc;
        acc[2] += v[j].z * sc;
        acc[3] += v[j].w * sc;
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    uint2 o;
    o.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
    o.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
    *reinterpret_cast<uint2*>(out + size_t(gw) * kAttnD + lane * 4) = o;
    return;
  }
  // the splits' maxima and sums: lane s takes splits s, s+32, ... (one round
  // trip), then warp reductions
  float M = -INFINITY;
  for (int s = lane; s < nsplit; s += 32) M = fmaxf(M, part_ml[(base_idx + s) * 2]);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, off));
  const float mb = M == -INFINITY ? 0.f : M;
  float L = 0.f;
  for (int s = lane; s < nsplit; s += 32)
    L += part_ml[(base_idx + s) * 2 + 1] * exp2f(part_ml[(base_idx + s) * 2] - mb);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) L += __shfl_xor_sync(0xFFFFFFFFu, L, off);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
  for (int s = 0; s < nsplit; ++s) {
    const float sc = exp2f(part_ml[(base_idx + s) * 2] - mb);
    const float4 v = *reinterpret_cast<const float4*>(part_o + (base_idx + s) * kAttnD + lane * 4);
    acc[0] += v.x * sc;
    acc[1] += v.y * sc;
    acc[2] += v.z * sc;
    acc[3] += v.w * sc;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  uint2 o;
  o.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  o.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  *reinterpret_cast<uint2*>(out + size_t(gw) * kAttnD + lane * 4) = o;
}

}  // namespace qmoe
