// K5 prefill: causal GQA flash attention on the 5th-generation tensor cores.
//
// Reference semantics: NxDI NeuronAttentionBase with GQA (qwen.py:313-341;
// flash kernel imported at qwen.py:25-28, 49):
//   out_h = softmax(q_h K_g^T * scale + causal mask) V_g,  g = h / (nh / nkv),
// query i of sequence b at absolute position q_start[b] + i attending to
// cache positions kv_start[b] .. q_start[b] + i (kv_start: left padding,
// 0 without it).  head_dim 128, bf16 in, fp32 scores / softmax / sums.
//
// One CTA = 128 queries (the TMEM lanes) of one (sequence, head); 192
// threads in three roles:
//   warp 4  TMA producer: Q once, then K and V tiles of 128 keys into two
//           stages each (3D tensor maps; the cache's (slot, kv head) is the
//           outer coordinate, so no load crosses into another head);
//   warp 5  MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM score
//           buffers (M=128 queries, N=128 keys, K=128 dims, both operands
//           K-major), and O_j = P_j V_j into one of two TMEM output buffers
//           (A = P from shared memory, K-major; B = V straight from its TMA
//           tile, MN-major: dims are V's contiguous axis);
//   warps 0-3  softmax: thread r owns query row r (TMEM lane r): row max of
//           S_j, the running max / sum, P_j = exp2(S_j*scale - max) written
//           as bf16 into the 128B-swizzled P tile, and the output kept in
//           fp32 registers: o = (o + O_{j-1}) * exp2(m_{j-1} - m_j).
// The MMA warp issues S_{j+1} before P_j V_j, so the tensor core computes the
// next scores while the softmax warps work on the current ones.
//
// Shared memory (1024-aligned tiles of 32 KB: two 64-column halves of 128
// rows x 128 B, 128-byte swizzle): Q | K[2] | V[2] | P = 192 KB, one CTA per
// SM.  TMEM: 512 columns = S[2] + O[2].
//
// Keys past the end of the tile's last query (the last tile's tail) hold
// whatever the cache holds there; their scores are masked, and the producer
// zeroes those V rows in shared memory before the last P V product, so a
// non-finite value in unused cache rows cannot reach the output (0 * inf).
//
// Every wait is bounded (kWaitLimitNs): on time-out the role records a
// device error, raises the CTA's abort flag, the MMA thread drains its
// outstanding MMAs, the producer waits for its loads in flight, TMEM is
// freed and the CTA returns without writing its rows.
#pragma once

#include "common.cuh"

namespace qmoe {

constexpr int kFaRows = 128;                    // queries per CTA = keys per tile
constexpr int kFaD = 128;                       // head dim
constexpr int kFaThreads = 192;
constexpr int kFaHalfBytes = kFaRows * 128;     // 128 rows x 64 bf16
constexpr int kFaTileBytes = 2 * kFaHalfBytes;  // 32 KB
constexpr int kFaTiles = 6;                     // Q, K[2], V[2], P
constexpr int kFaBarriers = 20;
constexpr int kFaSmemBytes = kFaTiles * kFaTileBytes + 1024 + kFaBarriers * 8 + 16;

struct FlashPrefillArgs {
  const int32_t* q_start;
  const int32_t* cache_slot;
  const int32_t* kv_start;
  __nv_bfloat16* out;
  int S, nh, nkv, max_seq, n_slots, B, n_qtiles;
  float scale_log2;
};

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* tmap, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory descriptor of an MN-major operand, 128-byte swizzle: 64
// contiguous MN elements per 128-byte row, one row per K index, 8-row groups
// `sbo` bytes apart, 64-element MN blocks `lbo` bytes apart.
__device__ __forceinline__ uint64_t make_sw128_desc_mn(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr & 0x3FFFFu) >> 4);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;   // sm_100 descriptor version
  d |= uint64_t(2) << 61;   // 128B swizzle
  return d;
}

// Bounded wait on an mbarrier phase for one thread; on time-out records
// `code` and raises the abort flag.  Gives up at once if the flag is up.
__device__ __forceinline__ bool fa_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        unsigned int code) {
  return mbar_wait_bounded(bar, parity, abort_flag, code);
}

// The same wait taken by every lane of a warp, with one verdict for all of
// them (a lane that timed out never leaves the others at a warp barrier).
__device__ __forceinline__ bool fa_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                             unsigned int code) {
  return __all_sync(0xFFFFFFFFu, mbar_wait_bounded(bar, parity, abort_flag, code));
}

// Wait (bounded, whatever the abort flag says) for a phase that TMA loads
// already issued will complete: the CTA must not exit with copies in flight.
__device__ __forceinline__ void fa_wait_landed(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_device_error(kDevErrWaitTimeoutProducer);
      return;
    }
  }
}

__global__ void __launch_bounds__(kFaThreads, 1)
    flash_prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const FlashPrefillArgs a) {
  extern __shared__ uint8_t fa_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kFaTileBytes;       // [2]
  uint8_t* sV = sK + 2 * kFaTileBytes;     // [2]
  uint8_t* sP = sV + 2 * kFaTileBytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kFaTiles * kFaTileBytes);
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;    // [2]
  uint64_t* v_full = bar + 3;    // [2]
  uint64_t* k_empty = bar + 5;   // [2]
  uint64_t* v_empty = bar + 7;   // [2]
  uint64_t* s_full = bar + 9;    // [2]
  uint64_t* s_empty = bar + 11;  // [2]
  uint64_t* p_full = bar + 13;
  uint64_t* o_full = bar + 14;   // [2]
  uint64_t* o_empty = bar + 16;  // [2]
  uint64_t* v_tail = bar + 18;
  uint64_t* drain = bar + 19;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kFaBarriers);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // heaviest query tiles (the latest ones: most keys) first over all heads
  const int per_tile = a.nh * a.B;
  const int qt = a.n_qtiles - 1 - int(blockIdx.x) / per_tile;
  const int rest = int(blockIdx.x) % per_tile;
  const int h = rest % a.nh;
  const int b = rest / a.nh;
  const int q0 = qt * kFaRows;
  const int kvh = h / (a.nh / a.nkv);

  griddep_wait();
  const int L0 = a.q_start[b];
  const int slot = a.cache_slot ? a.cache_slot[b] : b;
  if (L0 < 0 || L0 + a.S > a.max_seq || slot < 0 || slot >= a.n_slots) {  // block-uniform
    if (threadIdx.x == 0) record_device_error(kDevErrBadIndex);
    return;
  }
  const int nq = min(kFaRows, a.S - q0);
  const int n_keys = L0 + q0 + nq;  // keys visible to the tile's last query
  int kv0 = a.kv_start ? a.kv_start[b] : 0;
  kv0 = max(0, min(kv0, L0 + a.S));
  const int j0 = kv0 / kFaRows;
  const int n_tiles = kv0 < n_keys ? (n_keys + kFaRows - 1) / kFaRows - j0 : 0;
  const size_t out_ld = size_t(a.nh) * kFaD;
  __nv_bfloat16* out_tile = a.out + (size_t(b) * a.S + q0) * out_ld + size_t(h) * kFaD;
  if (n_tiles == 0) {
    // every query of the tile is a padding position: no visible key, zeros
    for (int i = threadIdx.x; i < nq * (kFaD / 8); i += blockDim.x)
      reinterpret_cast<uint4*>(out_tile + size_t(i / (kFaD / 8)) * out_ld)[i % (kFaD / 8)] = make_uint4(0, 0, 0, 0);
    return;
  }
  const bool tail = (n_keys % kFaRows) != 0;  // the last tile has rows past n_keys

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(v_tail, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    const int kv_z = slot * a.nkv + kvh;
    int issued_k[2] = {0, 0}, issued_v[2] = {0, 0};
    bool ok = true;
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kFaTileBytes);
      tma_load_3d(sQ, &tm_q, 0, h, b * a.S + q0, q_full);
      tma_load_3d(sQ + kFaHalfBytes, &tm_q, 64, h, b * a.S + q0, q_full);
      for (int i = 0; i < n_tiles; ++i) {
        const int st = i & 1, use = i >> 1;
        const int key0 = (j0 + i) * kFaRows;
        if (i >= 2 && !fa_wait(&k_empty[st], (use - 1) & 1, abort_flag, kDevErrWaitTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], kFaTileBytes);
        tma_load_3d(sK + st * kFaTileBytes, &tm_k, 0, key0, kv_z, &k_full[st]);
        tma_load_3d(sK + st * kFaTileBytes + kFaHalfBytes, &tm_k, 64, key0, kv_z, &k_full[st]);
        ++issued_k[st];
        if (i >= 2 && !fa_wait(&v_empty[st], (use - 1) & 1, abort_flag, kDevErrWaitTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], kFaTileBytes);
        tma_load_3d(sV + st * kFaTileBytes, &tm_v, 0, key0, kv_z, &v_full[st]);
        tma_load_3d(sV + st * kFaTileBytes + kFaHalfBytes, &tm_v, 64, key0, kv_z, &v_full[st]);
        ++issued_v[st];
      }
    }
    ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
    if (ok && tail) {
      // zero the V rows of the last tile past the last visible key
      const int last = n_tiles - 1;
      const int st = last & 1;
      if (fa_wait_warp(&v_full[st], (last >> 1) & 1, abort_flag, kDevErrWaitTimeoutProducer)) {
        const int first = n_keys - (j0 + last) * kFaRows;  // rows [first, 128) are past n_keys
        uint8_t* vt = sV + st * kFaTileBytes;
        for (int i = first * 8 + lane; i < kFaRows * 8; i += 32) {  // 16-byte chunks of whole rows
          const int r = i >> 3, c = i & 7;
          *reinterpret_cast<uint4*>(vt + r * 128 + c * 16) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(vt + kFaHalfBytes + r * 128 + c * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(v_tail);
      }
    }
    if (lane == 0) {
      // loads still in flight land before the CTA can exit
      fa_wait_landed(q_full, 0);
      for (int st = 0; st < 2; ++st) {
        if (issued_k[st]) fa_wait_landed(&k_full[st], (issued_k[st] - 1) & 1);
        if (issued_v[st]) fa_wait_landed(&v_full[st], (issued_v[st] - 1) & 1);
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_bf16(kFaRows, kFaRows);
      const uint32_t idesc_o = make_idesc_bf16(kFaRows, kFaD) | (1u << 16);  // B (V) MN-major
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      bool ok = fa_wait(q_full, 0, abort_flag, kDevErrWaitTimeoutMma);
      for (int i = 0; ok && i <= n_tiles; ++i) {
        if (i < n_tiles) {
          const int st = i & 1, use = i >> 1;
          if (!fa_wait(&k_full[st], use & 1, abort_flag, kDevErrWaitTimeoutMma) ||
              (i >= 2 && !fa_wait(&s_empty[st], (use - 1) & 1, abort_flag, kDevErrWaitTimeoutMma))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + st * kFaTileBytes);
          const uint32_t d = tmem_base + st * kFaRows;
#pragma unroll
          for (int kk = 0; kk < kFaD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kFaHalfBytes + (kk & 3) * 32;
            umma_bf16(d, make_sw128_desc(q_addr + off), make_sw128_desc(k_addr + off), idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[st]);
          umma_commit(&k_empty[st]);
        }
        if (i >= 1) {
          const int pi = i - 1;
          const int st = pi & 1, use = pi >> 1;
          if (!fa_wait(p_full, pi & 1, abort_flag, kDevErrWaitTimeoutMma) ||
              !fa_wait(&v_full[st], use & 1, abort_flag, kDevErrWaitTimeoutMma) ||
              (tail && pi == n_tiles - 1 && !fa_wait(v_tail, 0, abort_flag, kDevErrWaitTimeoutMma)) ||
              (pi >= 2 && !fa_wait(&o_empty[st], (use - 1) & 1, abort_flag, kDevErrWaitTimeoutMma))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sV + st * kFaTileBytes);
          const uint32_t d = tmem_base + 2 * kFaRows + st * kFaD;
#pragma unroll
          for (int kk = 0; kk < kFaRows / 16; ++kk) {  // 16 keys per MMA
            const uint64_t adesc = make_sw128_desc(p_addr + (kk >> 2) * kFaHalfBytes + (kk & 3) * 32);
            const uint64_t bdesc = make_sw128_desc_mn(v_addr + kk * 16 * 128, kFaHalfBytes, 1024);
            umma_bf16(d, adesc, bdesc, idesc_o, kk > 0 ? 1u : 0u);
          }
          umma_commit(&o_full[st]);
          umma_commit(&v_empty[st]);
        }
      }
      if (!ok) *abort_flag = 1;
      umma_commit(drain);
      const unsigned long long t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          record_device_error(kDevErrWaitTimeoutMma);
          break;
        }
      }
    }
  } else {
    // ---------------- softmax (warps 0-3, one query row per thread) ----------------
    const int row = warp * 32 + lane;
    const int qpos = L0 + q0 + row;
    const uint32_t t_lane = uint32_t(warp * 32) << 16;
    const uint32_t p_row = smem_u32(sP) + row * 128;
    const int sw = row & 7;
    float o[kFaD];
#pragma unroll
    for (int d = 0; d < kFaD; ++d) o[d] = 0.f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      const int st = i & 1, use = i >> 1;
      if (!fa_wait_warp(&s_full[st], use & 1, abort_flag, kDevErrWaitTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int key0 = (j0 + i) * kFaRows;
      const uint32_t sa = tmem_base + t_lane + st * kFaRows;
      // pass 1: row max of the visible scores
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kFaRows / 16; ++c) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(sa + c * 16, v);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int key = key0 + c * 16 + e;
          if (key >= kv0 && key <= qpos) mx = fmaxf(mx, __uint_as_float(v[e]));
        }
      }
      const float m_new = fmaxf(m, mx * a.scale_log2);
      const float alpha = m == -INFINITY ? 0.f : exp2f(m - m_new);
      // fold the previous tile's P V into the registers (its P buffer is then free)
      if (i >= 1) {
        const int pst = (i - 1) & 1, puse = (i - 1) >> 1;
        if (!fa_wait_warp(&o_full[pst], puse & 1, abort_flag, kDevErrWaitTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t oa = tmem_base + t_lane + 2 * kFaRows + pst * kFaD;
#pragma unroll
        for (int c = 0; c < kFaD / 16; ++c) {
          uint32_t v[16];
          tmem_ld_32x32b_x16(oa + c * 16, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[c * 16 + e] = (o[c * 16 + e] + __uint_as_float(v[e])) * alpha;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_empty[pst]);
      }
      // pass 2: P = exp2(S*scale - m_new) as bf16 into the swizzled P tile
      const float mb = m_new == -INFINITY ? 0.f : m_new;
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < kFaRows / 16; ++c) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(sa + c * 16, v);
        tmem_ld_wait();
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const int key = key0 + c * 16 + e;
          const float p0 = (key >= kv0 && key <= qpos) ? exp2f(__uint_as_float(v[e]) * a.scale_log2 - mb) : 0.f;
          const float p1 =
              (key + 1 >= kv0 && key + 1 <= qpos) ? exp2f(__uint_as_float(v[e + 1]) * a.scale_log2 - mb) : 0.f;
          lsum += p0 + p1;
          const __nv_bfloat162 pp = __floats2bfloat162_rn(p0, p1);
          pk[e >> 1] = *reinterpret_cast<const uint32_t*>(&pp);
        }
        // columns c*16 .. c*16+15: half c/4, 16-byte chunks 2*(c%4) and +1
        const uint32_t base = p_row + (c >> 2) * kFaHalfBytes;
        const int ch = (c & 3) * 2;
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(base + ((ch ^ sw) << 4)), "r"(pk[0]),
                     "r"(pk[1]), "r"(pk[2]), "r"(pk[3])
                     : "memory");
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(base + (((ch + 1) ^ sw) << 4)), "r"(pk[4]),
                     "r"(pk[5]), "r"(pk[6]), "r"(pk[7])
                     : "memory");
      }
      tc_fence_before();
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_empty[st]);
        mbar_arrive(p_full);
      }
      l = l * alpha + lsum;
      m = m_new;
    }
    if (ok) {
      const int last = n_tiles - 1;
      const int pst = last & 1;
      if (fa_wait_warp(&o_full[pst], (last >> 1) & 1, abort_flag, kDevErrWaitTimeoutEpilogue)) {
        tc_fence_after();
        const uint32_t oa = tmem_base + t_lane + 2 * kFaRows + pst * kFaD;
#pragma unroll
        for (int c = 0; c < kFaD / 16; ++c) {
          uint32_t v[16];
          tmem_ld_32x32b_x16(oa + c * 16, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[c * 16 + e] += __uint_as_float(v[e]);
        }
        tc_fence_before();
        if (row < nq) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          uint4* dst = reinterpret_cast<uint4*>(out_tile + size_t(row) * out_ld);
#pragma unroll
          for (int c = 0; c < kFaD / 8; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_bfloat162 pp = __floats2bfloat162_rn(o[c * 8 + 2 * e] * inv, o[c * 8 + 2 * e + 1] * inv);
              w[e] = *reinterpret_cast<const uint32_t*>(&pp);
            }
            dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }

  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace qmoe
