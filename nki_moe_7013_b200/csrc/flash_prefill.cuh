// K5 prefill: causal GQA flash attention on the 5th-generation tensor cores.
//
// Reference semantics: NxDI NeuronAttentionBase with GQA (qwen.py:313-341;
// flash kernel imported at qwen.py:25-28, 49):
//   out_h = softmax(q_h K_g^T * scale + causal mask) V_g,  g = h / (nh / nkv),
// query i of sequence b at absolute position q_start[b] + i attending to
// cache positions kv_start[b] .. q_start[b] + i (kv_start: left padding,
// 0 without it).  head_dim 128, bf16 in, fp32 scores / softmax / sums.
//
// One CTA = two tiles of 128 queries (A: rows q0..q0+127, B: the next 128)
// of one (sequence, head), sharing every K / V tile of 128 keys; 320 threads:
//   warps 0-3  softmax of tile A, warps 4-7 softmax of tile B: thread r of a
//              group owns query row r (TMEM lane r);
//   warp 8     TMA producer: Q_A and Q_B once, then K_0, V_0, K_1, V_1, ...
//              through a pool of three 32 KB slots (3D tensor maps, the
//              cache's (slot, kv head) as the outer coordinate);
//   warp 9     MMA issuer (one thread), in the order
//              S_A(0) S_B(0) | PV_A(0) S_A(1) PV_B(0) S_B(1) | PV_A(1) ...
//              so the tensor core computes one tile's scores while the other
//              tile's softmax runs.
// S_X = Q_X K^T (M=128 queries, N=128 keys, K=128 dims, both K-major) lands
// in TMEM; O_X += P_X V (A = P_X from shared memory, K-major; B = V straight
// from its TMA tile, MN-major) accumulates in TMEM across the key tiles.
// The softmax keeps a per-row running max m and sum l; P = exp2(S*scale - m)
// in bf16.  When a row's max grows by more than 2^8 the group rescales its O
// rows in TMEM (load, multiply, store) before releasing P; otherwise m stays
// (P <= 2^8, exact enough in bf16) and O is never touched by the softmax.
// A tile's whole score row is read with four TMEM loads and one wait.
//
// Shared memory (1024-aligned 32 KB tiles = two 64-column halves of 128
// rows x 128 B, 128-byte swizzle): Q_A | Q_B | pool[3] | P_A | P_B = 224 KB,
// one CTA per SM.  TMEM: S_A | S_B | O_A | O_B = 512 columns.
//
// Keys past the last query of the CTA (the last tile's tail) hold whatever
// the cache holds there; their scores are masked, and the producer zeroes
// those V rows in shared memory before the last P V products, so a
// non-finite value in unused cache rows cannot reach a valid output row.
//
// Every wait is bounded (kWaitLimitNs): on time-out the role records a
// device error and raises the CTA's abort flag, the MMA thread drains its
// outstanding MMAs, the producer waits for its loads in flight, TMEM is
// freed and the CTA returns without writing its rows.
#pragma once

#include "common.cuh"

namespace qmoe {

constexpr int kFaRows = 128;                    // queries per tile = keys per tile
constexpr int kFaD = 128;                       // head dim
constexpr int kFaThreads = 320;                 // 2 softmax groups, producer, MMA
constexpr int kFaHalfBytes = kFaRows * 128;     // 128 rows x 64 bf16
constexpr int kFaTileBytes = 2 * kFaHalfBytes;  // 32 KB
constexpr int kFaPool = 3;                      // K / V slots
constexpr int kFaTiles = 4 + kFaPool;           // Q_A, Q_B, pool, P_A, P_B
constexpr int kFaBarriers = 16;
constexpr int kFaSmemBytes = kFaTiles * kFaTileBytes + 1024 + kFaBarriers * 8 + 16;
constexpr float kFaRescaleLog2 = 8.f;           // rescale O when a row max grows by more than 2^8

struct FlashPrefillArgs {
  const int32_t* q_start;
  const int32_t* cache_slot;
  const int32_t* kv_start;
  __nv_bfloat16* out;
  int S, nh, nkv, max_seq, n_slots, B, n_pairs;
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

// 32 lanes x 32 bit, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 2^x with the SFU's approximate exp2, denormal results flushed to zero (the
// probabilities are stored as bf16 and lie in [0, 2^8]; exp2(-inf) = 0).
__device__ __forceinline__ float fa_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Bounded wait on an mbarrier phase for one thread; on time-out records
// `code` and raises the abort flag.  Gives up at once if the flag is up.
__device__ __forceinline__ bool fa_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        unsigned int code) {
  return mbar_wait_bounded(bar, parity, abort_flag, code);
}

// The same wait taken by every lane of a warp, with one outcome for all of
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
  uint8_t* sQ = smem;                              // [2]: tiles A, B
  uint8_t* sPool = smem + 2 * kFaTileBytes;        // [kFaPool]: K_0, V_0, K_1, V_1, ... in rotation
  uint8_t* sP = sPool + kFaPool * kFaTileBytes;    // [2]: tiles A, B
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kFaTiles * kFaTileBytes);
  uint64_t* q_full = bar + 0;
  uint64_t* full = bar + 1;     // [kFaPool]
  uint64_t* empty = bar + 4;    // [kFaPool]
  uint64_t* s_full = bar + 7;   // [2] per query tile
  uint64_t* p_full = bar + 9;   // [2]
  uint64_t* o_full = bar + 11;  // [2]
  uint64_t* v_tail = bar + 13;
  uint64_t* drain = bar + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kFaBarriers);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // heaviest tile pairs (the latest queries: most keys) first over all heads
  const int per_pair = a.nh * a.B;
  const int pc = a.n_pairs - 1 - int(blockIdx.x) / per_pair;
  const int rest = int(blockIdx.x) % per_pair;
  const int h = rest % a.nh;
  const int b = rest / a.nh;
  const int q0 = pc * 2 * kFaRows;
  const int kvh = h / (a.nh / a.nkv);

  griddep_wait();
  const int L0 = a.q_start[b];
  const int slot = a.cache_slot ? a.cache_slot[b] : b;
  if (L0 < 0 || L0 + a.S > a.max_seq || slot < 0 || slot >= a.n_slots) {  // block-uniform
    if (threadIdx.x == 0) record_device_error(kDevErrBadIndex);
    return;
  }
  const int nq_a = min(kFaRows, a.S - q0);
  const int nq_b = max(0, min(kFaRows, a.S - q0 - kFaRows));
  const int n_keys = L0 + q0 + (nq_b > 0 ? kFaRows + nq_b : nq_a);  // keys visible to the last query
  int kv0 = a.kv_start ? a.kv_start[b] : 0;
  kv0 = max(0, min(kv0, L0 + a.S));
  const int j0 = kv0 / kFaRows;
  const int n_tiles = kv0 < n_keys ? (n_keys + kFaRows - 1) / kFaRows - j0 : 0;
  const size_t out_ld = size_t(a.nh) * kFaD;
  __nv_bfloat16* out_tile = a.out + (size_t(b) * a.S + q0) * out_ld + size_t(h) * kFaD;
  if (n_tiles == 0) {
    // every query of the pair is a padding position: no visible key, zeros
    for (int i = threadIdx.x; i < (nq_a + nq_b) * (kFaD / 8); i += blockDim.x)
      reinterpret_cast<uint4*>(out_tile + size_t(i / (kFaD / 8)) * out_ld)[i % (kFaD / 8)] = make_uint4(0, 0, 0, 0);
    return;
  }
  const bool tail = (n_keys % kFaRows) != 0;  // the last tile has rows past n_keys

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kFaPool; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], 4);
      mbar_init(&o_full[g], 1);
    }
    mbar_init(v_tail, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    const int kv_z = slot * a.nkv + kvh;
    int issued[kFaPool] = {0, 0, 0};
    bool ok = true;
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * kFaTileBytes);
      for (int g = 0; g < 2; ++g) {
        const int z = b * a.S + q0 + g * kFaRows;
        tma_load_3d(sQ + g * kFaTileBytes, &tm_q, 0, h, z, q_full);
        tma_load_3d(sQ + g * kFaTileBytes + kFaHalfBytes, &tm_q, 64, h, z, q_full);
      }
      for (int n = 0; n < 2 * n_tiles; ++n) {  // K_i = item 2i, V_i = item 2i + 1
        const int sl = n % kFaPool, u = n / kFaPool;
        if (n >= kFaPool && !fa_wait(&empty[sl], (u - 1) & 1, abort_flag, kDevErrWaitTimeoutProducer)) {
          ok = false;
          break;
        }
        const int key0 = (j0 + (n >> 1)) * kFaRows;
        const CUtensorMap* tm = (n & 1) ? &tm_v : &tm_k;
        uint8_t* dst = sPool + sl * kFaTileBytes;
        mbar_arrive_expect_tx(&full[sl], kFaTileBytes);
        tma_load_3d(dst, tm, 0, key0, kv_z, &full[sl]);
        tma_load_3d(dst + kFaHalfBytes, tm, 64, key0, kv_z, &full[sl]);
        ++issued[sl];
      }
    }
    ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
    if (ok && tail) {
      // zero the last V tile's rows past the last visible key
      const int n = 2 * n_tiles - 1;
      const int sl = n % kFaPool;
      if (fa_wait_warp(&full[sl], (n / kFaPool) & 1, abort_flag, kDevErrWaitTimeoutProducer)) {
        const int first = n_keys - (j0 + n_tiles - 1) * kFaRows;  // rows [first, 128) lie past n_keys
        uint8_t* vt = sPool + sl * kFaTileBytes;
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
      for (int sl = 0; sl < kFaPool; ++sl)
        if (issued[sl]) fa_wait_landed(&full[sl], (issued[sl] - 1) & 1);
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_bf16(kFaRows, kFaRows);
      const uint32_t idesc_o = make_idesc_bf16(kFaRows, kFaD) | (1u << 16);  // B (V) MN-major
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP), pool = smem_u32(sPool);
      auto item_full = [&](int n) {
        return fa_wait(&full[n % kFaPool], (n / kFaPool) & 1, abort_flag, kDevErrWaitTimeoutMma);
      };
      auto issue_s = [&](int g, int i) {  // S_g = Q_g K_i^T
        const uint32_t k_addr = pool + ((2 * i) % kFaPool) * kFaTileBytes;
        const uint32_t qa = q_addr + g * kFaTileBytes;
        const uint32_t d = tmem_base + g * kFaRows;
#pragma unroll
        for (int kk = 0; kk < kFaD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kFaHalfBytes + (kk & 3) * 32;
          umma_bf16(d, make_sw128_desc(qa + off), make_sw128_desc(k_addr + off), idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[g]);
      };
      auto issue_pv = [&](int g, int i) {  // O_g (+)= P_g V_i
        const uint32_t v_addr = pool + ((2 * i + 1) % kFaPool) * kFaTileBytes;
        const uint32_t pa = p_addr + g * kFaTileBytes;
        const uint32_t d = tmem_base + 2 * kFaRows + g * kFaD;
#pragma unroll
        for (int kk = 0; kk < kFaRows / 16; ++kk) {  // 16 keys per MMA
          const uint64_t adesc = make_sw128_desc(pa + (kk >> 2) * kFaHalfBytes + (kk & 3) * 32);
          const uint64_t bdesc = make_sw128_desc_mn(v_addr + kk * 16 * 128, kFaHalfBytes, 1024);
          umma_bf16(d, adesc, bdesc, idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = fa_wait(q_full, 0, abort_flag, kDevErrWaitTimeoutMma) && item_full(0);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(&empty[0]);  // K_0 read by both
      }
      for (int i = 0; ok && i < n_tiles; ++i) {
        const int nv = 2 * i + 1, nk = 2 * i + 2;
        const bool last = i == n_tiles - 1;
        // PV_A(i), then S_A(i+1)
        if (!fa_wait(&p_full[0], i & 1, abort_flag, kDevErrWaitTimeoutMma) || !item_full(nv) ||
            (tail && last && !fa_wait(v_tail, 0, abort_flag, kDevErrWaitTimeoutMma))) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv(0, i);
        if (last) umma_commit(&o_full[0]);
        if (!last) {
          if (!item_full(nk)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(0, i + 1);
        }
        // PV_B(i), then S_B(i+1)
        if (!fa_wait(&p_full[1], i & 1, abort_flag, kDevErrWaitTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv(1, i);
        umma_commit(&empty[nv % kFaPool]);  // V_i read by both
        if (last) umma_commit(&o_full[1]);
        if (!last) {
          issue_s(1, i + 1);
          umma_commit(&empty[nk % kFaPool]);  // K_{i+1} read by both
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
    // ---------------- softmax: warps 0-3 tile A, warps 4-7 tile B ----------------
    const int g = warp >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qbase = L0 + q0 + g * kFaRows + quad * 32;  // the warp's first query position
    const int qpos = qbase + lane;
    const uint32_t t_lane = uint32_t(quad * 32) << 16;
    const uint32_t s_col = tmem_base + t_lane + g * kFaRows;
    const uint32_t o_col = tmem_base + t_lane + 2 * kFaRows + g * kFaD;
    const uint32_t p_row = smem_u32(sP + g * kFaTileBytes) + r * 128;
    const int sw = r & 7;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      if (!fa_wait_warp(&s_full[g], i & 1, abort_flag, kDevErrWaitTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int key0 = (j0 + i) * kFaRows;
      float sv[kFaRows];
#pragma unroll
      for (int c = 0; c < kFaRows / 32; ++c) tmem_ld_x32(s_col + c * 32, sv + c * 32);
      tmem_ld_wait();
      if (!(key0 >= kv0 && key0 + kFaRows - 1 <= qbase)) {  // a tile this warp does not see whole
#pragma unroll
        for (int e = 0; e < kFaRows; ++e) {
          const int key = key0 + e;
          if (key < kv0 || key > qpos) sv[e] = -INFINITY;
        }
      }
      // row max as 8 independent chains (a single 128-long chain is ~4 cycles
      // a step with only two softmax warps per scheduler to hide it)
      float mx8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) mx8[j] = sv[j];
#pragma unroll
      for (int e = 8; e < kFaRows; ++e) mx8[e & 7] = fmaxf(mx8[e & 7], sv[e]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float m_new = fmaxf(m_used, mx * a.scale_log2);
      float alpha = 1.f;
      if (m_new > m_used + kFaRescaleLog2) {
        alpha = m_used == -INFINITY ? 0.f : exp2f(m_used - m_new);
        m_used = m_new;
      }
      const float mb = m_used == -INFINITY ? 0.f : m_used;
      // P = exp2(S*scale - m) as bf16 into the swizzled P tile
      float ls8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // 8 independent partial sums
#pragma unroll
      for (int c = 0; c < kFaRows / 16; ++c) {
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float p0 = fa_exp2(sv[c * 16 + e] * a.scale_log2 - mb);
          const float p1 = fa_exp2(sv[c * 16 + e + 1] * a.scale_log2 - mb);
          ls8[e >> 1] += p0 + p1;
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
      const float lsum = ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
      l = l * alpha + lsum;
      // a grown row max: rescale this group's O rows (PV of the earlier tiles
      // is complete -- it was issued before S of this tile)
      if (i > 0 && __any_sync(0xFFFFFFFFu, alpha != 1.f)) {
#pragma unroll
        for (int c = 0; c < kFaD / 32; ++c) {
          float ov[32];
          tmem_ld_x32(o_col + c * 32, ov);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] *= alpha;
          tmem_st_x32(o_col + c * 32, ov);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
    }
    if (ok && fa_wait_warp(&o_full[g], 0, abort_flag, kDevErrWaitTimeoutEpilogue)) {
      tc_fence_after();
      const int nq = g ? nq_b : nq_a;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(out_tile + size_t(g * kFaRows + r) * out_ld);
#pragma unroll
      for (int c = 0; c < kFaD / 32; ++c) {
        float ov[32];
        tmem_ld_x32(o_col + c * 32, ov);
        tmem_ld_wait();
        if (r < nq) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_bfloat162 pp = __floats2bfloat162_rn(ov[q * 8 + 2 * e] * inv, ov[q * 8 + 2 * e + 1] * inv);
              w[e] = *reinterpret_cast<const uint32_t*>(&pp);
            }
            dst[c * 4 + q] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace qmoe
