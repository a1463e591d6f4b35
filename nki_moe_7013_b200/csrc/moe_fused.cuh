// K3a + K3b in ONE persistent kernel (prefill sizes).
//
// The separate gate/up and down launches leave two gaps at a layer's core:
// the gate/up grid's last partial wave (a 1024-token layer has ~5.3 waves of
// 1 MB weight units: the last CTAs finish ~20 us after the median one), and
// the down kernel's start-up after the whole gate/up grid has drained.  Here
// the unit list is every gate/up unit (tile-major) followed by every down
// unit (tile-major), run by one CTA per SM that draws units in order from a
// global atomic counter: a CTA out of gate/up work moves straight on to down
// units while others finish theirs, and the dynamic draw balances the unequal
// units (a gate/up unit streams ~5x the bytes of a down unit, so a static deal
// would leave the CTAs that drew an extra gate/up unit a unit behind).
//
// Dependency: down unit (tile t, feature block f) multiplies the activations
// of tile t, which the n_mt_gu gate/up units of tile t write.  Each gate/up
// unit's epilogue bumps done[t] after its stores (fenced); the producer of a
// down unit waits (bounded) for done[t] == n_mt_gu before loading those
// activation rows with TMA.  Deadlock-free: units are drawn in order, so a
// down unit is drawn only after every gate/up unit has been drawn by a CTA
// that is running it (gate/up units wait on nothing), and the grid (one CTA
// per SM) is co-resident.
// Down weights do not depend on anything, so the wait only gates the
// activation loads of the unit's first stage.
//
// Unit shapes: a gate/up unit is 128 gate + the matching 128 up features of
// one tile (two accumulators sharing the row operand); a down unit is 256
// output features of one tile (two 128-feature accumulators sharing the
// activation rows) when H is a multiple of 256, else 128.  Every stage then
// carries two 16 KB weight tiles and the rows: 8 MMAs per 48 KB instead of 4
// per 32 KB for single-tile down units, and the activation rows are read
// half as often.
//
// The producer claims the unit after the one it is loading as soon as it has
// claimed that one, so the counter's round trip overlaps a unit's loads
// instead of draining the ring between units.  A CTA's first unit is its
// blockIdx.x (no atomic before the first loads); the counter hands out units
// from gridDim.x on.  (Every CTA is resident, so units are still taken in
// order by running CTAs.)  (Deadlock-free as above: a CTA
// holding an unstarted unit is working on an earlier-drawn one, and only down
// units wait -- on gate/up units, all of which were drawn before them.)
//
// Gate/up rows come from the permuted copy of the tokens (16-row boxes) or
// straight from the token rows (TMA gather4 by row_token; no copy to write).
//
// A tile outside its limits (more than 128 rows, or rows outside [0, R)) is
// skipped by every warp role with device error 4, never loaded into a stage.
//
// Pipeline, warp roles, TMEM double-buffering, swizzles and epilogues are
// those of grouped_gemm_kernel (gate/up: two accumulators, SiLU(gate)*up;
// down: weighted rows reduced into the fp32 combine accumulator).  The
// producer draws each unit from the counter and passes it to the MMA and
// epilogue warps through a small shared-memory queue (kUnitQueue slots, full
// / empty mbarriers); -1 ends the stream.
#pragma once

#include "common.cuh"
#include "grouped_gemm.cuh"

namespace qmoe {

struct FusedCfg {
  static constexpr int kMaxRows = kBNMax;                    // rows of a tile
  static constexpr int kABytes = kBM * kBK * 2;              // 16 KB
  static constexpr int kBBytes = kMaxRows * kBK * 2;         // 16 KB
  static constexpr int kStageBytes = 2 * kABytes + kBBytes;  // two weight tiles + the rows
  static constexpr int kStages = 4;
  static constexpr int kAccCols = 256;                       // one TMEM buffer: two 128-column accumulators
  static constexpr int kTmemCols = 512;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kUnitQueue = 4;
  // per-warp transpose tiles, then per row: destination, weight, source
  // rank and (return epilogue) the row's address in its return buffer
  static constexpr int kStagingBytes = 4 * 16 * 33 * 4 + kMaxRows * 20;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kBarrierBytes + kStagingBytes;
  static_assert(1024 + kStages * kStageBytes + kBarrierBytes + kStagingBytes <= 232448, "227 KB per CTA");
};

struct FusedArgs {
  const int32_t* tiles;  // [0] = ntiles, then expert[max_tiles], row0[max_tiles], nrows[max_tiles]
  int max_tiles;
  int n_rows;            // R: rows of the permuted operands (a tile outside [0, R) is refused)
  int n_mt_gu, n_mt_dn;      // units per tile: I / 128 and H / (128 * (1 + dn_two))
  int dn_two;                // 1: a down unit covers 256 features (two accumulators)
  int full_boxes;            // 1: tmB_*_full map whole 128-row tiles (one TMA load per stage)
  int num_kb_gu, num_kb_dn;  // k blocks: H / 64 and I / 64
  int a_rows_gu;             // 2I
  int up_off;                // I
  int a_rows_dn;             // H
  __nv_bfloat16* act;        // (R, I)
  int act_ld;
  const int32_t* row_dst;
  const float* row_w;
  float* acc;
  int acc_ld;
  int n_acc;
  int* done;  // [max_tiles + 2]: gate/up units finished per tile, the unit
              // counter, the grid-barrier counter; all zero on entry
  // when fin_out is set, after one grid-wide barrier on done[max_tiles + 1]
  // every CTA finalises a slice of the combine: fin_out = bf16(acc +
  // fin_residual) -- the finalize kernel folded in
  const __nv_bfloat16* fin_residual;
  __nv_bfloat16* fin_out;
  // expert-parallel return (kReturn): per row {weight bits, source rank,
  // return row, 0}; the weighted bf16 row goes to peer_ret[source] +
  // (ret_row0 + return row) * acc_ld instead of the fp32 accumulator
  const int4* row_meta;
  __nv_bfloat16* const* peer_ret;
  int ret_row0;
  int n_ranks;
  // non-null: gate/up row r of a tile is token row gather_rows[r] of x (TMA
  // gather4; tmB_gu maps x with 1-row boxes), else row r of the permuted copy
  const int32_t* gather_rows;
};


// One unit's shape, derived identically by the producer, MMA and epilogue
// warps.  rows == 0: a tile outside its limits -- the unit is skipped by all
// three (a gate/up unit still counts as done for its tile's down units).
struct FusedUnit {
  bool gu;      // gate/up (else down)
  int tile, mt;
  int e, row0, rows, nb;  // expert, first row, rows, 16-row boxes
  bool two;     // two accumulators (gate + up, or two 128-feature halves)
};

// TMEM buffer sequence of the MMA and epilogue warps: each unit that is not
// skipped takes buffer `next` (256 columns) and flips it; uses(b) counts the
// buffer's completed uses (its barrier phases).
struct AccSeq {
  int next = 0;
  uint32_t u0 = 0u, u1 = 0u;
  __device__ __forceinline__ uint32_t uses(int b) const { return b ? u1 : u0; }
  __device__ __forceinline__ void bump(int b) {
    if (b)
      ++u1;
    else
      ++u0;
  }
};

template <bool kReturn = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_fused_kernel(const __grid_constant__ CUtensorMap tmA_gu, const __grid_constant__ CUtensorMap tmB_gu,
                     const __grid_constant__ CUtensorMap tmA_dn, const __grid_constant__ CUtensorMap tmB_dn,
                     const __grid_constant__ CUtensorMap tmB_gu_full, const __grid_constant__ CUtensorMap tmB_dn_full,
                     const FusedArgs args) {
  using C = FusedCfg;
  extern __shared__ uint8_t fused_smem_raw[];
  __shared__ int4 tile_cache[kTileCache];
  __shared__ int tile_meta[2];
  __shared__ int unit_q[C::kUnitQueue];
  __shared__ __align__(8) uint64_t uq_full[C::kUnitQueue];
  __shared__ __align__(8) uint64_t uq_empty[C::kUnitQueue];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(fused_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint64_t* drain = acc_empty + 2;          // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* staging = reinterpret_cast<float*>(smem + C::kStages * C::kStageBytes + C::kBarrierBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    QMOE_TRACE_AT(1, 0);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(drain, 1);
    for (int q = 0; q < C::kUnitQueue; ++q) {
      mbar_init(&uq_full[q], 1);
      mbar_init(&uq_empty[q], 2);  // the MMA issuer and the epilogue
    }
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tmA_gu);
    prefetch_tmap(&tmB_gu);
    prefetch_tmap(&tmA_dn);
    prefetch_tmap(&tmB_dn);
    prefetch_tmap(&tmB_gu_full);
    prefetch_tmap(&tmB_dn_full);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x == 0) QMOE_TRACE_AT(1, 1);

  const TileView tv{args.tiles + 1, args.tiles + 1 + args.max_tiles, args.tiles + 1 + 2 * args.max_tiles, 0,
                    tile_cache};
  if (warp == 0) {
    const int cnt = args.tiles[0];
    int4 c = make_int4(0, 0, 0, 0);
    if (lane < args.max_tiles) c = make_int4(tv.exp[lane], tv.row0[lane], tv.rows[lane], 0);
    tile_cache[lane] = c;
    if (lane == 0) tile_meta[0] = min(cnt, args.max_tiles);
  }
  __syncthreads();
  const int ntiles = tile_meta[0];
  const int units_gu = ntiles * args.n_mt_gu;
  const int total_units = units_gu + ntiles * args.n_mt_dn;
  // unit u -> (gate/up?, tile, feature block) and its shape
  auto unit_of = [&](int u) {
    FusedUnit f;
    f.gu = u < units_gu;
    const int v = f.gu ? u : u - units_gu;
    const int n = f.gu ? args.n_mt_gu : args.n_mt_dn;
    f.tile = v / n;
    f.mt = v - f.tile * n;
    f.e = tv.expert(f.tile);
    f.row0 = tv.first_row(f.tile);
    f.rows = tv.nrows(f.tile);
    if (f.rows < 0 || f.rows > C::kMaxRows || f.row0 < 0 || f.row0 > args.n_rows - f.rows) f.rows = 0;
    f.nb = (f.rows + kBoxRows - 1) / kBoxRows;
    f.two = f.gu || args.dn_two;
    return f;
  };

  if (warp == 0 && args.gather_rows == nullptr) {
    // ---------------- TMA producer, permuted rows (lane 0 alone) ----------------
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      bool first = true;
      int* counter = args.done + args.max_tiles;
      int next_u = -2;  // -2: nothing claimed ahead yet
      for (int i = 0;; ++i) {
        const int q = i % C::kUnitQueue;
        if (!mbar_wait_bounded(&uq_empty[q], ((i / C::kUnitQueue) & 1) ^ 1u, abort_flag,
                               kDevErrWaitTimeoutProducer)) {
          ok = false;
          break;
        }
        int u = next_u == -2 ? int(blockIdx.x) : next_u;
        if (!ok || u >= total_units) u = -1;
        next_u = u >= 0 ? int(gridDim.x) + atomicAdd(counter, 1) : -1;
        unit_q[q] = u;
        mbar_arrive(&uq_full[q]);
        if (u < 0) break;
        const FusedUnit f = unit_of(u);
        if (f.rows == 0) {
          record_device_error(kDevErrBadIndex);
          continue;
        }
        const bool gu = f.gu;
        const int tile = f.tile, mt = f.mt, e = f.e, row0 = f.row0, nb = f.nb;
        if (!gu && !wait_tile_done(args.done + tile, args.n_mt_gu, abort_flag)) {
          ok = false;
          continue;  // the next slot carries the end marker
        }
        const CUtensorMap* ta = gu ? &tmA_gu : &tmA_dn;
        const CUtensorMap* tb = gu ? &tmB_gu : &tmB_dn;
        const bool two_a = f.two;
        const int a_row = gu ? e * args.a_rows_gu + mt * kBM : e * args.a_rows_dn + mt * kBM * (1 + args.dn_two);
        const int a2_row = a_row + (gu ? args.up_off : kBM);
        const int nkb = gu ? args.num_kb_gu : args.num_kb_dn;
        const uint32_t bytes = (two_a ? 2 : 1) * C::kABytes + nb * kBoxRows * kBK * 2;
        for (int kb = 0; kb < nkb; ++kb) {
          uint8_t* sb = stages + stage * C::kStageBytes;
          uint8_t* bs = sb + 2 * C::kABytes;
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, kDevErrWaitTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], bytes);
          tma_load_2d_hint(sb, ta, kb * kBK, a_row, &full[stage], pol_w);
          if (two_a) tma_load_2d_hint(sb + C::kABytes, ta, kb * kBK, a2_row, &full[stage], pol_w);
          if (args.full_boxes && nb == C::kMaxRows / kBoxRows)
            tma_load_2d_hint(bs, gu ? &tmB_gu_full : &tmB_dn_full, kb * kBK, row0, &full[stage], pol_x);
          else
            for (int b = 0; b < nb; ++b)
              tma_load_2d_hint(bs + b * (kBoxRows * kBK * 2), tb, kb * kBK, row0 + b * kBoxRows, &full[stage],
                               pol_x);
          if (first) {
            QMOE_TRACE_AT(1, 2);
            first = false;
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        for (int s = 0; s < C::kStages; ++s) {
          if ((issued_mask >> s) & 1u) {
            const unsigned long long t0 = globaltimer_ns();
            while (!mbar_try_wait(&full[s], (issued_parity >> s) & 1u)) {
              if (globaltimer_ns() - t0 > kWaitLimitNs) break;
            }
          }
        }
      }
    }
  } else if (warp == 0) {
    // ---------------- TMA producer, gathered rows (warp 0) ----------------
    // Lane 0 draws units, waits on the ring and issues the weight loads (and
    // the activation boxes of down units); for gate/up units each lane
    // issues one gather4 of 4 token rows per stage.
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const bool gather = args.gather_rows != nullptr;
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0, issued_parity = 0;
    bool ok = true;
    bool first = true;
    int* counter = args.done + args.max_tiles;
    int next_u = -2;  // lane 0: the unit claimed ahead (-2: none yet)
    for (int i = 0;; ++i) {
      const int q = i % C::kUnitQueue;
      int u = -1;
      int got = 1;
      if (lane == 0) {
        if (!mbar_wait_bounded(&uq_empty[q], ((i / C::kUnitQueue) & 1) ^ 1u, abort_flag,
                               kDevErrWaitTimeoutProducer)) {
          got = 0;
        } else {
          u = next_u == -2 ? int(blockIdx.x) : next_u;
          if (!ok || u >= total_units) u = -1;
          next_u = u >= 0 ? int(gridDim.x) + atomicAdd(counter, 1) : -1;
          unit_q[q] = u;
          mbar_arrive(&uq_full[q]);
        }
      }
      got = __shfl_sync(0xFFFFFFFFu, got, 0);
      u = __shfl_sync(0xFFFFFFFFu, u, 0);
      if (!got) {
        ok = false;
        break;
      }
      if (u < 0) break;
      const FusedUnit f = unit_of(u);
      if (f.rows == 0) {
        if (lane == 0) record_device_error(kDevErrBadIndex);
        continue;
      }
      const bool gu = f.gu;
      const int tile = f.tile, mt = f.mt, e = f.e, row0 = f.row0, nrows = f.rows, nb = f.nb;
      if (!gu) {
        int dep = 1;
        if (lane == 0) dep = wait_tile_done(args.done + tile, args.n_mt_gu, abort_flag);
        if (!__shfl_sync(0xFFFFFFFFu, dep, 0)) {
          ok = false;
          continue;  // the next slot carries the end marker
        }
      }
      const bool g4 = gu && gather;
      const int n_g4 = (nrows + 3) / 4;
      int src[4] = {0, 0, 0, 0};
      if (g4 && lane < n_g4) {
        const int last = args.gather_rows[row0 + nrows - 1];  // filler for rows past the tile
#pragma unroll
        for (int r = 0; r < 4; ++r) src[r] = lane * 4 + r < nrows ? args.gather_rows[row0 + lane * 4 + r] : last;
      }
      const CUtensorMap* ta = gu ? &tmA_gu : &tmA_dn;
      const CUtensorMap* tb = gu ? &tmB_gu : &tmB_dn;
      const bool two_a = f.two;
      const int a_row = gu ? e * args.a_rows_gu + mt * kBM : e * args.a_rows_dn + mt * kBM * (1 + args.dn_two);
      const int a2_row = a_row + (gu ? args.up_off : kBM);
      const int nkb = gu ? args.num_kb_gu : args.num_kb_dn;
      const uint32_t bytes =
          (two_a ? 2 : 1) * C::kABytes + (g4 ? n_g4 * 4 * kBK * 2 : nb * kBoxRows * kBK * 2);
      for (int kb = 0; kb < nkb; ++kb) {
        uint8_t* sb = stages + stage * C::kStageBytes;
        uint8_t* bs = sb + 2 * C::kABytes;
        int w_ok = 1;
        if (lane == 0) {
          w_ok = mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, kDevErrWaitTimeoutProducer);
          if (w_ok) {
            mbar_arrive_expect_tx(&full[stage], bytes);
            tma_load_2d_hint(sb, ta, kb * kBK, a_row, &full[stage], pol_w);
            if (two_a) tma_load_2d_hint(sb + C::kABytes, ta, kb * kBK, a2_row, &full[stage], pol_w);
            if (!g4 && args.full_boxes && nb == C::kMaxRows / kBoxRows)
              tma_load_2d_hint(bs, gu ? &tmB_gu_full : &tmB_dn_full, kb * kBK, row0, &full[stage], pol_x);
            else if (!g4)
              for (int b = 0; b < nb; ++b)
                tma_load_2d_hint(bs + b * (kBoxRows * kBK * 2), tb, kb * kBK, row0 + b * kBoxRows,
                                 &full[stage], pol_x);
            if (first) {
              QMOE_TRACE_AT(1, 2);
              first = false;
            }
          }
        }
        if (!__shfl_sync(0xFFFFFFFFu, w_ok, 0)) {
          ok = false;
          break;
        }
        // the expect_tx above precedes every gather's complete_tx
        if (g4 && lane < n_g4)
          tma_gather4_hint(bs + lane * 4 * (kBK * 2), tb, kb * kBK, src[0], src[1], src[2], src[3], &full[stage],
                           pol_x);
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      for (int s = 0; s < C::kStages; ++s) {
        if ((issued_mask >> s) & 1u) {
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[s], (issued_parity >> s) & 1u)) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      AccSeq acc;
      for (int local = 0; ok; ++local) {
        const int q = local % C::kUnitQueue;
        if (!mbar_wait_bounded(&uq_full[q], (local / C::kUnitQueue) & 1, abort_flag, kDevErrWaitTimeoutMma)) {
          ok = false;
          break;
        }
        const int u = unit_q[q];
        mbar_arrive(&uq_empty[q]);
        if (u < 0) break;
        const FusedUnit f = unit_of(u);
        if (f.rows == 0) continue;
        const uint32_t idesc = make_idesc_bf16(kBM, f.nb * kBoxRows);
        const int nkb = f.gu ? args.num_kb_gu : args.num_kb_dn;
        const bool two_a = f.two;
        const int buf = acc.next;
        if (!mbar_wait_bounded(&acc_empty[buf], (acc.uses(buf) & 1u) ^ 1u, abort_flag, kDevErrWaitTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem_base + buf * C::kAccCols;
        const uint32_t d1 = d0 + kBM;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, kDevErrWaitTimeoutMma)) {
            ok = false;
            break;
          }
          if (local == 0 && kb == 0) QMOE_TRACE_AT(1, 3);
          tc_fence_after();
          const uint32_t sb = smem_u32(stages + stage * C::kStageBytes);
          const uint32_t bsb = sb + 2 * C::kABytes;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            const uint32_t accum = (kb | k) != 0 ? 1u : 0u;
            const uint64_t bdesc = make_sw128_desc(bsb + k * kUmmaK * 2);
            umma_bf16(d0, make_sw128_desc(sb + k * kUmmaK * 2), bdesc, idesc, accum);
            if (two_a) umma_bf16(d1, make_sw128_desc(sb + C::kABytes + k * kUmmaK * 2), bdesc, idesc, accum);
          }
          umma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
        acc.bump(buf);
        acc.next = buf ^ 1;
      }
      if (!ok) *abort_flag = 1;
      QMOE_TRACE_AT(1, 4);
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
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;
    const int m = quad * 32 + lane;  // feature row inside the unit = TMEM lane
    const int et = threadIdx.x - 64;
    int32_t* meta_dst = reinterpret_cast<int32_t*>(staging + 4 * 16 * 33);
    float* meta_w = reinterpret_cast<float*>(meta_dst + C::kMaxRows);
    int32_t* meta_src = meta_dst + 2 * C::kMaxRows;
    __nv_bfloat16** meta_ptr = reinterpret_cast<__nv_bfloat16**>(meta_dst + 3 * C::kMaxRows);
    AccSeq acc;
    for (int local = 0;; ++local) {
      const int q = local % C::kUnitQueue;
      const bool got = mbar_wait_bounded(&uq_full[q], (local / C::kUnitQueue) & 1, abort_flag,
                                         kDevErrWaitTimeoutEpilogue);
      const int u = got ? unit_q[q] : -1;
      // all four warps have the unit (or give up together) before the slot is released
      if (named_barrier_or(1, 128, !got)) break;
      if (et == 0) mbar_arrive(&uq_empty[q]);
      if (u < 0) break;
      const FusedUnit f = unit_of(u);
      if (f.rows == 0) continue;  // skipped by every role
      const bool gu = f.gu;
      const int tile = f.tile, mt = f.mt, row0 = f.row0, nrows = f.rows, nb = f.nb;
      const int buf = acc.next;
      int my_dst = -1, my_src = 0;
      float my_w = 0.f;
      __nv_bfloat16* my_ptr = nullptr;
      if (!gu && et < nrows) {
        if constexpr (kReturn) {
          const int4 m4 = args.row_meta[row0 + et];
          my_w = __int_as_float(m4.x);
          my_src = (m4.y >= 0 && m4.y < args.n_ranks) ? m4.y : -1;
          my_dst = my_src >= 0 ? m4.z : -1;
          if (my_dst >= 0 && my_dst < args.n_acc)
            my_ptr = args.peer_ret[my_src] + (size_t(args.ret_row0) + my_dst) * args.acc_ld;
        } else {
          my_dst = args.row_dst[row0 + et];
          my_w = args.row_w[row0 + et];
        }
      }
      const bool ok = mbar_wait_bounded(&acc_full[buf], acc.uses(buf) & 1u, abort_flag, kDevErrWaitTimeoutEpilogue);
      if (named_barrier_or(1, 128, !ok)) break;
      if (local == 0 && et == 0) QMOE_TRACE_AT(1, 5);
      if (!gu) {
        meta_dst[et] = (my_dst >= 0 && my_dst < args.n_acc) ? my_dst : -1;
        meta_w[et] = my_w;
        meta_src[et] = my_src;
        if constexpr (kReturn) meta_ptr[et] = my_ptr;
        named_barrier_sync(1, 128);
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(quad * 32) << 16) + buf * C::kAccCols;
      const uint32_t tsecond = kBM;
      const int feat = mt * kBM + m;
      for (int c = 0; c < nb; ++c) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(taddr + c * 16, v);
        if (gu) {
          uint32_t up[16];
          tmem_ld_32x32b_x16(taddr + tsecond + c * 16, up);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = c * 16 + i;
            if (n < nrows) {
              const float g = __uint_as_float(v[i]);
              const float h = g / (1.0f + __expf(-g)) * __uint_as_float(up[i]);
              args.act[size_t(row0 + n) * args.act_ld + feat] = __float2bfloat16_rn(h);
            }
          }
        } else {
          for (int h = 0; h <= args.dn_two; ++h) {  // the unit's 128-feature halves
            if (h) tmem_ld_32x32b_x16(taddr + tsecond + c * 16, v);
            tmem_ld_wait();
            // transpose through shared memory: a lane then holds 4 consecutive
            // features of one row, added with one 16-byte vector reduction
            float* wsb = staging + (warp - 2) * (16 * 33);
#pragma unroll
            for (int i = 0; i < 16; ++i) wsb[i * 33 + lane] = __uint_as_float(v[i]);
            __syncwarp();
            if constexpr (kReturn) {
              // weighted row segments straight into the source ranks' return
              // buffers: a lane stores 8 consecutive features (16 bytes) of
              // one row, 8 rows per pass (row stride 33 words: conflict-free)
              const int f8 = (lane & 3) * 8;
              const int fcol = (mt * (1 + args.dn_two) + h) * kBM + quad * 32 + f8;
#pragma unroll
              for (int it = 0; it < 2; ++it) {
                const int i = it * 8 + (lane >> 2);
                const int n = c * 16 + i;
                if (n < nrows) {
                  __nv_bfloat16* ret = meta_ptr[n];
                  if (ret != nullptr) {
                    const float wv = meta_w[n];
                    const float* sv = wsb + i * 33 + f8;
                    uint4 pk;
                    uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                      const __nv_bfloat162 b2 = __floats2bfloat162_rn(wv * sv[2 * j], wv * sv[2 * j + 1]);
                      pw[j] = *reinterpret_cast<const uint32_t*>(&b2);
                    }
                    *reinterpret_cast<uint4*>(ret + fcol) = pk;
                  }
                }
              }
            } else {
              const int fq = (lane & 7) * 4;
              const int fcol = (mt * (1 + args.dn_two) + h) * kBM + quad * 32 + fq;
#pragma unroll
              for (int it = 0; it < 4; ++it) {
                const int i = it * 4 + (lane >> 3);
                const int n = c * 16 + i;
                if (n < nrows) {
                  const int dst = meta_dst[n];
                  if (dst >= 0) {
                    const float wv = meta_w[n];
                    red_add_v4_f32(args.acc + size_t(dst) * args.acc_ld + fcol, wv * wsb[i * 33 + fq],
                                   wv * wsb[i * 33 + fq + 1], wv * wsb[i * 33 + fq + 2], wv * wsb[i * 33 + fq + 3]);
                  }
                }
              }
            }
            __syncwarp();
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      acc.bump(buf);
      acc.next = buf ^ 1;
      if (gu) {
        // publish this unit's activation rows to the down units of the tile
        asm volatile("fence.proxy.async;" ::: "memory");
        __threadfence();
        named_barrier_sync(1, 128);
        if (et == 0) atom_add_release_gpu(args.done + tile, 1);
      }
    }
    if (threadIdx.x == 64) QMOE_TRACE_AT(1, 6);
  }

  if constexpr (kReturn) __threadfence_system();  // peer stores before the step's next signal
  __syncthreads();
  if (threadIdx.x == 0) QMOE_TRACE_AT(1, 7);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if (!kReturn && args.fin_out != nullptr &&
      grid_barrier_once(args.done + args.max_tiles + 1, kDevErrWaitTimeoutEpilogue)) {
    const long long n8 = (long long)args.n_acc * args.acc_ld / 8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
         i += (long long)gridDim.x * blockDim.x)
      finalize_vec8(args.acc, args.fin_residual, args.fin_out, i);
  }
}

}  // namespace qmoe
