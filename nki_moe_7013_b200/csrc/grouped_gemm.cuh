// K3a / K3b: persistent TMA + tcgen05 grouped GEMMs over expert tiles.
//
// Both kernels compute D = W_e[f0:f0+128, :] . X_tile^T ("swap AB"): the
// 128-row MMA M dimension runs over output features of one expert (weights
// are K-major in the (E, 2I, H) / (E, H, I) layout), and the MMA N dimension
// runs over the tile's token rows (16..128, a multiple of 16).  Decode tiles
// with a handful of tokens therefore cost one N=16 MMA column block while the
// weights stream from HBM at full width, and prefill tiles use N up to 128.
//
// Work unit = (tile, feature block).  Units are assigned round-robin to a
// persistent grid of one CTA per SM; consecutive CTAs share a tile so the
// tile's activation rows are reused from L2.
//
// Warp roles (192 threads):
//   warp 0      one lane issues TMA loads (weights evict-first, rows evict-last)
//   warp 1      allocates TMEM; one lane issues tcgen05.mma and commits
//   warps 2..5  epilogue: tcgen05.ld from TMEM (lane quadrant = warp % 4)
// The smem ring has kStages stages guarded by full/empty mbarriers; the TMEM
// accumulator is double-buffered so the epilogue of unit i overlaps the
// main loop of unit i+1.  Every wait is bounded (see mbar_wait_bounded).
//
// K3a (gate/up) issues two MMAs per k-step into two accumulators -- gate rows
// f0.. and up rows I+f0.. of the same expert -- so a thread's TMEM lane holds
// gate and up of the same feature and SiLU(gate)*up needs no exchange.
// K3b (down) multiplies each column (row r of the tile) by row_w[r] and adds
// it into the fp32 accumulator row row_dst[r] (the weighted combine) with
// 16-byte vector reductions.
//
// Split K.  With few units (decode batches) a unit's K range can be split
// over several CTAs so that more SMs stream weights.  Down: the partial sums
// meet in the fp32 accumulator (the combine is linear).  Gate/up (SiLU is
// not): each split stores its fp32 gate/up partials in a scratch slot and
// bumps the unit's arrival counter; the last CTA to arrive adds the S
// partials in split order (so the result does not depend on which CTA came
// last), applies SiLU(gate)*up and resets the counter to zero.
#pragma once

#include "common.cuh"

namespace qmoe {

constexpr int kBM = 128;       // MMA M: output features per unit
constexpr int kBK = 64;        // k elements per stage (one 128-byte swizzle row)
constexpr int kBNMax = 128;    // token rows per tile
constexpr int kBoxRows = 16;   // rows per activation TMA box
constexpr int kUmmaK = 16;     // k per tcgen05.mma (bf16)
constexpr int kGemmThreads = 192;
// GemmArgs::flags: the tile list was complete before the previous kernel on
// the stream started (true for the down GEMM after a gate/up GEMM on the same
// tiles), so a small-tile down GEMM may read it and stream weights before its
// dependency wait.
constexpr int kGemmTilesReady = 1;
// split-K scratch: kSplitSlots partial slots of [2][16 rows][128 features]
// fp32, then kSplitSlots arrival counters and 4 spare words (word kSplitSlots:
// the grid-barrier counter of the fused decode finalisation)
constexpr int kSplitSlots = 256;
constexpr int kSplitSlotFloats = 2 * kBoxRows * kBM;
// Per-tile unit counters of the decode forward (the down GEMM starts a tile
// once its gate/up units are done), after the arrival counters and spares.
constexpr int kSplitTileDoneWords = 260;
constexpr int kSplitTileDoneOffset = kSplitSlots + 4;
constexpr int kSplitCounterWords = kSplitTileDoneOffset + kSplitTileDoneWords;
constexpr size_t kSplitWorkspaceBytes = size_t(kSplitSlots) * kSplitSlotFloats * 4 + kSplitCounterWords * 4;

// Epilogue modes of the one GEMM kernel.
enum GemmMode : int {
  kModeDown = 0,    // weighted rows reduced into an fp32 accumulator (combine)
  kModeGateUp = 1,  // two accumulators (gate, up) -> bf16 SiLU(gate)*up
  kModePlain = 2,   // one accumulator -> bf16 store (dense projections)
  kModeDownReturn = 3,  // weighted bf16 rows stored into the source rank's return buffer (EP)
  kModePlainPair = 4,   // two accumulators (features f0.. and f0+128.. of a 256-feature unit) sharing
                        // the row operand -> bf16 stores (dense projections of prefill size)
};

// kSmall: every tile has at most 16 rows (decode batches).  A stage's
// activation slot and the TMEM accumulators shrink to 16 rows, so that a
// gate/up CTA and a down CTA fit on one SM together (shared memory and TMEM):
// the down GEMM, launched while the gate/up GEMM still runs, streams its
// weights into its ring before the gate/up results it multiplies exist.
template <int kMode, bool kSmall = false>
struct GemmCfg {
  static constexpr bool kGateUp = kMode == kModeGateUp;
  // two weight tiles per stage, two accumulators sharing the row tile
  static constexpr bool kTwoA = kGateUp || kMode == kModePlainPair;
  static constexpr int kATiles = kTwoA ? 2 : 1;
  static constexpr int kABytes = kBM * kBK * 2;           // 16 KB
  static constexpr int kBRows = kSmall ? kBoxRows : kBNMax;
  static constexpr int kBBytes = kBRows * kBK * 2;        // 16 KB (2 KB small)
  static constexpr int kStageBytes = kATiles * kABytes + kBBytes;
  // small plain GEMMs (decode projections) run alone: the deepest ring
  static constexpr int kStages =
      kTwoA ? (kSmall ? 3 : 4) : kMode == kModePlain ? (kSmall ? 10 : 6) : (kSmall ? 5 : 6);
  static constexpr int kUpCol = kSmall ? kBoxRows : kBM;  // TMEM column of the up accumulator
  static constexpr int kAccCols = kTwoA ? 2 * kUpCol : kBRows;  // TMEM columns per accumulator buffer
  static constexpr int kTmemCols = 2 * kAccCols < 32 ? 32 : 2 * kAccCols;
  static constexpr int kBarrierBytes = 256;
  // down epilogue: per epilogue warp a [16 rows][33] fp32 transpose buffer
  // (+ the tile's row destinations, weights and source ranks, 128 x 12 bytes)
  static constexpr bool kDownLike = kMode == kModeDown || kMode == kModeDownReturn;
  static constexpr int kStagingBytes = kDownLike ? 4 * 16 * 33 * 4 + 128 * 12 : 0;
  static constexpr int kSmemBytes =
      1024 /*align slack*/ + kStages * kStageBytes + kBarrierBytes + kStagingBytes;
};

struct GemmArgs {
  const int32_t* tiles;  // [0] = ntiles, then expert[max_tiles], row0[max_tiles], nrows[max_tiles];
                         // nullptr = dense: ceil(dense_rows/128) tiles of expert 0
  int max_tiles;
  int dense_rows;
  int n_mtiles;          // feature blocks per tile
  int num_kb;            // K / kBK
  int k_splits;          // down: >1 splits each (tile, feature block) unit over K (the
                         // partial sums meet in the fp32 accumulator)
  // gate/up: split-K scratch (kSplitWorkspaceBytes; counters zero on entry,
  // left zero on exit) and the most splits to use; the kernel picks the
  // count from the tile list (splits only when every tile has <= 16 rows)
  float* split_ws;
  int max_k_splits;
  int flags;             // kGemmTilesReady
  int full_boxes;        // 1: tmB_full maps whole 128-row tiles (one TMA load per stage for them)
  // gate/up: when non-null, each finished unit (after its activation rows are
  // written; the last split of a split unit) adds 1 to tile_done[tile].
  // down: when non-null, a tile's activation rows are loaded once
  // tile_done[tile] reaches tile_done_target (bounded wait) -- instead of
  // waiting for the whole previous grid, which runs concurrently.
  int* tile_done;
  int tile_done_target;
  // down: when fin_out is set, after one grid-wide barrier on *grid_bar (zero
  // before the launch) every CTA finalises a slice of the combine --
  // fin_out = bf16(acc + fin_residual), the finalize kernel folded in
  const __nv_bfloat16* fin_residual;
  __nv_bfloat16* fin_out;
  int* grid_bar;
  int a_rows_per_expert; // 2I (gate/up) or H (down)
  int up_row_offset;     // I (gate/up only)
  // gate/up: when non-null, B row r of a tile is row gather_rows[r] of the
  // source activations (TMA gather4 from x) instead of row r of x_perm
  const int32_t* gather_rows;
  // gate/up and plain epilogues: bf16 output rows
  __nv_bfloat16* act;
  int act_ld;
  // down epilogue
  const int32_t* row_dst;
  const float* row_w;
  float* acc;
  int acc_ld;
  int n_acc;
  // down-return (EP): per row {weight bits, source rank, return row, 0}; the
  // output row goes to peer_ret[source] + (ret_row0 + return row) * acc_ld
  const int4* row_meta;
  __nv_bfloat16* const* peer_ret;
  int ret_row0;
  int n_ranks;
};

// Tile accessors: the device-built tile list (its first kTileCache entries
// copied to shared memory), or a dense row range.
constexpr int kTileCache = 32;
struct TileView {
  const int32_t* exp;
  const int32_t* row0;
  const int32_t* rows;
  int dense_rows;
  const int4* cache;  // {expert, first row, rows, 0} of tiles [0, kTileCache)
  __device__ __forceinline__ int expert(int t) const { return exp ? (t < kTileCache ? cache[t].x : exp[t]) : 0; }
  __device__ __forceinline__ int first_row(int t) const {
    return exp ? (t < kTileCache ? cache[t].y : row0[t]) : t * kBNMax;
  }
  __device__ __forceinline__ int nrows(int t) const {
    return exp ? (t < kTileCache ? cache[t].z : rows[t]) : min(kBNMax, dense_rows - t * kBNMax);
  }
};

// Bounded wait for a tile's activations; false (and a device error) on time-out.
__device__ __forceinline__ bool wait_tile_done(const int* done, int target, volatile int* abort_flag) {
  const unsigned long long t0 = globaltimer_ns();
  while (ld_acquire_gpu(done) < target) {
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_device_error(kDevErrWaitTimeoutProducer);
      return false;
    }
    __nanosleep(64);
  }
  // the activation rows were written through the generic proxy by other SMs;
  // order them before this thread's TMA (async proxy) loads
  asm volatile("fence.proxy.async;" ::: "memory");
  return true;
}

// Work items of a launch.  Units (tile x feature block) fill whole grid
// waves unsplit (n_full of them); each unit of the last, partial wave is
// split over `split` CTAs along K, so the last wave keeps every SM busy
// instead of a few (decode: 312 gate/up units on 148 SMs ran 3 units deep,
// now 2 + 4 quarter units).  Item u (CTA u % grid, wave u / grid) is unit
// tm, split ks of nsplit.
struct WorkPlan {
  int n_full;  // unsplit units
  int split;   // splits of each remaining unit
  int total;   // work items
  __device__ __forceinline__ void item(int u, int& tm, int& ks, int& nsplit) const {
    if (u < n_full) {
      tm = u;
      ks = 0;
      nsplit = 1;
    } else {
      const int j = u - n_full;
      tm = n_full + j / split;
      ks = j - (j / split) * split;
      nsplit = split;
    }
  }
};

// Gate/up and plain launches: split the last partial wave's units over up to
// max_k_splits CTAs each (only when every tile has at most 16 rows and a
// scratch is given: the fixed-order fix-up needs one slot per split).
__device__ __forceinline__ WorkPlan gateup_work_plan(const GemmArgs& a, int ntiles, int max_rows) {
  const int units = max(0, ntiles) * a.n_mtiles;
  WorkPlan p{units, 1, units};
  if (a.split_ws == nullptr || a.max_k_splits < 2 || units <= 0 || max_rows > kBoxRows) return p;
  const int grid = int(gridDim.x);
  const int n_full = (units / grid) * grid;
  const int tail = units - n_full;
  if (tail == 0) return p;
  const int s = min(min(a.max_k_splits, a.num_kb), min(grid, kSplitSlots) / tail);
  if (s < 2) return p;
  return WorkPlan{n_full, s, n_full + tail * s};
}

// Split-K fix-up, run by the 128 epilogue threads of one split unit (tm, ks)
// after loading this split's partials into g (and u for gate/up: kTwo) --
// feature m, 16 rows.  tm: the unit's index among the split units.  Stores
// them into slot (tm, ks), counts the arrival, and returns true in the CTA
// that arrived last, with g / u replaced by the sums over the splits in
// split order.
template <bool kTwo = true>
__device__ __forceinline__ bool gateup_split_reduce(const GemmArgs& a, int tm, int ks, int nsplit, int m, int et,
                                                    float (&g)[16], float (&u)[16], volatile int* last_s) {
  float* slots = a.split_ws;
  int* arrivals = reinterpret_cast<int*>(slots + size_t(kSplitSlots) * kSplitSlotFloats);
  float* mine = slots + size_t(tm * nsplit + ks) * kSplitSlotFloats;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    __stcg(mine + i * kBM + m, g[i]);
    if (kTwo) __stcg(mine + (16 + i) * kBM + m, u[i]);
  }
  __threadfence();
  named_barrier_sync(1, 128);
  if (et == 0) {
    const int last = atom_add_acq_rel_gpu(arrivals + tm, 1) == nsplit - 1;
    if (last) arrivals[tm] = 0;  // every split has arrived: ready for the next launch
    *last_s = last;
  }
  named_barrier_sync(1, 128);
  if (!*last_s) return false;
  __threadfence();
  float gs[16], us[16];
  for (int s = 0; s < nsplit; ++s) {
    const float* p = slots + size_t(tm * nsplit + s) * kSplitSlotFloats;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float gv = s == ks ? g[i] : __ldcg(p + i * kBM + m);
      const float uv = !kTwo ? 0.f : s == ks ? u[i] : __ldcg(p + (16 + i) * kBM + m);
      gs[i] = s == 0 ? gv : gs[i] + gv;
      us[i] = s == 0 ? uv : us[i] + uv;
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    g[i] = gs[i];
    u[i] = us[i];
  }
  return true;
}

// Down GEMM, small tiles, tile list ready: issue the weight loads of the
// first ring stages before the dependency wait (one warp reads the tile list
// through L2; lane 0 issues).  Each stage's full barrier is armed with the
// stage's whole byte count (weights + activation rows); the activation loads
// follow in the main loop.  Returns the number of stages issued (lane 0; 0
// elsewhere, and 0 when some tile is too large for the small configuration,
// which the main path then refuses).
template <typename C>
__device__ __forceinline__ int down_pre_issue(const GemmArgs& a, const CUtensorMap* tmA, uint8_t* stages,
                                              uint64_t* full, int lane) {
  const int nt = min(__ldcg(a.tiles), a.max_tiles);
  const int32_t* t_exp = a.tiles + 1;
  const int32_t* t_rows = a.tiles + 1 + 2 * a.max_tiles;
  int mr = 0;
  for (int t = lane; t < nt; t += 32) mr = max(mr, __ldcg(t_rows + t));
  mr = __reduce_max_sync(0xFFFFFFFFu, mr);
  if (mr > kBoxRows || nt <= 0 || lane != 0) return 0;
  const int units = nt * a.n_mtiles;
  const int ksplit = max(1, min(min(a.k_splits, a.num_kb), int(gridDim.x) / units));
  const int total = units * ksplit;
  const uint64_t pol_w = policy_evict_first();
  int n = 0;
  for (int u = blockIdx.x; u < total && n < C::kStages; u += gridDim.x) {
    const int tm = u / ksplit, ks = u - tm * ksplit;
    const int tile = tm / a.n_mtiles, mt = tm - tile * a.n_mtiles;
    const int a_row = __ldcg(t_exp + tile) * a.a_rows_per_expert + mt * kBM;
    const uint32_t bytes = C::kABytes + kBoxRows * kBK * 2;  // one 16-row box (<= 16 rows)
    const int kb_end = (ks + 1) * a.num_kb / ksplit;
    for (int kb = ks * a.num_kb / ksplit; kb < kb_end && n < C::kStages; ++kb, ++n) {
      mbar_arrive_expect_tx(&full[n], bytes);
      tma_load_2d_hint(stages + n * C::kStageBytes, tmA, kb * kBK, a_row, &full[n], pol_w);
    }
  }
  return n;
}

template <int kMode, bool kSmall = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmB_full, const GemmArgs args) {
  using C = GemmCfg<kMode, kSmall>;
  constexpr bool kGateUp = C::kGateUp;
  extern __shared__ uint8_t gemm_smem_raw[];
  __shared__ int split_last;
  __shared__ int4 tile_cache[kTileCache];
  __shared__ int tile_meta[2];  // tile count, largest tile
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
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
  constexpr int kTid = kMode == kModeGateUp ? 1 : kMode == kModeDown ? 2 : -1;  // trace slot
  if constexpr (kTid >= 0) if (threadIdx.x == 0) QMOE_TRACE_AT(kTid, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Small-tile down GEMM with a tile list that predates the previous kernel:
  // the producer fills its ring with weight tiles now, while the previous
  // kernel (the gate/up GEMM producing this GEMM's activations) still runs;
  // their activation tiles follow after the wait.  Metadata is read through
  // L2 (ld.global.cg) since this precedes the wait.
  int n_pre = 0;
  if constexpr (kSmall && kMode == kModeDown) {
    if ((args.flags & kGemmTilesReady) && args.tiles != nullptr && warp == 0)
      n_pre = down_pre_issue<C>(args, &tmA, stages, full, lane);
  }
  // everything above overlapped the previous kernel; its outputs are read below
  // (a down GEMM with per-tile counters waits per tile in its producer instead)
  if (!(kMode == kModeDown && args.tile_done != nullptr)) griddep_wait();
  griddep_launch_dependents();
  if constexpr (kTid >= 0) if (threadIdx.x == 0) QMOE_TRACE_AT(kTid, 1);

  const TileView tv{args.tiles ? args.tiles + 1 : nullptr,
                    args.tiles ? args.tiles + 1 + args.max_tiles : nullptr,
                    args.tiles ? args.tiles + 1 + 2 * args.max_tiles : nullptr, args.dense_rows, tile_cache};
  // Tile metadata in one round trip: warp 0 reads the count and the first
  // kTileCache tiles together (lane l: tile l), keeps them in shared memory
  // and finds the largest tile (the small configuration holds 16 rows per
  // stage; gate/up splits K only over one-chunk tiles).
  if (warp == 0) {
    int nt, mr;
    if (args.tiles) {
      const int cnt = args.tiles[0];
      int4 c = make_int4(0, 0, 0, 0);
      if (lane < args.max_tiles) c = make_int4(tv.exp[lane], tv.row0[lane], tv.rows[lane], 0);
      nt = min(cnt, args.max_tiles);
      tile_cache[lane] = c;
      mr = lane < nt ? c.z : 0;
      for (int t = lane + kTileCache; t < nt; t += 32) mr = max(mr, tv.rows[t]);
      mr = __reduce_max_sync(0xFFFFFFFFu, mr);
    } else {
      nt = (args.dense_rows + kBNMax - 1) / kBNMax;
      mr = min(kBNMax, args.dense_rows);
    }
    if (lane == 0) {
      tile_meta[0] = nt;
      tile_meta[1] = mr;
    }
  }
  __syncthreads();
  int ntiles = tile_meta[0];
  const int max_rows = tile_meta[1];
  if (max_rows > C::kBRows) {
    if (threadIdx.x == 0) record_device_error(kDevErrBadIndex);
    ntiles = 0;  // refuse the launch rather than overrun a stage
  }
  WorkPlan plan{ntiles * args.n_mtiles, 1, ntiles * args.n_mtiles};
  if constexpr (kMode == kModeDown) {
    // as many splits (<= k_splits) of every unit as the grid runs at once
    // (the splits' partials meet in the fp32 accumulator)
    const int units = max(1, ntiles * args.n_mtiles);
    const int ksplit = max(1, min(min(args.k_splits, args.num_kb), int(gridDim.x) / units));
    plan = WorkPlan{0, ksplit, ntiles * args.n_mtiles * ksplit};
  }
  if constexpr (kGateUp || kMode == kModePlain || kMode == kModePlainPair)
    plan = gateup_work_plan(args, ntiles, max_rows);
  const int total_units = plan.total;

  if (warp == 0) {
    // ---------------- TMA producer (warp 0) ----------------
    // Lane 0 waits on the ring and issues the weight loads; with a gather,
    // every lane then issues one gather4 of 4 activation rows.
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const bool gather = kGateUp && args.gather_rows != nullptr;
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued_mask = 0;       // stages holding a load issued by this warp
    uint32_t issued_parity = 0;     // parity of that load's full-barrier phase
    bool ok = gather || lane == 0;  // box path: only lane 0 runs the loop
    int step = 0;                   // (unit, k-block) steps issued so far
    if (lane == 0)
      for (int s = 0; s < n_pre; ++s) issued_mask |= 1u << s;  // pre-issued: phase 0
    for (int u = blockIdx.x; ok && u < total_units; u += gridDim.x) {
      int tm, ks, nsplit;
      plan.item(u, tm, ks, nsplit);
      const int tile = tm / args.n_mtiles;
      const int mt = tm - tile * args.n_mtiles;
      const int e = tv.expert(tile);
      const int row0 = tv.first_row(tile);
      const int nrows = tv.nrows(tile);
      const int nb = (nrows + kBoxRows - 1) / kBoxRows;
      // a paired plain unit covers features [256 mt, 256 mt + 256): its second
      // weight tile sits up_row_offset (128) rows below the first
      const int a_row = e * args.a_rows_per_expert + mt * kBM * (kMode == kModePlainPair ? 2 : 1);
      const int n_g4 = (nrows + 3) / 4;
      int src[4] = {0, 0, 0, 0};
      if (gather && lane < n_g4) {
        const int last = args.gather_rows[row0 + nrows - 1];  // filler for rows past the tile
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int r = lane * 4 + q;
          src[q] = r < nrows ? args.gather_rows[row0 + r] : last;
        }
      }
      const uint32_t bytes = C::kATiles * C::kABytes +
                             (gather ? n_g4 * 4 * kBK * 2 : nb * kBoxRows * kBK * 2);
      if constexpr (kMode == kModeDown) {
        if (args.tile_done != nullptr && lane == 0 &&
            !wait_tile_done(args.tile_done + tile, args.tile_done_target, abort_flag)) {
          ok = false;
          break;
        }
      }
      const int kb_end = (ks + 1) * args.num_kb / nsplit;
      for (int kb = ks * args.num_kb / nsplit; kb < kb_end; ++kb) {
        uint8_t* sb = stages + stage * C::kStageBytes;
        uint8_t* bs = sb + C::kATiles * C::kABytes;
        if (!gather) {
          // box path: lane 0 alone runs the ring (no per-stage warp sync)
          if (lane == 0) {
            if (step >= n_pre) {
              if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, kDevErrWaitTimeoutProducer)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&full[stage], bytes);
              tma_load_2d_hint(sb, &tmA, kb * kBK, a_row, &full[stage], pol_w);
              if (C::kTwoA)
                tma_load_2d_hint(sb + C::kABytes, &tmA, kb * kBK, a_row + args.up_row_offset,
                                 &full[stage], pol_w);
            }  // else: weights and the byte count were issued before the wait
            if (!kSmall && args.full_boxes && nb == kBNMax / kBoxRows)
              tma_load_2d_hint(bs, &tmB_full, kb * kBK, row0, &full[stage], pol_x);
            else
              for (int b = 0; b < nb; ++b)
                tma_load_2d_hint(bs + b * (kBoxRows * kBK * 2), &tmB, kb * kBK, row0 + b * kBoxRows,
                                 &full[stage], pol_x);
          }
        } else {
          int w_ok = 1;
          if (lane == 0)
            w_ok = mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, kDevErrWaitTimeoutProducer);
          if (!__shfl_sync(0xFFFFFFFFu, w_ok, 0)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            mbar_arrive_expect_tx(&full[stage], bytes);
            tma_load_2d_hint(sb, &tmA, kb * kBK, a_row, &full[stage], pol_w);
            tma_load_2d_hint(sb + C::kABytes, &tmA, kb * kBK, a_row + args.up_row_offset, &full[stage],
                             pol_w);
          }
          __syncwarp();  // the expect_tx above precedes every gather's complete_tx
          if (lane < n_g4)
            tma_gather4_hint(bs + lane * 4 * (kBK * 2), &tmB, kb * kBK, src[0], src[1], src[2], src[3],
                             &full[stage], pol_x);
        }
        if constexpr (kTid >= 0) if (step == 0 && lane == 0) QMOE_TRACE_AT(kTid, 2);
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        ++step;
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && lane == 0) {
      // Let every load this warp issued land before the CTA's smem goes away.
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
      int local = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < total_units; u += gridDim.x, ++local) {
        int tm, ks, nsplit;
        plan.item(u, tm, ks, nsplit);
        const int tile = tm / args.n_mtiles;
        const int n_kb = (ks + 1) * args.num_kb / nsplit - ks * args.num_kb / nsplit;
        const int nb = (tv.nrows(tile) + kBoxRows - 1) / kBoxRows;
        const uint32_t idesc = make_idesc_bf16(kBM, nb * kBoxRows);
        const int buf = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&acc_empty[buf], acc_phase ^ 1u, abort_flag, kDevErrWaitTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_gate = tmem_base + buf * C::kAccCols;
        const uint32_t d_up = d_gate + C::kUpCol;
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, kDevErrWaitTimeoutMma)) {
            ok = false;
            break;
          }
          if constexpr (kTid >= 0) if (local == 0 && kb == 0) QMOE_TRACE_AT(kTid, 3);
          tc_fence_after();
          const uint32_t sb = smem_u32(stages + stage * C::kStageBytes);
          const uint32_t bsb = sb + C::kATiles * C::kABytes;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            const uint32_t accum = (kb | k) != 0 ? 1u : 0u;
            const uint64_t bdesc = make_sw128_desc(bsb + k * kUmmaK * 2);
            umma_bf16(d_gate, make_sw128_desc(sb + k * kUmmaK * 2), bdesc, idesc, accum);
            if (C::kTwoA)
              umma_bf16(d_up, make_sw128_desc(sb + C::kABytes + k * kUmmaK * 2), bdesc, idesc,
                        accum);
          }
          umma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
      }
      if constexpr (kTid >= 0) QMOE_TRACE_AT(kTid, 4);
      // Drain: every MMA issued above has completed once this barrier fires.
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
    const int et = threadIdx.x - 64;  // 0..127: epilogue thread index
    int32_t* meta_dst = reinterpret_cast<int32_t*>(staging + 4 * 16 * 33);
    float* meta_w = reinterpret_cast<float*>(meta_dst + 128);
    int32_t* meta_src = meta_dst + 256;
    int local = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++local) {
      int tm, ks, nsplit;
      plan.item(u, tm, ks, nsplit);
      const int su = tm - plan.n_full;  // split unit (slots, arrival counter)
      const int tile = tm / args.n_mtiles;
      const int mt = tm - tile * args.n_mtiles;
      const int row0 = tv.first_row(tile);
      const int nrows = tv.nrows(tile);
      const int nb = (nrows + kBoxRows - 1) / kBoxRows;
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // down: fetch the tile's row destinations / weights before waiting on the MMA
      int my_dst = -1, my_src = 0;
      float my_w = 0.f;
      if constexpr (kMode == kModeDown) {
        if (et < nrows) {
          my_dst = args.row_dst[row0 + et];
          my_w = args.row_w[row0 + et];
        }
      } else if constexpr (kMode == kModeDownReturn) {
        if (et < nrows) {
          const int4 mt4 = args.row_meta[row0 + et];
          my_w = __int_as_float(mt4.x);
          my_src = (mt4.y >= 0 && mt4.y < args.n_ranks) ? mt4.y : -1;
          my_dst = my_src >= 0 ? mt4.z : -1;
        }
      }
      const bool ok =
          mbar_wait_bounded(&acc_full[buf], acc_phase, abort_flag, kDevErrWaitTimeoutEpilogue);
      if constexpr (kTid >= 0) if (local == 0 && et == 0) QMOE_TRACE_AT(kTid, 5);
      // The four epilogue warps agree before going on, so a failed wait in one
      // of them can never leave the others waiting at a named barrier.  This
      // barrier also ends every read of the previous unit's row metadata.
      if (named_barrier_or(1, 128, !ok)) break;
      if constexpr (kMode == kModeDown) {
        meta_dst[et] = (my_dst >= 0 && my_dst < args.n_acc) ? my_dst : -1;
        meta_w[et] = my_w;
        named_barrier_sync(1, 128);
      } else if constexpr (kMode == kModeDownReturn) {
        meta_dst[et] = (my_dst >= 0 && my_dst < args.n_acc) ? my_dst : -1;
        meta_w[et] = my_w;
        meta_src[et] = my_src;
        named_barrier_sync(1, 128);
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t(quad * 32) << 16) + buf * C::kAccCols;
      const int feat = mt * kBM + m;
      for (int c = 0; c < nb; ++c) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(taddr + c * 16, v);
        if constexpr (kMode == kModePlain) {
          tmem_ld_wait();
          float g[16], unused[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) g[i] = __uint_as_float(v[i]);
          // split K (one 16-row chunk per unit): only the last split stores
          if (nsplit > 1 && !gateup_split_reduce<false>(args, su, ks, nsplit, m, et, g, unused, &split_last))
            break;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = c * 16 + i;
            if (n < nrows) args.act[size_t(row0 + n) * args.act_ld + feat] = __float2bfloat16_rn(g[i]);
          }
        } else if constexpr (kMode == kModePlainPair) {
          uint32_t hi[16];
          tmem_ld_32x32b_x16(taddr + C::kUpCol + c * 16, hi);
          tmem_ld_wait();
          const int f_lo = mt * 2 * kBM + m;  // this thread's features in the unit's two halves
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = c * 16 + i;
            if (n < nrows) {
              __nv_bfloat16* orow = args.act + size_t(row0 + n) * args.act_ld;
              orow[f_lo] = __float2bfloat16_rn(__uint_as_float(v[i]));
              orow[f_lo + kBM] = __float2bfloat16_rn(__uint_as_float(hi[i]));
            }
          }
        } else if constexpr (kGateUp) {
          uint32_t up[16];
          tmem_ld_32x32b_x16(taddr + C::kUpCol + c * 16, up);
          tmem_ld_wait();
          float g[16], uv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            g[i] = __uint_as_float(v[i]);
            uv[i] = __uint_as_float(up[i]);
          }
          // split K (one 16-row chunk per unit): only the last split finishes
          if (nsplit > 1 && !gateup_split_reduce(args, su, ks, nsplit, m, et, g, uv, &split_last))
            break;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = c * 16 + i;
            if (n < nrows) {
              const float h = g[i] / (1.0f + __expf(-g[i])) * uv[i];
              args.act[size_t(row0 + n) * args.act_ld + feat] = __float2bfloat16_rn(h);
            }
          }
        } else {
          tmem_ld_wait();
          // Each warp transposes its [32 features x 16 rows] block through
          // shared memory so that a lane holds 4 consecutive features of one
          // row, then adds them into acc[row_dst] with one 16-byte vector
          // reduction (red.global.add.v4.f32): 4 per lane per chunk.
          float* wsb = staging + (warp - 2) * (16 * 33);
#pragma unroll
          for (int i = 0; i < 16; ++i) wsb[i * 33 + lane] = __uint_as_float(v[i]);
          __syncwarp();
          const int fq = (lane & 7) * 4;        // feature offset inside the warp's 32
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int i = it * 4 + (lane >> 3);  // row inside the chunk
            const int n = c * 16 + i;
            if (n < nrows) {
              const int dst = meta_dst[n];
              if (dst >= 0) {
                const float wv = meta_w[n];
                if constexpr (kMode == kModeDownReturn) {
                  // weighted row segment straight into the source rank's return buffer
                  __nv_bfloat16* ret = args.peer_ret[meta_src[n]] +
                                       (size_t(args.ret_row0) + dst) * args.acc_ld + mt * kBM + quad * 32 + fq;
                  const __nv_bfloat162 lo = __floats2bfloat162_rn(wv * wsb[i * 33 + fq], wv * wsb[i * 33 + fq + 1]);
                  const __nv_bfloat162 hi =
                      __floats2bfloat162_rn(wv * wsb[i * 33 + fq + 2], wv * wsb[i * 33 + fq + 3]);
                  uint2 pk;
                  pk.x = *reinterpret_cast<const uint32_t*>(&lo);
                  pk.y = *reinterpret_cast<const uint32_t*>(&hi);
                  *reinterpret_cast<uint2*>(ret) = pk;
                } else {
                  red_add_v4_f32(args.acc + size_t(dst) * args.acc_ld + mt * kBM + quad * 32 + fq,
                                 wv * wsb[i * 33 + fq], wv * wsb[i * 33 + fq + 1],
                                 wv * wsb[i * 33 + fq + 2], wv * wsb[i * 33 + fq + 3]);
                }
              }
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      if constexpr (kGateUp) {
        if (args.tile_done != nullptr && (nsplit == 1 || split_last)) {
          // publish the unit's activation rows to the down GEMM's producer
          asm volatile("fence.proxy.async;" ::: "memory");
          __threadfence();
          named_barrier_sync(1, 128);
          if (et == 0) atom_add_release_gpu(args.tile_done + tile, 1);
        }
      }
    }
  }

  if constexpr (kTid >= 0) if (threadIdx.x == 64) QMOE_TRACE_AT(kTid, 6);
  if constexpr (kMode == kModeDownReturn) __threadfence_system();  // peer stores before the next signal
  __syncthreads();
  if constexpr (kTid >= 0) if (threadIdx.x == 0) QMOE_TRACE_AT(kTid, 7);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if constexpr (kMode == kModeDown) {
    if (args.fin_out != nullptr && grid_barrier_once(args.grid_bar, kDevErrWaitTimeoutEpilogue)) {
      const long long n8 = (long long)args.n_acc * args.acc_ld / 8;
      for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
           i += (long long)gridDim.x * blockDim.x)
        finalize_vec8(args.acc, args.fin_residual, args.fin_out, i);
    }
  }
}

}  // namespace qmoe
