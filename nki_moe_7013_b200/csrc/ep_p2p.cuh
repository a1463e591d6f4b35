// Expert parallelism over peer memory (NVLink / NVSwitch), no host sync.
//
// Every rank maps its peers' EP buffers (CUDA IPC) and a step runs as:
//
//   1. ep_exchange_counts (1 CTA): my per-expert row counts -> row `me` of
//      every peer's count matrix, then a flag; wait for all N rows; derive
//        dest_base[e]  first row of my rows of expert e in the receive buffer
//                      of e's rank (rows there are grouped by expert, then by
//                      source rank, then by token),
//        the tile list of my local experts over my receive buffer, and the
//        number of rows I receive;
//   2. ep_dispatch: each token row crosses to every rank that owns one of
//      its experts ONCE (peer stores into that rank's token buffer, at a
//      fixed row per (parity, source rank, token)), and each (token, slot)
//      leaves its meta in the destination's expert-grouped receive list:
//      routing weight, return address (source rank, token*k + slot) and the
//      token buffer row (a token whose 8 experts sit on 5 ranks sends 5
//      rows instead of 8);
//   3. ep_wait_expand: flag every peer "my rows are in your buffer", wait for
//      everyone's flag, then copy each receive-list entry's token row into
//      the expert-grouped receive rows (local memory, so the expert kernel
//      reads whole 128-row tiles with one TMA box per stage);
//   4. grouped gate/up + down GEMMs on the receive buffer; the down epilogue
//      writes each weighted bf16 row back into the SOURCE rank's return
//      buffer through peer stores (the combine, fused into the GEMM);
//   5. ep_wait_unpack: flag "your rows are back" to every peer, wait for
//      every peer's flag, then sum the k returned rows of every token in fp32
//      (+ residual), all CTAs; the step's device counter advances here.
//
// Receive / return buffers and the control block have two halves used on
// alternate steps (parity), so a fast rank can never overwrite data a peer
// is still reading: writing parity p of step i+2 requires the peer's step
// i+2 counts, which the peer publishes only after finishing step i.
//
// Step epochs: the flags carry the step number (epoch), so a flag from an
// older step never satisfies a newer wait.  A caller passes the epoch, or 0
// to use the rank's own device-side step counter (the last word of its
// control block, advanced by the step's final signal kernel): then a step is
// a fixed sequence of kernels with fixed arguments per parity, and two CUDA
// graphs (one per parity) replay the steps alternately.
//
// Every cross-GPU wait is bounded (kWaitLimitNs); on time-out the kernel
// records a device error and returns.  Peer memory is touched only by plain
// loads and stores and by release/acquire flags; no load is broadcast
// across a cluster.
#pragma once

#include "common.cuh"

namespace qmoe {

// Control block of one rank (int32 words); per parity half:
//   counts[N][E] | flag_counts[N] | flag_dispatch[N] | flag_combine[N]
__host__ __device__ __forceinline__ size_t ep_ctrl_words_per_parity(int N, int E) {
  return size_t(N) * E + 3 * size_t(N);
}
enum EpFlagKind : int { kEpFlagCounts = 0, kEpFlagDispatch = 1, kEpFlagCombine = 2 };

// Index of the device-side step counter (after both parity halves); the
// word after it counts the CTAs of ep_wait_unpack that have read the epoch,
// the next two carry the epochs whose returned rows (ep_wait_unpack) and
// dispatched rows (ep_wait_expand) have all landed.
__host__ __device__ __forceinline__ size_t ep_step_word(int N, int E) { return 2 * ep_ctrl_words_per_parity(N, E); }

// The step's epoch: the caller's, or (epoch == 0) the device counter + 1.
// Its parity must be p (the caller's buffers); false + device error if not.
__device__ __forceinline__ bool ep_resolve_epoch(const int* my_ctrl, int N, int E, int p, int& epoch) {
  if (epoch == 0) epoch = *reinterpret_cast<const volatile int*>(my_ctrl + ep_step_word(N, E)) + 1;
  if ((epoch & 1) != p) {
    record_device_error(kDevErrBadIndex);
    return false;
  }
  return true;
}

__device__ __forceinline__ size_t ep_flag_word(int N, int E, int p, int kind, int s) {
  return p * ep_ctrl_words_per_parity(N, E) + size_t(N) * E + size_t(kind) * N + s;
}

__device__ __forceinline__ void st_release_sys(int* ptr, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* ptr) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(int* ptr, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
// Spin (bounded) until *flag >= epoch on a word of this GPU written by this
// GPU.  Returns false and records `code` on time-out.
__device__ __forceinline__ bool ep_wait_flag_gpu(const int* flag, int epoch, unsigned int code) {
  const unsigned long long t0 = globaltimer_ns();
  while (ld_acquire_gpu(flag) < epoch) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_device_error(code);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Spin (bounded) until *flag >= epoch.  Returns false and records `code` on
// time-out.
__device__ __forceinline__ bool ep_wait_flag(const int* flag, int epoch, unsigned int code) {
  const unsigned long long t0 = globaltimer_ns();
  while (ld_acquire_sys(flag) < epoch) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_device_error(code);
      return false;
    }
    __nanosleep(100);
  }
  return true;
}

constexpr unsigned int kDevErrPeerTimeout = 5;

// Write `epoch` into flag (kind, p, me) of every peer, then wait until every
// peer has written flag (kind, p, s) of mine.  One warp.
__device__ __forceinline__ bool ep_signal_and_wait(int* const* peer_ctrl, int* my_ctrl, int N, int E, int me,
                                                   int p, int kind, int epoch) {
  const int lane = threadIdx.x & 31;
  __threadfence_system();
  __syncwarp();
  for (int d = lane; d < N; d += 32) st_release_sys(peer_ctrl[d] + ep_flag_word(N, E, p, kind, me), epoch);
  bool ok = true;
  for (int s = lane; s < N; s += 32) ok &= ep_wait_flag(my_ctrl + ep_flag_word(N, E, p, kind, s), epoch, kDevErrPeerTimeout);
  ok = __all_sync(0xFFFFFFFFu, ok);
  __threadfence_system();
  return ok;
}

// Exclusive scan of one int per thread over the CTA (blockDim.x a multiple
// of 32, at most 1024); *total = the sum.  warp_sums: 32 ints of shared
// memory.  Every thread of the CTA must call it.
__device__ __forceinline__ int ep_block_exclusive_scan(int v, int* total, int* warp_sums) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(0xFFFFFFFFu, incl, off);
    if (lane >= off) incl += n;
  }
  __syncthreads();  // warp_sums free from any earlier use
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int ws = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(0xFFFFFFFFu, ws, off);
      if (lane >= off) ws += n;
    }
    if (lane < nw) warp_sums[lane] = ws;
  }
  __syncthreads();
  *total = warp_sums[nw - 1];
  return (warp > 0 ? warp_sums[warp - 1] : 0) + incl - v;
}

// ---------------------------------------------------------------------------
// 1. count exchange (one CTA of 256 threads; E <= 256, N <= 32)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    ep_exchange_counts_kernel(const int32_t* __restrict__ counts, int* const* __restrict__ peer_ctrl,
                              int* __restrict__ my_ctrl, int me, int N, int E, int e_local, int p, int epoch,
                              int32_t* __restrict__ dest_base, int32_t* __restrict__ tiles, int max_tiles,
                              int32_t* __restrict__ recv_rows, int cap_rows, int32_t* __restrict__ zero_words,
                              int n_zero_words) {
  __shared__ int tot[256];
  __shared__ int expert_off[257];
  __shared__ int scan_s[32];
  __shared__ int ok_s;
  const int tid = threadIdx.x;
  griddep_wait();
  // scratch the step's expert kernel needs zeroed (its tile counters)
  for (int i = tid; i < n_zero_words; i += blockDim.x) zero_words[i] = 0;
  if (!ep_resolve_epoch(my_ctrl, N, E, p, epoch)) {
    if (tid == 0) {
      tiles[0] = 0;
      recv_rows[0] = 0;
    }
    return;
  }
  // my counts row into every peer's matrix
  for (int i = tid; i < N * E; i += blockDim.x) {
    const int d = i / E, e = i - d * E;
    peer_ctrl[d][size_t(p) * ep_ctrl_words_per_parity(N, E) + size_t(me) * E + e] = counts[e];
  }
  __threadfence_system();
  __syncthreads();
  if (tid < 32) {
    const bool ok = ep_signal_and_wait(peer_ctrl, my_ctrl, N, E, me, p, kEpFlagCounts, epoch);
    if (tid == 0) ok_s = ok;
  }
  __syncthreads();
  if (!ok_s) {
    // leave an empty tile list and zero received rows so later kernels do nothing
    if (tid == 0) {
      tiles[0] = 0;
      recv_rows[0] = 0;
    }
    return;
  }
  const volatile int* M = my_ctrl + size_t(p) * ep_ctrl_words_per_parity(N, E);
  // thread e (E <= 256 = blockDim.x): expert e's rows over all sources
  const int tot_e = tid < E ? [&] {
    int t = 0;
    for (int s = 0; s < N; ++s) t += M[s * E + tid];
    return t;
  }()
                            : 0;
  if (tid < E) tot[tid] = tot_e;
  // row offset of each expert inside its owner's receive buffer: an exclusive
  // scan of the totals, less the scan at the owner's first expert
  int all = 0;
  const int excl = ep_block_exclusive_scan(tot_e, &all, scan_s);
  if (tid < E) expert_off[tid] = excl;
  __syncthreads();
  const int off_e = tid < E ? excl - expert_off[(tid / e_local) * e_local] : 0;
  __syncthreads();
  if (tid < E) expert_off[tid] = off_e;
  // tiles of my local experts: thread le writes expert me*e_local + le's
  // 128-row tiles after those of the local experts before it
  const int e_mine = me * e_local + tid;
  const int tot_mine = tid < e_local ? tot[e_mine] : 0;
  const int nt_e = (tot_mine + 127) / 128;
  int nt = 0;
  const int first_tile = ep_block_exclusive_scan(nt_e, &nt, scan_s);
  if (tid < e_local) {
    for (int j = 0; j < nt_e; ++j) {
      const int i = first_tile + j;
      if (i < max_tiles) {
        tiles[1 + i] = tid;
        tiles[1 + max_tiles + i] = expert_off[e_mine] + j * 128;
        tiles[1 + 2 * max_tiles + i] = min(128, tot_mine - j * 128);
      }
    }
  }
  if (tid == 0) {
    tiles[0] = min(nt, max_tiles);
    const int last = me * e_local + e_local - 1;  // my rows end where my last expert's do
    recv_rows[0] = expert_off[last] + tot[last];
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    int before = 0;
    for (int s = 0; s < me; ++s) before += M[s * E + e];
    const int b = expert_off[e] + before;
    dest_base[e] = b;
    if (b + counts[e] > cap_rows) record_device_error(kDevErrBadIndex);
  }
}

// ---------------------------------------------------------------------------
// 2. dispatch: one warp per (token, slot), grid-stride
//   token buffer row of (parity p, source me, token t): (p*N + me)*max_tokens + t
//   receive-list meta = {weight bits, source rank, token*k + slot, token buffer row}
//   The row itself is stored by the warp of the token's first slot on each
//   destination rank (experts of one token are distinct; slots are few).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    ep_dispatch_kernel(const __nv_bfloat16* __restrict__ x, const int32_t* __restrict__ topk_idx,
                       const float* __restrict__ topk_w, const int32_t* __restrict__ slot_row,
                       const int32_t* __restrict__ offsets, const int32_t* __restrict__ dest_base,
                       __nv_bfloat16* const* __restrict__ peer_tok, int4* const* __restrict__ peer_recv_meta,
                       int T, int k, int H, int e_local, int me, int N, int p, int cap_rows, int max_tokens) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x / 32);
  const int vec = H / 8;  // 16-byte vectors per row
  for (int i = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); i < T * k; i += warps) {
    const int t = i / k;
    const int j = i - t * k;
    const int e = topk_idx[i];
    const int d = e / e_local;
    const int row = dest_base[e] + (slot_row[i] - offsets[e]);
    if (row < 0 || row >= cap_rows || d < 0 || d >= N || t >= max_tokens) {
      if (lane == 0) record_device_error(kDevErrBadIndex);
      continue;
    }
    const int xrow = (p * N + me) * max_tokens + t;
    bool first = true;
    for (int jj = 0; jj < j; ++jj) first &= topk_idx[t * k + jj] / e_local != d;
    if (first) {
      const uint4* src = reinterpret_cast<const uint4*>(x + size_t(t) * H);
      uint4* dst = reinterpret_cast<uint4*>(peer_tok[d] + size_t(xrow) * H);
      for (int v = lane; v < vec; v += 32) dst[v] = src[v];
    }
    if (lane == 0)
      peer_recv_meta[d][size_t(p) * cap_rows + row] = make_int4(__float_as_int(topk_w[i]), me, i, xrow);
  }
  __threadfence_system();
}

// ---------------------------------------------------------------------------
// 3. signal, wait, expand: CTA 0 flags every peer "my rows are in your
// buffer"; every CTA waits (bounded) for every peer's flag, then the CTAs copy
// receive-list entry r's token row into receive row r (one warp per two rows,
// grid-stride; every 16-byte load of both rows is issued before the first
// store, so a warp keeps 8 KB in flight; rows past recv_rows are left alone).
// On a time-out the rows are not copied (the device error is set; the step's
// results are void).  kV: 16-byte vectors per lane per row (H = 256 * kV).
// ---------------------------------------------------------------------------
template <int kV>
__device__ __forceinline__ void ep_expand_rows(const __nv_bfloat16* __restrict__ tok, int tok_rows,
                                               const int4* __restrict__ recv_meta, __nv_bfloat16* __restrict__ recv_x,
                                               int n, int H, int lane, int gw, int nw) {
  for (int r0 = 2 * gw; r0 < n; r0 += 2 * nw) {
    int xr[2];
    bool ok[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      xr[u] = r0 + u < n ? __ldcg(&recv_meta[r0 + u].w) : -1;
      ok[u] = xr[u] >= 0 && xr[u] < tok_rows;
      if (r0 + u < n && !ok[u] && lane == 0) record_device_error(kDevErrBadIndex);
    }
    uint4 v[2][kV];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint4* src = reinterpret_cast<const uint4*>(tok + size_t(ok[u] ? xr[u] : 0) * H);
#pragma unroll
      for (int i = 0; i < kV; ++i) v[u][i] = ok[u] ? __ldcg(src + lane + 32 * i) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!ok[u]) continue;
      uint4* dst = reinterpret_cast<uint4*>(recv_x + size_t(r0 + u) * H);
#pragma unroll
      for (int i = 0; i < kV; ++i) dst[lane + 32 * i] = v[u][i];
    }
  }
}

__global__ void __launch_bounds__(256)
    ep_wait_expand_kernel(int* const* __restrict__ peer_ctrl, int* __restrict__ my_ctrl, int N, int E, int me,
                          int p, int epoch, const __nv_bfloat16* __restrict__ tok, int tok_rows,
                          const int4* __restrict__ recv_meta, __nv_bfloat16* __restrict__ recv_x,
                          const int32_t* __restrict__ recv_rows, int cap_rows, int H) {
  __shared__ int ok_s;
  griddep_wait();
  griddep_launch_dependents();
  if (!ep_resolve_epoch(my_ctrl, N, E, p, epoch)) return;
  const int lane = threadIdx.x & 31;
  // CTA 0 signals and waits for the peers (system scope), then publishes the
  // epoch in a local word the other CTAs wait on at GPU scope
  int* local_go = my_ctrl + ep_step_word(N, E) + 3;
  if (threadIdx.x < 32) {
    bool ok = true;
    if (blockIdx.x == 0) {
      __threadfence_system();
      __syncwarp();
      for (int d = lane; d < N; d += 32)
        st_release_sys(peer_ctrl[d] + ep_flag_word(N, E, p, kEpFlagDispatch, me), epoch);
      for (int s = lane; s < N; s += 32)
        ok &= ep_wait_flag(my_ctrl + ep_flag_word(N, E, p, kEpFlagDispatch, s), epoch, kDevErrPeerTimeout);
      ok = __all_sync(0xFFFFFFFFu, ok);
      __threadfence_system();
      if (ok && lane == 0) st_release_gpu(local_go, epoch);
    } else if (lane == 0) {
      ok = ep_wait_flag_gpu(local_go, epoch, kDevErrPeerTimeout);
    }
    if (lane == 0) ok_s = ok;
  }
  __syncthreads();
  if (!ok_s) return;
  const int n = min(recv_rows[0], cap_rows);
  const int nw = gridDim.x * (blockDim.x / 32);
  const int gw = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (H == 2048) {
    ep_expand_rows<8>(tok, tok_rows, recv_meta, recv_x, n, H, lane, gw, nw);
  } else if (H == 4096) {
    ep_expand_rows<16>(tok, tok_rows, recv_meta, recv_x, n, H, lane, gw, nw);
  } else {
    const int vec = H / 8;
    for (int r = gw; r < n; r += nw) {
      const int xrow = __ldcg(&recv_meta[r].w);
      if (xrow < 0 || xrow >= tok_rows) {
        if (lane == 0) record_device_error(kDevErrBadIndex);
        continue;
      }
      const uint4* src = reinterpret_cast<const uint4*>(tok + size_t(xrow) * H);
      uint4* dst = reinterpret_cast<uint4*>(recv_x + size_t(r) * H);
      for (int v = lane; v < vec; v += 32) dst[v] = __ldcg(src + v);
    }
  }
}

// ---------------------------------------------------------------------------
// 5. signal, wait, unpack: CTA 0 flags every peer "your rows are back"; every
// CTA waits (bounded) for every peer's flag, then one warp per (token,
// 256-column slab), grid-stride, sums the token's k returned rows in fp32,
// adds the residual and stores bf16.  With the device epoch (epoch == 0) the
// step counter advances once every CTA has read it: the last CTA to arrive
// (counted in the word after the counter, which it resets) writes it.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    ep_wait_unpack_kernel(int* const* __restrict__ peer_ctrl, int* __restrict__ my_ctrl, int N, int E, int me,
                          int p, int epoch, const __nv_bfloat16* __restrict__ y_back,
                          const __nv_bfloat16* __restrict__ residual, int T, int H, int k,
                          __nv_bfloat16* __restrict__ out) {
  __shared__ int ok_s, epoch_s;
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x == 0) {
    // thread 0 alone reads the counter; the CTA's last reader advances it
    const bool device_epoch = epoch == 0;
    int ep = epoch;
    const bool epoch_ok = ep_resolve_epoch(my_ctrl, N, E, p, ep);
    epoch_s = epoch_ok ? ep : -1;
    if (device_epoch) {
      int* arrive = my_ctrl + ep_step_word(N, E) + 1;
      __threadfence();
      if (atomicAdd(arrive, 1) == int(gridDim.x) - 1) {
        *arrive = 0;
        if (epoch_ok) my_ctrl[ep_step_word(N, E)] = ep;
      }
    }
  }
  __syncthreads();
  if (epoch_s < 0) return;
  epoch = epoch_s;
  const int lane = threadIdx.x & 31;
  // CTA 0 signals the peers and waits for theirs (system scope), then
  // publishes the epoch in a local word; the other CTAs wait on that word at
  // GPU scope (the peers' stores happen before CTA 0's acquire, which comes
  // before its release of the word)
  int* local_go = my_ctrl + ep_step_word(N, E) + 2;
  if (threadIdx.x < 32) {
    bool ok = true;
    if (blockIdx.x == 0) {
      __threadfence_system();
      __syncwarp();
      for (int d = lane; d < N; d += 32)
        st_release_sys(peer_ctrl[d] + ep_flag_word(N, E, p, kEpFlagCombine, me), epoch);
      for (int s = lane; s < N; s += 32)
        ok &= ep_wait_flag(my_ctrl + ep_flag_word(N, E, p, kEpFlagCombine, s), epoch, kDevErrPeerTimeout);
      ok = __all_sync(0xFFFFFFFFu, ok);
      __threadfence_system();
      if (ok && lane == 0) st_release_gpu(local_go, epoch);
    } else if (lane == 0) {
      ok = ep_wait_flag_gpu(local_go, epoch, kDevErrPeerTimeout);
    }
    if (lane == 0) ok_s = ok;
  }
  __syncthreads();
  if (!ok_s) return;
  const int slabs = H / 256;
  const int nw = gridDim.x * (blockDim.x / 32);
  for (int w = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); w < T * slabs; w += nw) {
    const int t = w / slabs;
    const int col = (w - t * slabs) * 256 + lane * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // the first 8 rows' loads all in flight before the sums (slot order kept)
    uint4 rv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < k) rv[j] = __ldcg(reinterpret_cast<const uint4*>(y_back + (size_t(t) * k + j) * H + col));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= k) break;
      const uint32_t u[4] = {rv[j].x, rv[j].y, rv[j].z, rv[j].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += bf16lo_to_f32(u[q]);
        acc[2 * q + 1] += bf16hi_to_f32(u[q]);
      }
    }
    for (int j = 8; j < k; ++j) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(y_back + (size_t(t) * k + j) * H + col));
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += bf16lo_to_f32(u[q]);
        acc[2 * q + 1] += bf16hi_to_f32(u[q]);
      }
    }
    if (residual) {
      const uint4 v = *reinterpret_cast<const uint4*>(residual + size_t(t) * H + col);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += bf16lo_to_f32(u[q]);
        acc[2 * q + 1] += bf16hi_to_f32(u[q]);
      }
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat162 b2 = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
      ow[q] = *reinterpret_cast<const uint32_t*>(&b2);
    }
    *reinterpret_cast<uint4*>(out + size_t(t) * H + col) = o;
  }
}

// ---------------------------------------------------------------------------
// 4. signal + wait (one warp)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(32)
    ep_signal_wait_kernel(int* const* __restrict__ peer_ctrl, int* __restrict__ my_ctrl, int N, int E, int me,
                          int p, int kind, int epoch) {
  griddep_wait();
  const bool device_epoch = epoch == 0;
  if (!ep_resolve_epoch(my_ctrl, N, E, p, epoch)) return;
  const bool ok = ep_signal_and_wait(peer_ctrl, my_ctrl, N, E, me, p, kind, epoch);
  // the step's last wait: advance the device step counter
  if (ok && device_epoch && kind == kEpFlagCombine && threadIdx.x == 0) my_ctrl[ep_step_word(N, E)] = epoch;
}

}  // namespace qmoe
