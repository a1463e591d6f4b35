// Shared device helpers for the sm_100a kernels: bf16 conversion, mbarriers,
// TMA (tiled cp.async.bulk.tensor loads into this CTA only), tcgen05 / TMEM,
// and the bounded-wait error protocol.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qmoe.h"

namespace qmoe {

// ---------------------------------------------------------------------------
// Device-side error word.  A kernel that gives up on a bounded wait records a
// code here (first writer wins) and returns instead of hanging; the host reads
// it with qmoe_device_error().
// ---------------------------------------------------------------------------
__device__ unsigned int g_device_error = 0;

enum DeviceErrorCode : unsigned int {
  kDevErrNone = 0,
  kDevErrWaitTimeoutProducer = 1,
  kDevErrWaitTimeoutMma = 2,
  kDevErrWaitTimeoutEpilogue = 3,
  kDevErrBadIndex = 4,
};

__device__ __forceinline__ void record_device_error(unsigned int code) {
  atomicCAS(&g_device_error, 0u, code);
}

// Wall-clock limit of every spin-wait in these kernels.  Legitimate waits are
// microseconds; a second means a broken pipeline.
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Optional timeline instrumentation (build with -DQMOE_TRACE): kernels stamp
// %globaltimer at a few points per CTA into g_qmoe_trace[kernel][cta][event],
// read back with qmoe_trace_read.  Compiled out otherwise.
// kernel slots: 0 router / route_small, 1 gate/up, 2 down, 3 finalize,
// 4 permute scan, 5 permute scatter
constexpr int kTraceKernels = 6, kTraceCtas = 160, kTraceEvents = 8;
#ifdef QMOE_TRACE
__device__ unsigned long long g_qmoe_trace[kTraceKernels * kTraceCtas * kTraceEvents];
#define QMOE_TRACE_AT(kid, ev)                                                                   \
  do {                                                                                           \
    if (blockIdx.x < kTraceCtas) g_qmoe_trace[((kid) * kTraceCtas + blockIdx.x) * kTraceEvents + (ev)] = \
        globaltimer_ns();                                                                        \
  } while (0)
#else
#define QMOE_TRACE_AT(kid, ev) \
  do {                         \
  } while (0)
#endif

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Kernels of the MoE chain are launched with
// programmatic stream serialization: each waits for its predecessor's grid
// (griddepcontrol.wait) before reading what it produced, and lets its own
// dependents start launching as soon as all of its CTAs are resident.  Both
// are no-ops for a kernel launched without the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// bf16 helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16lo_to_f32(uint32_t packed) {
  return __uint_as_float(packed << 16);
}
__device__ __forceinline__ float bf16hi_to_f32(uint32_t packed) {
  return __uint_as_float(packed & 0xFFFF0000u);
}

// One step of an RMSNorm sum of squares: ss + (((a*a + b*b) + c*c) + d*d)
// with the rounding fixed (one multiply, three fused multiply-adds, one add),
// so every kernel that normalises a row in the same lane layout gets the
// same bits whatever the compiler would contract.
__device__ __forceinline__ float sumsq4(float ss, float a, float b, float c, float d) {
  float q = __fmul_rn(a, a);
  q = __fmaf_rn(b, b, q);
  q = __fmaf_rn(c, c, q);
  q = __fmaf_rn(d, d, q);
  return __fadd_rn(ss, q);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records `code`) if
// the phase does not complete within kWaitLimitNs, or if another role of the
// CTA already aborted (`*abort` set).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort, unsigned int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (((++spins) & 255u) == 0u) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_device_error(code);
        *abort = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (tiled, 2D, one destination CTA)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* tmap, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* tmap, int x,
                                                 int y, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Four rows (y0..y3) of box width starting at column x, into 512 consecutive
// bytes of shared memory (the tensor map's box is 1 row high).
__device__ __forceinline__ void tma_gather4_hint(void* smem_dst, const CUtensorMap* tmap, int x, int y0,
                                                 int y1, int y2, int y3, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3),
      "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Release / acquire-release adds at GPU scope.  A thread that publishes a
// flag for the stores of its whole CTA (or warp group) issues one of these
// after the CTA-level barrier that follows those stores: the barrier orders
// the other threads' stores before this thread's release, so a reader that
// acquires the flag sees them.
__device__ __forceinline__ int atom_add_release_gpu(int* p, int v) {
  int old;
  asm volatile("atom.release.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One grid-wide barrier of a co-resident grid (at most one CTA per SM, all
// launched): every CTA arrives once on *counter (zero before the launch) and
// waits, bounded, for the others.  Every thread's earlier global writes and
// reductions are visible grid-wide afterwards.  Returns false (device error
// `code` recorded) if the others did not arrive within the wait limit.
__device__ __forceinline__ bool grid_barrier_once(int* counter, unsigned int code) {
  __shared__ int arrived_ok;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    atom_add_release_gpu(counter, 1);
    int good = 1;
    const unsigned long long t0 = globaltimer_ns();
    while (ld_acquire_gpu(counter) < int(gridDim.x)) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_device_error(code);
        good = 0;
        break;
      }
      __nanosleep(128);
    }
    arrived_ok = good;
  }
  __syncthreads();
  return arrived_ok != 0;
}

// Combine finalisation of 8 features: out = bf16(acc [+ residual]), fp32
// sum, one rounding.  acc is read through L2 (it may have been reduced into
// by other SMs in the same kernel).
__device__ __forceinline__ void finalize_vec8(const float* __restrict__ acc, const __nv_bfloat16* __restrict__ residual,
                                              __nv_bfloat16* __restrict__ out, long long i) {
  const float4 a = __ldcg(reinterpret_cast<const float4*>(acc) + 2 * i);
  const float4 b = __ldcg(reinterpret_cast<const float4*>(acc) + 2 * i + 1);
  float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  if (residual) {
    const uint4 r = reinterpret_cast<const uint4*>(residual)[i];
    const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] += __uint_as_float(rw[j] << 16);
      v[2 * j + 1] += __uint_as_float(rw[j] & 0xFFFF0000u);
    }
  }
  uint4 o;
  uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
    ow[j] = *reinterpret_cast<const uint32_t*>(&p);
  }
  reinterpret_cast<uint4*>(out)[i] = o;
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------
// tcgen05 / TMEM
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Instruction descriptor for kind::f16 with bf16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N) {
  return (1u << 4)      // D format: f32
         | (1u << 7)    // A format: bf16
         | (1u << 10)   // B format: bf16
         | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128 B,
// 8-row core groups 1024 B apart.  `smem_addr` must lie in a 1024-aligned tile
// (plus a k offset < 128 B).
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr & 0x3FFFFu) >> 4);
  d |= uint64_t(1) << 16;             // leading byte offset (unused with 128B swizzle)
  d |= uint64_t(1024 >> 4) << 32;     // stride byte offset: 8 rows * 128 B
  d |= uint64_t(1) << 46;             // descriptor version for sm_100
  d |= uint64_t(2) << 61;             // swizzle mode: 128B
  return d;
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 16-byte vector reduction into global memory (no return value).
__device__ __forceinline__ void red_add_v4_f32(float* gdst, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(gdst), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// Bulk (non-tensor) reduce-add of `bytes` fp32 values from shared to global
// memory through the TMA engine; both addresses 16-byte aligned.
__device__ __forceinline__ void bulk_reduce_add_f32(float* gdst, const float* ssrc, uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(
                   reinterpret_cast<uint64_t>(gdst)),
               "r"(smem_u32(ssrc)), "r"(bytes)
               : "memory");
}
// Bulk (non-tensor) copy of `bytes` from global memory into this CTA's shared
// memory, completing on `bar`; both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_load(void* sdst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(sdst)),
               "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Bulk copy of `bytes` from shared to global memory (bulk group); same
// alignment rules.
__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(gdst)),
               "r"(smem_u32(ssrc)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most one committed bulk group still reads shared memory.
__device__ __forceinline__ void bulk_wait_read_le1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// Wait until every committed bulk group has finished reading shared memory
// (the global writes complete on their own; a dependent grid sees them).
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Barrier over `nthreads` threads that also returns the OR of `pred` over them.
__device__ __forceinline__ bool named_barrier_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t elect_one_lane() {
  return (threadIdx.x & 31u) == 0u;
}

}  // namespace qmoe

// Host-side launch-check helper used by the C-ABI entry points.
namespace qmoe_host {
int set_error(int status, const char* fmt, ...);
int check_launch(const char* what);
int num_sms(int device);
}  // namespace qmoe_host
