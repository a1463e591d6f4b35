// C ABI of the Qwen3-MoE hot path (include/qmoe.h): host-side argument checks,
// TMA descriptor encoding, workspace carving and kernel launches.
//
// One translation unit: the kernels live in the *.cuh files included below.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>

#include "attention.cuh"
#include "flash_prefill.cuh"
#include "blockwise.cuh"
#include "common.cuh"
#include "ep.cuh"
#include "ep_p2p.cuh"
#include "finalize.cuh"
#include "grouped_gemm.cuh"
#include "moe_fused.cuh"
#include "norm_rope.cuh"
#include "permute.cuh"
#include "route_small.cuh"
#include "gemv.cuh"
#include "router.cuh"

// ---------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------
namespace qmoe_host {

static thread_local std::string t_last_error;

int set_error(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return status;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return set_error(QMOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  return QMOE_OK;
}

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  int minor = 0;
  bool ok = false;
};

static constexpr int kMaxDevices = 64;
static DeviceInfo g_dev[kMaxDevices];
static std::once_flag g_dev_once[kMaxDevices];

static int device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_error(QMOE_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices) return set_error(QMOE_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::call_once(g_dev_once[dev], [dev]() {
    DeviceInfo& d = g_dev[dev];
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return;
    if (cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return;
    if (cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return;
    d.ok = true;
  });
  DeviceInfo& d = g_dev[dev];
  if (!d.ok) return set_error(QMOE_ERR_CUDA, "could not query device %d", dev);
  if (d.major != 10 || d.minor != 0)
    return set_error(QMOE_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                     d.major, d.minor);
  *out = &d;
  return QMOE_OK;
}

int num_sms(int) {
  DeviceInfo* d = nullptr;
  if (device_info(&d) != QMOE_OK) return 0;
  return d->sms;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn g_encode = nullptr;
static std::once_flag g_encode_once;

static int get_encode(EncodeTiledFn* fn) {
  std::call_once(g_encode_once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!g_encode) return set_error(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  *fn = g_encode;
  return QMOE_OK;
}

// 2D bf16 tensor map, row-major (outer, inner), 128-byte swizzle, box
// (box_outer rows x 64 elements).  Out-of-range rows read as zero.
static int make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = nullptr;
  int st = get_encode(&enc);
  if (st != QMOE_OK) return st;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for %llux%llu box %ux%u",
                     int(r), (unsigned long long)outer, (unsigned long long)inner, box_outer,
                     box_inner);
  return QMOE_OK;
}

// 3D bf16 tensor map: dims (d0 inner, d1, d2), byte strides of d1 and d2,
// 128-byte swizzle, box (b0, b1, b2).  Out-of-range coordinates read as zero.
static int make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                             uint64_t stride1, uint64_t stride2, uint32_t b0, uint32_t b1, uint32_t b2) {
  EncodeTiledFn enc = nullptr;
  int st = get_encode(&enc);
  if (st != QMOE_OK) return st;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1, stride2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled (3D) failed (%d) for %llux%llux%llu", int(r),
                     (unsigned long long)d2, (unsigned long long)d1, (unsigned long long)d0);
  return QMOE_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename Kernel>
static int set_smem(Kernel k, int bytes) {
  cudaError_t err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err != cudaSuccess)
    return set_error(QMOE_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(err));
  return QMOE_OK;
}

// Kernel launch through cudaLaunchKernelEx; with `pdl` the launch allows
// programmatic stream serialization (the kernel overlaps its predecessor's
// tail and waits in griddepcontrol.wait before reading its outputs).
template <typename... KArgs, typename... Args>
static int launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                         bool pdl, const char* name, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess) return set_error(QMOE_ERR_CUDA, "%s: %s", name, cudaGetErrorString(err));
  return check_launch(name);
}

}  // namespace qmoe_host

using namespace qmoe_host;

#define QMOE_CHECK(expr)            \
  do {                              \
    int _st = (expr);               \
    if (_st != QMOE_OK) return _st; \
  } while (0)

#define QMOE_REQUIRE(cond, status, ...)                   \
  do {                                                    \
    if (!(cond)) return set_error((status), __VA_ARGS__); \
  } while (0)

// ---------------------------------------------------------------------------
// launches
// ---------------------------------------------------------------------------
namespace {

// Token counts up to which the router runs as logits kernel (E/8 x T/8
// CTAs) + selection kernel instead of the fused one-CTA-per-8-tokens kernel.
constexpr int64_t kRouterSmallMaxT = 64;
// Token counts up to which the gate/up GEMM gathers token rows itself (TMA
// gather4) instead of reading a permuted copy: at decode sizes the copy costs
// more than it saves; for prefill, 16-row boxes of the copy feed the tensor
// core faster than 4-row gathers.
constexpr int64_t kGatherMaxT = 64;
// Above kGatherMaxT tokens gate/up and down run as one persistent kernel
// (moe_fused_kernel) on the permuted copy of the rows: measured on B200 the
// copy plus 16-row boxes beats gathering token rows in the kernel (gather4,
// 4 rows per instruction) from 256 tokens up, and ties below.  The kernel
// keeps the gather form (qmoe_moe_experts with gather_rows) for callers
// without a copy.
constexpr int64_t kFusedGatherMaxT = kGatherMaxT;
// Above kFusedMinT tokens the forward runs the experts as the persistent
// fused kernel (dynamic units, per-tile dependencies, no split-K; decode
// sizes gather the token rows): measured on B200 it beats the split-K gate/up
// and down kernels from 3 tokens up (-10 % at 4, 8 and 16 tokens) and ties at
// 2; at 1 token (48 gate/up units) the splits keep more SMs streaming.
constexpr int64_t kFusedMinT = 2;
// Routed rows up to which the gate/up GEMM may split K (given a scratch), and
// the most splits.  Splits pay when the units leave SMs idle: at one token
// (8 rows) 48 units of a 148-SM B200 become 144.
constexpr int64_t kGateUpSplitMaxR = 128;
constexpr int kGateUpMaxSplits = 4;

int launch_router(const void* x, const void* w, const float* bias, int64_t T, int64_t H, int64_t E,
                  int64_t k, int normalize, float* logits, int32_t* topk_idx, float* topk_w,
                  int32_t* chunk_hist, cudaStream_t stream) {
  const int G = int(H / 256);
  const int nchunks = int((T + qmoe::kRouterChunk - 1) / qmoe::kRouterChunk);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  if (logits != nullptr && T <= kRouterSmallMaxT) {
    const int smem = int(sizeof(float) * qmoe::kRouterChunk * H);
    const dim3 grid(static_cast<unsigned>((E + qmoe::kRouterSmallWarps - 1) / qmoe::kRouterSmallWarps),
                    static_cast<unsigned>(nchunks));
#define QMOE_ROUTER_SMALL_CASE(GG)                                                                    \
  case GG: {                                                                                          \
    QMOE_CHECK(set_smem(qmoe::router_logits_small_kernel<GG>, smem));                                 \
    qmoe::router_logits_small_kernel<GG><<<grid, qmoe::kRouterSmallWarps * 32, smem, stream>>>(       \
        xb, wb, bias, int(T), int(E), logits);                                                        \
    break;                                                                                            \
  }
    switch (G) {
      QMOE_ROUTER_SMALL_CASE(1)
      QMOE_ROUTER_SMALL_CASE(2)
      QMOE_ROUTER_SMALL_CASE(4)
      QMOE_ROUTER_SMALL_CASE(8)
      QMOE_ROUTER_SMALL_CASE(16)
      default:
        return set_error(QMOE_ERR_UNSUPPORTED_SHAPE, "router: H/256 = %d not in {1,2,4,8,16}", G);
    }
#undef QMOE_ROUTER_SMALL_CASE
    QMOE_CHECK(check_launch("router_logits_small_kernel"));
    return launch_kernel(qmoe::router_select_kernel, dim3(nchunks), dim3(qmoe::kRouterChunk * 32), 0, stream,
                         true, "router_select_kernel", logits, int(T), int(E), int(k), normalize,
                         topk_idx, topk_w, chunk_hist);
  }
  const int smem = int(sizeof(float) * qmoe::kRouterChunk * (H + E));
  // more chunks than SMs: 8-warp CTAs, two per SM (H < 4096)
  const bool pairs = nchunks > num_sms(0);
#define QMOE_ROUTER_LAUNCH(GG, W)                                                                            \
  {                                                                                                          \
    QMOE_CHECK(set_smem(qmoe::router_topk_kernel<GG, W>, smem));                                             \
    return launch_kernel(qmoe::router_topk_kernel<GG, W>, dim3(nchunks), dim3((W) * 32), size_t(smem), stream, \
                         true, "router_topk_kernel", xb, wb, bias, int(T), int(E), int(k), normalize, logits,  \
                         topk_idx, topk_w, chunk_hist);                                                      \
  }
#define QMOE_ROUTER_CASE(GG)                                            \
  case GG: {                                                            \
    if (pairs && GG < 16) QMOE_ROUTER_LAUNCH(GG, 8)                     \
    QMOE_ROUTER_LAUNCH(GG, qmoe::router_warps<GG>())                    \
  }
  switch (G) {
    QMOE_ROUTER_CASE(1)
    QMOE_ROUTER_CASE(2)
    QMOE_ROUTER_CASE(4)
    QMOE_ROUTER_CASE(8)
    QMOE_ROUTER_CASE(16)
    default:
      return set_error(QMOE_ERR_UNSUPPORTED_SHAPE, "router: H/256 = %d not in {1,2,4,8,16}", G);
  }
#undef QMOE_ROUTER_CASE
#undef QMOE_ROUTER_LAUNCH
}

size_t route_small_smem(int64_t T, int64_t H, int64_t E, int64_t k) {
  const size_t rows = 2 * size_t((T + 3) & ~int64_t(3)) * size_t(H);
  return rows + 4 * size_t(T * E) + 8 * size_t(T * k);
}

// Router + permutation for T <= kRouteSmallMaxT: one cluster of
// kRouteSmallCtas CTAs (route_small_kernel).
int launch_route_small(const void* x, const void* w, const float* bias, int64_t T, int64_t H, int64_t E,
                       int64_t k, int normalize, float* logits, int32_t* topk_idx, float* topk_w,
                       int32_t* counts, int32_t* offsets, int32_t* row_token, float* row_w, int32_t* slot_row,
                       int32_t* tiles, int64_t max_tiles, float* acc_zero, cudaStream_t stream,
                       int32_t* zero_words = nullptr, int n_zero_words = 0) {
  const int G = int(H / 256);
  const int smem = int(route_small_smem(T, H, E, k));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(qmoe::kRouteSmallCtas);
  cfg.blockDim = dim3(unsigned(E / qmoe::kRouteSmallCtas * 32));
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = qmoe::kRouteSmallCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  cudaError_t err = cudaSuccess;
#define QMOE_ROUTE_SMALL_CASE(GG)                                                                        \
  case GG:                                                                                               \
    QMOE_CHECK(set_smem(qmoe::route_small_kernel<GG>, smem));                                            \
    err = cudaLaunchKernelEx(&cfg, qmoe::route_small_kernel<GG>, xb, wb, bias, int(T), int(E), int(k),   \
                             normalize, logits, topk_idx, topk_w, counts, offsets, row_token, row_w,     \
                             slot_row, tiles, int(max_tiles), acc_zero, zero_words, n_zero_words);       \
    break;
  switch (G) {
    QMOE_ROUTE_SMALL_CASE(1)
    QMOE_ROUTE_SMALL_CASE(2)
    QMOE_ROUTE_SMALL_CASE(4)
    QMOE_ROUTE_SMALL_CASE(8)
    QMOE_ROUTE_SMALL_CASE(16)
    default:
      return set_error(QMOE_ERR_UNSUPPORTED_SHAPE, "route_small: H/256 = %d not in {1,2,4,8,16}", G);
  }
#undef QMOE_ROUTE_SMALL_CASE
  if (err != cudaSuccess) return set_error(QMOE_ERR_CUDA, "route_small_kernel: %s", cudaGetErrorString(err));
  return check_launch("route_small_kernel");
}

int check_router_args(const void* x, const void* w, int64_t T, int64_t H, int64_t E, int64_t k,
                      const int32_t* topk_idx, const float* topk_w) {
  // an empty batch (T == 0) may come with a null x (an empty tensor's data)
  QMOE_REQUIRE((T == 0 || x) && w && topk_idx && topk_w, QMOE_ERR_INVALID_ARGUMENT, "router: null pointer");
  QMOE_REQUIRE(T >= 0 && T < (int64_t(1) << 31) / 32, QMOE_ERR_INVALID_ARGUMENT, "router: bad T=%lld",
               (long long)T);
  QMOE_REQUIRE(H > 0 && H % 256 == 0 && H <= 4096, QMOE_ERR_UNSUPPORTED_SHAPE,
               "router: H=%lld must be a multiple of 256 and <= 4096", (long long)H);
  QMOE_REQUIRE(E >= 32 && E <= 256 && E % 32 == 0, QMOE_ERR_UNSUPPORTED_SHAPE,
               "router: E=%lld must be a multiple of 32 in [32, 256]", (long long)E);
  QMOE_REQUIRE(k >= 1 && k <= E && k <= 32, QMOE_ERR_INVALID_ARGUMENT, "router: k=%lld invalid",
               (long long)k);
  QMOE_REQUIRE(aligned16(x) && aligned16(w), QMOE_ERR_MISALIGNED, "router: x / w_router not 16-byte aligned");
  return QMOE_OK;
}

int launch_permute(const int32_t* topk_idx, const float* topk_w, int32_t* chunk_hist, const void* x,
                   int64_t T, int64_t H, int64_t E, int64_t k, int32_t* counts, int32_t* offsets,
                   int32_t* row_token, float* row_w, int32_t* slot_row, int32_t* tiles,
                   void* x_perm, float* acc_zero, cudaStream_t stream, int32_t* zero_words = nullptr,
                   int n_zero_words = 0) {
  const int nchunks = int((T + qmoe::kRouterChunk - 1) / qmoe::kRouterChunk);
  const int64_t max_tiles = qmoe_max_tiles(T * k, E);
  QMOE_CHECK(launch_kernel(qmoe::permute_scan_kernel, dim3(unsigned(E)), dim3(qmoe::kScanThreads), 0, stream,
                           true, "permute_scan_kernel", chunk_hist, nchunks, int(E), counts));
  if (nchunks > 0) {
    // Enough CTAs to keep the row gather from being latency-bound.
    const int parts = x_perm ? int(std::max<int64_t>(1, std::min<int64_t>(8, (4 * num_sms(0) + nchunks - 1) / nchunks))) : 1;
    // the chunk's token rows in shared memory for the bulk row copy
    const int smem = x_perm ? int(2 * qmoe::kRouterChunk * H) : 0;
    QMOE_CHECK(set_smem(qmoe::permute_scatter_kernel, smem));
    QMOE_CHECK(launch_kernel(qmoe::permute_scatter_kernel, dim3(nchunks, parts), dim3(qmoe::kScatterThreads),
                             size_t(smem), stream, true, "permute_scatter_kernel", topk_idx, topk_w,
                             static_cast<const int32_t*>(chunk_hist), static_cast<const int32_t*>(counts),
                             offsets, static_cast<const __nv_bfloat16*>(x), int(T), int(H), int(E), int(k),
                             row_token, row_w, slot_row, static_cast<__nv_bfloat16*>(x_perm), acc_zero,
                             tiles, int(max_tiles), zero_words, n_zero_words));
  }
  return QMOE_OK;
}

// Router + scan + scatter in one launch (nchunks <= SMs, T > kRouterSmallMaxT):
// route_permute_kernel.  barrier: two int32 of scratch; zero on entry (every
// completed launch leaves them zero), or cleared here first with `clear`.
int launch_route_permute(const void* x, const void* w, const float* bias, int64_t T, int64_t H, int64_t E,
                         int64_t k, int normalize, int32_t* topk_idx, float* topk_w, int32_t* chunk_hist,
                         int32_t* counts, int32_t* offsets, int32_t* row_token, float* row_w, int32_t* slot_row,
                         int32_t* tiles, int64_t max_tiles, void* x_perm, float* acc_zero, int32_t* zero_words,
                         int n_zero_words, int* barrier, cudaStream_t stream, bool clear) {
  const int G = int(H / 256);
  const int nchunks = int((T + qmoe::kRouterChunk - 1) / qmoe::kRouterChunk);
  if (nchunks <= 0) return QMOE_OK;
  if (clear) {
    const cudaError_t err = cudaMemsetAsync(barrier, 0, 2 * sizeof(int), stream);
    if (err != cudaSuccess) return set_error(QMOE_ERR_CUDA, "route_permute barrier: %s", cudaGetErrorString(err));
  }
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  auto* xp = static_cast<__nv_bfloat16*>(x_perm);
#define QMOE_ROUTE_PERMUTE_CASE(GG)                                                                               \
  case GG: {                                                                                                      \
    constexpr int kThreads = qmoe::router_warps<GG>() * 32;                                                       \
    const int smem = qmoe::route_permute_smem_bytes(int(H), int(E), kThreads);                                   \
    QMOE_CHECK(set_smem(qmoe::route_permute_kernel<GG>, smem));                                                   \
    return launch_kernel(qmoe::route_permute_kernel<GG>, dim3(nchunks), dim3(kThreads), size_t(smem), stream,     \
                         true, "route_permute_kernel", xb, wb, bias, int(T), int(E), int(k), normalize, topk_idx, \
                         topk_w, chunk_hist, counts, offsets, row_token, row_w, slot_row, xp, acc_zero, tiles,     \
                         int(max_tiles), zero_words, n_zero_words, barrier);                                      \
  }
  switch (G) {
    QMOE_ROUTE_PERMUTE_CASE(1)
    QMOE_ROUTE_PERMUTE_CASE(2)
    QMOE_ROUTE_PERMUTE_CASE(4)
    QMOE_ROUTE_PERMUTE_CASE(8)
    QMOE_ROUTE_PERMUTE_CASE(16)
    default:
      return set_error(QMOE_ERR_UNSUPPORTED_SHAPE, "route_permute: H/256 = %d not in {1,2,4,8,16}", G);
  }
#undef QMOE_ROUTE_PERMUTE_CASE
}

// One grouped-GEMM launch in the normal or the small-tile configuration.
// tmB_full (with a.full_boxes) maps whole 128-row tiles of the B operand.
template <int kMode, bool kSmall>
int launch_gemm_cfg(const CUtensorMap& tmA, const CUtensorMap& tmB, const qmoe::GemmArgs& a, int grid,
                    cudaStream_t stream, const char* name, const CUtensorMap* tmB_full = nullptr) {
  using C = qmoe::GemmCfg<kMode, kSmall>;
  QMOE_CHECK(set_smem(qmoe::grouped_gemm_kernel<kMode, kSmall>, C::kSmemBytes));
  return launch_kernel(qmoe::grouped_gemm_kernel<kMode, kSmall>, dim3(grid), dim3(qmoe::kGemmThreads),
                       C::kSmemBytes, stream, true, name, tmA, tmB, tmB_full ? *tmB_full : tmB, a);
}

// Tiles of at most this many rows take the small configuration.
constexpr int64_t kSmallTileRows = qmoe::kBoxRows;

// x: x_perm (R rows, permuted) when gather_rows is null, else the source
// activations (x_rows rows) gathered by gather_rows[r] with TMA gather4.
// max_tile_rows: an upper bound on the rows of any tile.
int launch_gemm_gateup(const void* x, int64_t x_rows, const int32_t* gather_rows, const void* w_gate_up,
                       const int32_t* tiles, int64_t max_tiles, int64_t R, int64_t H, int64_t I, int64_t E,
                       void* act, void* split_ws, cudaStream_t stream, int64_t max_tile_rows = qmoe::kBNMax,
                       int32_t* tile_done = nullptr) {
  CUtensorMap tmA, tmB;
  QMOE_CHECK(make_tmap_bf16(&tmA, w_gate_up, uint64_t(H), uint64_t(E * 2 * I), qmoe::kBK, qmoe::kBM));
  if (gather_rows)
    QMOE_CHECK(make_tmap_bf16(&tmB, x, uint64_t(H), uint64_t(x_rows), qmoe::kBK, 1));
  else
    QMOE_CHECK(make_tmap_bf16(&tmB, x, uint64_t(H), uint64_t(R), qmoe::kBK, qmoe::kBoxRows));
  qmoe::GemmArgs a{};
  a.tiles = tiles;
  a.max_tiles = int(max_tiles);
  a.n_mtiles = int(I / qmoe::kBM);
  a.num_kb = int(H / qmoe::kBK);
  a.k_splits = 1;
  a.a_rows_per_expert = int(2 * I);
  a.up_row_offset = int(I);
  a.gather_rows = gather_rows;
  a.act = static_cast<__nv_bfloat16*>(act);
  a.act_ld = int(I);
  // decode sizes: let the kernel split K when its units leave SMs idle
  a.split_ws = R <= kGateUpSplitMaxR ? static_cast<float*>(split_ws) : nullptr;
  a.max_k_splits = a.split_ws ? kGateUpMaxSplits : 1;
  a.tile_done = tile_done;
  const int64_t units = max_tiles * a.n_mtiles * a.max_k_splits;
  const int grid = int(std::min<int64_t>(units, num_sms(0)));
  if (grid <= 0) return QMOE_OK;
  if (std::min(max_tile_rows, R) <= kSmallTileRows)
    return launch_gemm_cfg<qmoe::kModeGateUp, true>(tmA, tmB, a, grid, stream, "grouped_gemm_kernel<gate_up,small>");
  return launch_gemm_cfg<qmoe::kModeGateUp, false>(tmA, tmB, a, grid, stream, "grouped_gemm_kernel<gate_up>");
}

int launch_gemm_down(const void* act, const void* w_down, const int32_t* tiles, int64_t max_tiles,
                     const int32_t* row_dst, const float* row_w, int64_t R, int64_t H, int64_t I,
                     int64_t E, float* acc, int64_t n_acc, cudaStream_t stream,
                     int64_t max_tile_rows = qmoe::kBNMax, int flags = 0, const void* fin_residual = nullptr,
                     void* fin_out = nullptr, int32_t* grid_bar = nullptr, int32_t* tile_done = nullptr) {
  CUtensorMap tmA, tmB;
  QMOE_CHECK(make_tmap_bf16(&tmA, w_down, uint64_t(I), uint64_t(E * H), qmoe::kBK, qmoe::kBM));
  QMOE_CHECK(make_tmap_bf16(&tmB, act, uint64_t(I), uint64_t(R), qmoe::kBK, qmoe::kBoxRows));
  qmoe::GemmArgs a{};
  a.tiles = tiles;
  a.max_tiles = int(max_tiles);
  a.n_mtiles = int(H / qmoe::kBM);
  a.num_kb = int(I / qmoe::kBK);
  a.k_splits = 1;
  // Tiny batches: the kernel may split K (up to 3 ways, no more than the
  // grid holds at once) to put more SMs on the weight stream; the partials
  // meet in the accumulator.
  if (R <= 16) a.k_splits = 3;
  a.a_rows_per_expert = int(H);
  a.up_row_offset = 0;
  a.row_dst = row_dst;
  a.row_w = row_w;
  a.acc = acc;
  a.acc_ld = int(H);
  a.n_acc = int(n_acc);
  a.flags = flags;
  a.fin_residual = static_cast<const __nv_bfloat16*>(fin_residual);
  a.fin_out = static_cast<__nv_bfloat16*>(fin_out);
  a.grid_bar = grid_bar;
  // per-tile counters of the gate/up GEMM (its I / 128 units per tile)
  a.tile_done = tile_done;
  a.tile_done_target = int(I / qmoe::kBM);
  const int64_t units = max_tiles * a.n_mtiles * a.k_splits;
  const int grid = int(std::min<int64_t>(units, num_sms(0)));
  if (grid <= 0) return QMOE_OK;
  if (std::min(max_tile_rows, R) <= kSmallTileRows)
    return launch_gemm_cfg<qmoe::kModeDown, true>(tmA, tmB, a, grid, stream, "grouped_gemm_kernel<down,small>");
  return launch_gemm_cfg<qmoe::kModeDown, false>(tmA, tmB, a, grid, stream, "grouped_gemm_kernel<down>");
}

// Gate/up + down in one persistent kernel (prefill sizes).  x: the permuted
// rows (R) when gather_rows is null, else the token rows (x_rows) gathered by
// gather_rows[r].
int launch_moe_fused(const void* x, int64_t x_rows, const int32_t* gather_rows, const void* w_gate_up,
                     const void* w_down, const int32_t* tiles, int64_t max_tiles, const int32_t* row_dst,
                     const float* row_w, int64_t R, int64_t H, int64_t I, int64_t E, void* act, float* acc,
                     int64_t n_acc, int32_t* done, cudaStream_t stream, const void* fin_residual = nullptr,
                     void* fin_out = nullptr, const void* row_meta = nullptr, void* const* peer_ret = nullptr,
                     int64_t ret_row0 = 0, int64_t n_ranks = 0) {
  using C = qmoe::FusedCfg;
  CUtensorMap ta_gu, tb_gu, ta_dn, tb_dn;
  QMOE_CHECK(make_tmap_bf16(&ta_gu, w_gate_up, uint64_t(H), uint64_t(E * 2 * I), qmoe::kBK, qmoe::kBM));
  if (gather_rows)
    QMOE_CHECK(make_tmap_bf16(&tb_gu, x, uint64_t(H), uint64_t(x_rows), qmoe::kBK, 1));
  else
    QMOE_CHECK(make_tmap_bf16(&tb_gu, x, uint64_t(H), uint64_t(R), qmoe::kBK, qmoe::kBoxRows));
  QMOE_CHECK(make_tmap_bf16(&ta_dn, w_down, uint64_t(I), uint64_t(E * H), qmoe::kBK, qmoe::kBM));
  QMOE_CHECK(make_tmap_bf16(&tb_dn, act, uint64_t(I), uint64_t(R), qmoe::kBK, qmoe::kBoxRows));
  // whole 128-row tiles load as one box (eight times fewer TMA requests than
  // 16-row boxes; same shared-memory layout); with a gather the gate/up rows
  // come by gather4 and this map is not used
  CUtensorMap tb_gu_full = tb_gu, tb_dn_full = tb_dn;
  const bool full_boxes = R >= qmoe::kBNMax && !gather_rows;
  if (full_boxes) {
    QMOE_CHECK(make_tmap_bf16(&tb_gu_full, x, uint64_t(H), uint64_t(R), qmoe::kBK, qmoe::kBNMax));
    QMOE_CHECK(make_tmap_bf16(&tb_dn_full, act, uint64_t(I), uint64_t(R), qmoe::kBK, qmoe::kBNMax));
  }
  qmoe::FusedArgs a{};
  a.full_boxes = full_boxes ? 1 : 0;
  a.tiles = tiles;
  a.max_tiles = int(max_tiles);
  a.n_rows = int(R);
  a.n_mt_gu = int(I / qmoe::kBM);
  a.dn_two = H % (2 * qmoe::kBM) == 0 ? 1 : 0;
  a.n_mt_dn = int(H / (qmoe::kBM * (1 + a.dn_two)));
  a.num_kb_gu = int(H / qmoe::kBK);
  a.num_kb_dn = int(I / qmoe::kBK);
  a.a_rows_gu = int(2 * I);
  a.up_off = int(I);
  a.a_rows_dn = int(H);
  a.act = static_cast<__nv_bfloat16*>(act);
  a.act_ld = int(I);
  a.row_dst = row_dst;
  a.row_w = row_w;
  a.acc = acc;
  a.acc_ld = int(H);
  a.n_acc = int(n_acc);
  a.done = done;
  a.gather_rows = gather_rows;
  a.fin_residual = static_cast<const __nv_bfloat16*>(fin_residual);
  a.fin_out = static_cast<__nv_bfloat16*>(fin_out);
  a.row_meta = static_cast<const int4*>(row_meta);
  a.peer_ret = reinterpret_cast<__nv_bfloat16* const*>(peer_ret);
  a.ret_row0 = int(ret_row0);
  a.n_ranks = int(n_ranks);
  const int64_t units = max_tiles * (a.n_mt_gu + a.n_mt_dn);
  const int grid = int(std::min<int64_t>(units, num_sms(0)));
  if (grid <= 0) return QMOE_OK;
  if (a.peer_ret != nullptr) {
    QMOE_CHECK(set_smem(qmoe::moe_fused_kernel<true>, C::kSmemBytes));
    return launch_kernel(qmoe::moe_fused_kernel<true>, dim3(grid), dim3(qmoe::kGemmThreads), C::kSmemBytes, stream,
                         true, "moe_fused_kernel<return>", ta_gu, tb_gu, ta_dn, tb_dn, tb_gu_full, tb_dn_full, a);
  }
  QMOE_CHECK(set_smem(qmoe::moe_fused_kernel<false>, C::kSmemBytes));
  return launch_kernel(qmoe::moe_fused_kernel<false>, dim3(grid), dim3(qmoe::kGemmThreads), C::kSmemBytes, stream,
                       true, "moe_fused_kernel", ta_gu, tb_gu, ta_dn, tb_dn, tb_gu_full, tb_dn_full, a);
}

// RMSNorm launch with the row held in registers: kChunks 128-element chunks
// per warp (H <= 4096).
// Above this many rows, bf16 rows take the low-register prefill kernel.
constexpr int kNormPrefetchMaxRows = 1024;

template <typename Tin, typename Tout>
int launch_rmsnorm(int chunks, int grid, cudaStream_t s, const Tin* x, const __nv_bfloat16* res, const float* w,
                   int rows, int H, float eps, Tout* y, __nv_bfloat16* res_out) {
  if constexpr (sizeof(Tin) == 2) {
    if (rows > kNormPrefetchMaxRows) {
#define QMOE_RMSNORM_ROWS_CASE(CH)                                                                              \
  if (chunks <= CH)                                                                                             \
    return launch_kernel(qmoe::rmsnorm_rows_kernel<Tout, CH>, dim3(grid), dim3(qmoe::kNormThreads), 0, s, true, \
                         "rmsnorm_rows_kernel", x, res, w, rows, H, eps, y, res_out);
      QMOE_RMSNORM_ROWS_CASE(1)
      QMOE_RMSNORM_ROWS_CASE(2)
      QMOE_RMSNORM_ROWS_CASE(4)
      QMOE_RMSNORM_ROWS_CASE(8)
      QMOE_RMSNORM_ROWS_CASE(16)
      QMOE_RMSNORM_ROWS_CASE(32)
#undef QMOE_RMSNORM_ROWS_CASE
    }
  }
#define QMOE_RMSNORM_CASE(CH)                                                                               \
  if (chunks <= CH)                                                                                         \
    return launch_kernel(qmoe::rmsnorm_kernel<Tin, Tout, CH>, dim3(grid), dim3(qmoe::kNormThreads), 0, s, true, \
                         "rmsnorm_kernel", x, res, w, rows, H, eps, y, res_out);
  QMOE_RMSNORM_CASE(1)
  QMOE_RMSNORM_CASE(2)
  QMOE_RMSNORM_CASE(4)
  QMOE_RMSNORM_CASE(8)
  QMOE_RMSNORM_CASE(16)
  QMOE_RMSNORM_CASE(32)
#undef QMOE_RMSNORM_CASE
  return set_error(QMOE_ERR_UNSUPPORTED_SHAPE, "rmsnorm: H=%d > 4096", H);
}

// Decode-row projection on the CUDA cores (gemv.cuh): T <= kGemvMaxT rows,
// K of 1024, 2048 or 4096, weights up to kGemvMaxWeightElems.
constexpr int64_t kGemvMaxWeightElems = int64_t(32) << 20;  // 64 MB of bf16

bool linear_rows_applies(int64_t T, int64_t K, int64_t N) {
  return T >= 1 && T <= qmoe::kGemvMaxT && (K == 1024 || K == 2048 || K == 4096) && N * K <= kGemvMaxWeightElems;
}

int launch_linear_rows(const void* x, const void* w, int64_t T, int64_t K, int64_t N, void* out,
                       cudaStream_t stream) {
  const int TT = T <= 1 ? 1 : T <= 2 ? 2 : 4;
  const int smem = int(TT * K * 2);
  const dim3 grid(unsigned((N + qmoe::kGemvWarps - 1) / qmoe::kGemvWarps));
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  auto* ob = static_cast<__nv_bfloat16*>(out);
#define QMOE_GEMV_CASE(KC, TTV)                                                                            \
  if (K == 256 * (KC) && TT == (TTV)) {                                                                    \
    QMOE_CHECK(set_smem(qmoe::linear_rows_kernel<KC, TTV>, smem));                                        \
    return launch_kernel(qmoe::linear_rows_kernel<KC, TTV>, grid, dim3(qmoe::kGemvWarps * 32), size_t(smem), \
                         stream, true, "linear_rows_kernel", xb, wb, int(T), int(N), ob);                  \
  }
#define QMOE_GEMV_KC(KC) QMOE_GEMV_CASE(KC, 1) QMOE_GEMV_CASE(KC, 2) QMOE_GEMV_CASE(KC, 4)
  QMOE_GEMV_KC(4)
  QMOE_GEMV_KC(8)
  QMOE_GEMV_KC(16)
#undef QMOE_GEMV_KC
#undef QMOE_GEMV_CASE
  return set_error(QMOE_ERR_UNSUPPORTED_SHAPE, "linear_rows: K=%lld T=%lld", (long long)K, (long long)T);
}

// Expert GEMMs of a 1-2 token step on the CUDA cores (gemv.cuh).
bool expert_rows_applies(int64_t T, int64_t H, int64_t k, int64_t I) {
  return T >= 1 && T <= qmoe::kExpertRowsMaxT && (H == 1024 || H == 2048) && I % 256 == 0 &&
         I / 256 <= 4 && T * k <= qmoe::kExpertRowsMaxR && T * k * I * 2 <= 96 * 1024;
}

int launch_expert_rows(const void* x, const int32_t* row_token, const float* row_w, const void* w_gate_up,
                       const void* w_down, const int32_t* tiles, int64_t max_tiles, int64_t R, int64_t H,
                       int64_t I, int64_t E, int64_t T, void* act, const void* residual, void* out,
                       cudaStream_t s) {
  using bf16 = __nv_bfloat16;
  const dim3 block(qmoe::kGemvWarps * 32);
  const dim3 grid_gu(unsigned(std::min<int64_t>(2 * num_sms(0), max_tiles * (I / qmoe::kGemvWarps))));
  int st = QMOE_OK;
#define QMOE_GU_CASE(KC)                                                                                          \
  if (H == 256 * (KC))                                                                                             \
    st = launch_kernel(qmoe::expert_gateup_rows_kernel<KC>, grid_gu, block, 0, s, true, "expert_gateup_rows_kernel", \
                       static_cast<const bf16*>(x), row_token, static_cast<const bf16*>(w_gate_up), tiles,          \
                       int(max_tiles), int(R), int(I), int(E), int(T), static_cast<bf16*>(act));
  QMOE_GU_CASE(4)
  QMOE_GU_CASE(8)
#undef QMOE_GU_CASE
  if (st != QMOE_OK) return st;
  const int smem = int(R * I * 2);
  const dim3 grid_dn(unsigned(std::min<int64_t>(2 * num_sms(0), (H + qmoe::kGemvWarps - 1) / qmoe::kGemvWarps)));
#define QMOE_DN_CASE(IC)                                                                                          \
  if (I == 256 * (IC)) {                                                                                           \
    QMOE_CHECK(set_smem(qmoe::expert_down_rows_kernel<IC>, smem));                                                 \
    return launch_kernel(qmoe::expert_down_rows_kernel<IC>, grid_dn, block, size_t(smem), s, true,                 \
                         "expert_down_rows_kernel", static_cast<const bf16*>(act), static_cast<const bf16*>(w_down), \
                         tiles, int(max_tiles), row_token, row_w, int(R), int(H), int(E), int(T),                    \
                         static_cast<const bf16*>(residual), static_cast<bf16*>(out));                               \
  }
  QMOE_DN_CASE(1)
  QMOE_DN_CASE(2)
  QMOE_DN_CASE(3)
  QMOE_DN_CASE(4)
#undef QMOE_DN_CASE
  return set_error(QMOE_ERR_UNSUPPORTED_SHAPE, "expert rows: I=%lld", (long long)I);
}

// Rows from which dense projections may run 256-feature units (they do when
// that still gives every SM a unit; otherwise the 128-feature units leave
// fewer SMs idle).
constexpr int64_t kPlainPairMinRows = 512;

int launch_linear(const void* x, const void* w, int64_t T, int64_t K, int64_t N, void* out,
                  cudaStream_t stream, void* split_ws = nullptr) {
  if (linear_rows_applies(T, K, N)) return launch_linear_rows(x, w, T, K, N, out, stream);
  CUtensorMap tmA, tmB;
  QMOE_CHECK(make_tmap_bf16(&tmA, w, uint64_t(K), uint64_t(N), qmoe::kBK, qmoe::kBM));
  QMOE_CHECK(make_tmap_bf16(&tmB, x, uint64_t(K), uint64_t(T), qmoe::kBK, qmoe::kBoxRows));
  qmoe::GemmArgs a{};
  a.tiles = nullptr;
  a.dense_rows = int(T);
  a.n_mtiles = int(N / qmoe::kBM);
  a.num_kb = int(K / qmoe::kBK);
  a.k_splits = 1;
  a.a_rows_per_expert = 0;
  a.act = static_cast<__nv_bfloat16*>(out);
  a.act_ld = int(N);
  // decode rows (<= 16): the deep-ring small configuration, and K split over
  // up to 8 CTAs per feature block when a scratch is given
  const bool small = T <= kSmallTileRows;
  a.split_ws = small ? static_cast<float*>(split_ws) : nullptr;
  a.max_k_splits = a.split_ws ? 8 : 1;
  const int64_t units = ((T + qmoe::kBNMax - 1) / qmoe::kBNMax) * a.n_mtiles * a.max_k_splits;
  const int grid = int(std::min<int64_t>(units, num_sms(0)));
  if (grid <= 0) return QMOE_OK;
  if (small)
    return launch_gemm_cfg<qmoe::kModePlain, true>(tmA, tmB, a, grid, stream, "grouped_gemm_kernel<plain,small>");
  // whole 128-row tiles of x load as one TMA box
  CUtensorMap tmB_full = tmB;
  if (T >= qmoe::kBNMax) {
    QMOE_CHECK(make_tmap_bf16(&tmB_full, x, uint64_t(K), uint64_t(T), qmoe::kBK, qmoe::kBNMax));
    a.full_boxes = 1;
  }
  const int64_t units2 = ((T + qmoe::kBNMax - 1) / qmoe::kBNMax) * (N / (2 * qmoe::kBM));
  if (N % (2 * qmoe::kBM) == 0 && T >= kPlainPairMinRows && units2 >= num_sms(0)) {
    // prefill-sized projections with at least a unit per SM: 256-feature
    // units, two accumulators sharing each 128-row tile (a quarter fewer
    // operand bytes from L2 per FLOP)
    a.n_mtiles = int(N / (2 * qmoe::kBM));
    a.up_row_offset = qmoe::kBM;
    const int grid2 = int(std::min<int64_t>(units2, num_sms(0)));
    return launch_gemm_cfg<qmoe::kModePlainPair, false>(tmA, tmB, a, grid2, stream,
                                                        "grouped_gemm_kernel<plain pair>", &tmB_full);
  }
  return launch_gemm_cfg<qmoe::kModePlain, false>(tmA, tmB, a, grid, stream, "grouped_gemm_kernel<plain>",
                                                  &tmB_full);
}

int launch_finalize(const float* acc, const void* residual, int64_t T, int64_t H, void* out,
                    cudaStream_t stream) {
  const long long n8 = (long long)(T * H / 8);
  if (n8 == 0) return QMOE_OK;
  const int grid = int(std::min<long long>((n8 + 255) / 256, (long long)num_sms(0) * 8));
  return launch_kernel(qmoe::combine_finalize_kernel, dim3(grid), dim3(256), 0, stream, true,
                       "combine_finalize_kernel", acc, static_cast<const __nv_bfloat16*>(residual),
                       static_cast<__nv_bfloat16*>(out), (long long)n8);
}

// Workspace carving for the fused forward.
struct FwdLayout {
  size_t logits, chunk_hist, counts, offsets, row_token, row_w, slot_row, tiles, topk_idx, topk_w, x_perm,
      act, acc, split, done, route_barrier, norm_h, norm_res, total;
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// with_norm: room for the add & norm outputs (qmoe_moe_block_forward callers
// that do not take them).
FwdLayout fwd_layout(int64_t T, int64_t H, int64_t E, int64_t k, int64_t I, bool with_norm = false) {
  FwdLayout L{};
  const int64_t R = T * k;
  const int64_t nchunks = (T + qmoe::kRouterChunk - 1) / qmoe::kRouterChunk;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = align256(o + bytes);
    return at;
  };
  L.logits = take(T <= kRouterSmallMaxT ? sizeof(float) * size_t(T * E) : 0);
  L.chunk_hist = take(sizeof(int32_t) * size_t(nchunks * E));
  L.counts = take(sizeof(int32_t) * size_t(E));
  L.offsets = take(sizeof(int32_t) * size_t(E + 1));
  L.row_token = take(sizeof(int32_t) * size_t(R));
  L.row_w = take(sizeof(float) * size_t(R));
  L.slot_row = take(sizeof(int32_t) * size_t(R));
  L.tiles = take(sizeof(int32_t) * size_t(1 + 3 * qmoe_max_tiles(R, E)));
  L.topk_idx = take(sizeof(int32_t) * size_t(R));
  L.topk_w = take(sizeof(float) * size_t(R));
  L.x_perm = take(T > kFusedGatherMaxT ? 2 * size_t(R * H) : 0);
  L.act = take(2 * size_t(R * I));
  L.acc = take(sizeof(float) * size_t(T * H));
  L.split = take(T * k <= kGateUpSplitMaxR ? qmoe::kSplitWorkspaceBytes : 0);
  L.done = take(T > kFusedMinT ? sizeof(int32_t) * size_t(qmoe_max_tiles(R, E) + 2) : 0);
  // the one-launch route + permutation (and its two barrier words) serves
  // every fused batch that the decode route kernel does not
  L.route_barrier = take(T > kFusedMinT ? 2 * sizeof(int32_t) : 0);
  L.norm_h = take(with_norm ? 2 * size_t(T * H) : 0);
  L.norm_res = take(with_norm ? 2 * size_t(T * H) : 0);
  L.total = o;
  return L;
}

// The decoder layer's add & norm in front of the MoE block (qwen.py:423,
// 428): s = bf16(a + res) -> res_out, h = bf16(rmsnorm(s) * w) -> h_out; the
// MoE block reads h and its output adds s.
struct AddNorm {
  const void* a;
  const void* res;
  const float* w;
  float eps;
  void* h_out;
  void* res_out;
};

// The MoE forward on a workspace laid out by fwd_layout (shapes checked by
// the caller): routing, permutation, experts and the combine.  With `an`, x
// and residual are ignored: the add & norm kernel runs first and the block
// reads its outputs.  (Folding the add & norm into the decode route kernel
// measured slower: that kernel's 8-CTA cluster then follows the whole-GPU
// O projection directly and waits for eight free SMs of one GPC; behind
// the small norm kernel it is placed while the norm runs.)
int moe_forward_on(const void* x, const void* w_router, const float* router_bias, const void* w_gate_up,
                   const void* w_down, const void* residual, int64_t T, int64_t H, int64_t E, int64_t k, int64_t I,
                   int normalize, void* out, int32_t* topk_idx, float* topk_w, uint8_t* ws, const FwdLayout& L,
                   cudaStream_t s, const AddNorm* an = nullptr) {
  const bool small_route = T <= qmoe::kRouteSmallMaxT && E <= qmoe::kRouteSmallMaxE;
  if (an) {
    using bf16 = __nv_bfloat16;
    x = an->h_out;
    residual = an->res_out;
    const int st = launch_rmsnorm<bf16, bf16>(int((H + 127) / 128), int((T + 7) / 8), s,
                                              static_cast<const bf16*>(an->a), static_cast<const bf16*>(an->res),
                                              an->w, int(T), int(H), an->eps, static_cast<bf16*>(an->h_out),
                                              static_cast<bf16*>(an->res_out));
    if (st != QMOE_OK) return st;
  }
  int32_t* chunk_hist = reinterpret_cast<int32_t*>(ws + L.chunk_hist);
  int32_t* counts = reinterpret_cast<int32_t*>(ws + L.counts);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  int32_t* row_token = reinterpret_cast<int32_t*>(ws + L.row_token);
  float* row_w = reinterpret_cast<float*>(ws + L.row_w);
  int32_t* slot_row = reinterpret_cast<int32_t*>(ws + L.slot_row);
  int32_t* tiles = reinterpret_cast<int32_t*>(ws + L.tiles);
  int32_t* idx = topk_idx ? topk_idx : reinterpret_cast<int32_t*>(ws + L.topk_idx);
  float* tw = topk_w ? topk_w : reinterpret_cast<float*>(ws + L.topk_w);
  const bool fused = T > kFusedMinT;
  void* x_perm = T > kFusedGatherMaxT ? ws + L.x_perm : nullptr;
  void* act = ws + L.act;
  float* acc = reinterpret_cast<float*>(ws + L.acc);
  float* split_ws = T * k <= kGateUpSplitMaxR ? reinterpret_cast<float*>(ws + L.split) : nullptr;
  int32_t* done = fused ? reinterpret_cast<int32_t*>(ws + L.done) : nullptr;
  int32_t* split_counters = split_ws ? reinterpret_cast<int32_t*>(split_ws + size_t(qmoe::kSplitSlots) *
                                                                               qmoe::kSplitSlotFloats)
                                     : nullptr;
  const int64_t R = T * k;
  const int64_t max_tiles = qmoe_max_tiles(R, E);
  // a token's k experts are distinct, so no expert gets more than T rows
  const int64_t tile_rows = std::min<int64_t>(T, qmoe::kBNMax);

  float* logits = T <= kRouterSmallMaxT ? reinterpret_cast<float*>(ws + L.logits) : nullptr;
  const int64_t nchunks = (T + qmoe::kRouterChunk - 1) / qmoe::kRouterChunk;
  if (small_route) {
    // decode sizes: router + permutation in one launch, which also zeroes
    // the gate/up split counters (the workspace may hold anything on entry)
    QMOE_CHECK(launch_route_small(x, w_router, router_bias, T, H, E, k, normalize, logits, idx, tw, counts,
                                  offsets, row_token, row_w, slot_row, tiles, max_tiles, acc, s,
                                  fused ? done : split_counters,
                                  fused ? int(max_tiles + 2) : split_counters ? qmoe::kSplitCounterWords : 0));
  } else if (fused && nchunks <= num_sms(0)) {
    // prefill batches of at most one router chunk per SM: router, scan and
    // scatter in one launch (one grid-wide barrier), which also zeroes the
    // fused kernel's tile counters
    QMOE_CHECK(launch_route_permute(x, w_router, router_bias, T, H, E, k, normalize, idx, tw, chunk_hist, counts,
                                    offsets, row_token, row_w, slot_row, tiles, max_tiles, x_perm, acc, done,
                                    int(max_tiles + 2), reinterpret_cast<int*>(ws + L.route_barrier), s, true));
  } else {
    QMOE_CHECK(launch_router(x, w_router, router_bias, T, H, E, k, normalize, logits, idx, tw,
                             chunk_hist, s));
    // the permutation also zeroes the gate/up split counters or the fused
    // kernel's tile counters (the workspace may hold anything on entry)
    int32_t* zero = fused ? done : split_counters;
    const int n_zero = fused ? int(max_tiles + 2) : (split_counters ? qmoe::kSplitCounterWords : 0);
    QMOE_CHECK(launch_permute(idx, tw, chunk_hist, x, T, H, E, k, counts, offsets, row_token, row_w,
                              slot_row, tiles, x_perm, acc, s, zero, n_zero));
  }
  if (fused) {
    // prefill: gate/up and down in one persistent kernel, which also
    // finalises the combine after a grid-wide barrier
    if (x_perm)
      return launch_moe_fused(x_perm, R, nullptr, w_gate_up, w_down, tiles, max_tiles, row_token, row_w, R, H, I,
                              E, act, acc, T, done, s, residual, out);
    return launch_moe_fused(x, T, row_token, w_gate_up, w_down, tiles, max_tiles, row_token, row_w, R, H, I, E, act,
                            acc, T, done, s, residual, out);
  }
  // 1-2 tokens: the expert GEMMs are matrix-vector products, run on the CUDA
  // cores; the down kernel also adds the residual and writes the output
  if (expert_rows_applies(T, H, k, I))
    return launch_expert_rows(x, row_token, row_w, w_gate_up, w_down, tiles, max_tiles, R, H, I, E, T, act,
                              residual, out, s);
  // with the split scratch (decode sizes) the gate/up GEMM counts finished
  // units per tile there, so the down GEMM starts each tile as soon as its
  // activations are written rather than after the whole gate/up grid
  int32_t* tile_done = split_counters && max_tiles <= qmoe::kSplitTileDoneWords
                           ? split_counters + qmoe::kSplitTileDoneOffset
                           : nullptr;
  QMOE_CHECK(launch_gemm_gateup(x, T, row_token, w_gate_up, tiles, max_tiles, R, H, I, E, act, split_ws, s,
                                tile_rows, tile_done));
  // the tile list comes from the routing kernels, before the gate/up GEMM;
  // with the split scratch (decode sizes) the down GEMM finalises too
  if (split_counters)
    return launch_gemm_down(act, w_down, tiles, max_tiles, row_token, row_w, R, H, I, E, acc, T, s, tile_rows,
                            qmoe::kGemmTilesReady, residual, out, split_counters + qmoe::kSplitSlots, tile_done);
  QMOE_CHECK(launch_gemm_down(act, w_down, tiles, max_tiles, row_token, row_w, R, H, I, E, acc, T, s, tile_rows,
                              qmoe::kGemmTilesReady));
  return launch_finalize(acc, residual, T, H, out, s);
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

int qmoe_version(void) { return 100; }

const char* qmoe_status_string(int status) {
  switch (status) {
    case QMOE_OK: return "ok";
    case QMOE_ERR_INVALID_ARGUMENT: return "invalid argument";
    case QMOE_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
    case QMOE_ERR_MISALIGNED: return "misaligned pointer";
    case QMOE_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case QMOE_ERR_CUDA: return "CUDA error";
    case QMOE_ERR_DEVICE: return "unsupported device";
    default: return "unknown status";
  }
}

const char* qmoe_last_error(void) { return t_last_error.c_str(); }

int qmoe_device_error(int clear, unsigned int* code_out) {
  QMOE_REQUIRE(code_out, QMOE_ERR_INVALID_ARGUMENT, "device_error: null output");
  cudaError_t err = cudaDeviceSynchronize();
  if (err != cudaSuccess) return set_error(QMOE_ERR_CUDA, "cudaDeviceSynchronize: %s", cudaGetErrorString(err));
  unsigned int v = 0;
  err = cudaMemcpyFromSymbol(&v, qmoe::g_device_error, sizeof(v));
  if (err != cudaSuccess) return set_error(QMOE_ERR_CUDA, "read device error: %s", cudaGetErrorString(err));
  if (clear) {
    unsigned int z = 0;
    err = cudaMemcpyToSymbol(qmoe::g_device_error, &z, sizeof(z));
    if (err != cudaSuccess) return set_error(QMOE_ERR_CUDA, "clear device error: %s", cudaGetErrorString(err));
  }
  *code_out = v;
  return QMOE_OK;
}

int64_t qmoe_max_tiles(int64_t rows, int64_t E) {
  if (rows < 0 || E < 0) return 0;
  return E + rows / qmoe::kTileRows + 1;
}

int qmoe_router_topk(const void* x, const void* w_router, const float* bias, int64_t T, int64_t H,
                     int64_t E, int64_t k, int normalize, float* logits, int32_t* topk_idx,
                     float* topk_w, int32_t* chunk_hist, void* stream) {
  QMOE_CHECK(check_router_args(x, w_router, T, H, E, k, topk_idx, topk_w));
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (T == 0) return QMOE_OK;
  return launch_router(x, w_router, bias, T, H, E, k, normalize, logits, topk_idx, topk_w,
                       chunk_hist, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace {
int check_permute_args(const int32_t* topk_idx, const float* topk_w, const int32_t* chunk_hist, const void* x,
                       int64_t T, int64_t H, int64_t E, int64_t k, const int32_t* counts, const int32_t* offsets,
                       const int32_t* row_token, const float* row_w, const int32_t* slot_row, const int32_t* tiles,
                       const void* x_perm, const float* acc_zero, const int32_t* zero_words, int64_t n_zero_words) {
  QMOE_REQUIRE(!zero_words == (n_zero_words == 0) && n_zero_words >= 0 && n_zero_words < (int64_t(1) << 24),
               QMOE_ERR_INVALID_ARGUMENT, "permute: bad zero_words / n_zero_words");
  QMOE_REQUIRE(topk_idx && topk_w && chunk_hist && counts && offsets && row_token && row_w &&
                   slot_row && tiles,
               QMOE_ERR_INVALID_ARGUMENT, "permute: null pointer");
  QMOE_REQUIRE(T >= 0 && T < (int64_t(1) << 31) / 32, QMOE_ERR_INVALID_ARGUMENT, "permute: bad T");
  QMOE_REQUIRE(E >= 1 && E <= 256, QMOE_ERR_UNSUPPORTED_SHAPE, "permute: E=%lld not in [1, 256]",
               (long long)E);
  QMOE_REQUIRE(k >= 1 && k <= E && k <= 32, QMOE_ERR_INVALID_ARGUMENT, "permute: k=%lld invalid",
               (long long)k);
  if (x_perm || acc_zero) {
    QMOE_REQUIRE(H > 0 && H % 8 == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "permute: H must be a multiple of 8");
    QMOE_REQUIRE(!x_perm || (x && aligned16(x) && aligned16(x_perm)), QMOE_ERR_MISALIGNED,
                 "permute: x / x_perm null or not 16-byte aligned");
    QMOE_REQUIRE(!acc_zero || aligned16(acc_zero), QMOE_ERR_MISALIGNED, "permute: acc not aligned");
  }
  return QMOE_OK;
}
}  // namespace

extern "C" {

int qmoe_moe_permute(const int32_t* topk_idx, const float* topk_w, int32_t* chunk_hist,
                     const void* x, int64_t T, int64_t H, int64_t E, int64_t k, int32_t* counts,
                     int32_t* offsets, int32_t* row_token, float* row_w, int32_t* slot_row,
                     int32_t* tiles, void* x_perm, float* acc_zero, int32_t* zero_words, int64_t n_zero_words,
                     void* stream) {
  QMOE_CHECK(check_permute_args(topk_idx, topk_w, chunk_hist, x, T, H, E, k, counts, offsets, row_token, row_w,
                                slot_row, tiles, x_perm, acc_zero, zero_words, n_zero_words));
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  return launch_permute(topk_idx, topk_w, chunk_hist, x, T, H, E, k, counts, offsets, row_token,
                        row_w, slot_row, tiles, x_perm, acc_zero, static_cast<cudaStream_t>(stream), zero_words,
                        int(n_zero_words));
}

// An empty batch still leaves consistent routing outputs: zero counts and
// offsets, an empty tile list and the scratch words zeroed (a consumer that
// reads the counts -- the expert-parallel count exchange -- then sees no rows
// instead of a previous batch's).
static int route_empty(int32_t* counts, int32_t* offsets, int32_t* tiles, int64_t E, int32_t* zero_words,
                int64_t n_zero_words, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(counts, 0, size_t(E) * 4, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(offsets, 0, size_t(E + 1) * 4, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(tiles, 0, 4, s);
  if (e == cudaSuccess && zero_words && n_zero_words > 0) e = cudaMemsetAsync(zero_words, 0, size_t(n_zero_words) * 4, s);
  QMOE_REQUIRE(e == cudaSuccess, QMOE_ERR_CUDA, "route (empty batch): %s", cudaGetErrorString(e));
  return QMOE_OK;
}

int qmoe_route_permute(const void* x, const void* w_router, const float* bias, int64_t T, int64_t H, int64_t E,
                       int64_t k, int normalize, int32_t* topk_idx, float* topk_w, int32_t* chunk_hist,
                       int32_t* counts, int32_t* offsets, int32_t* row_token, float* row_w, int32_t* slot_row,
                       int32_t* tiles, void* x_perm, float* acc_zero, int32_t* zero_words, int64_t n_zero_words,
                       int32_t* barrier, void* stream) {
  QMOE_CHECK(check_router_args(x, w_router, T, H, E, k, topk_idx, topk_w));
  QMOE_CHECK(check_permute_args(topk_idx, topk_w, chunk_hist, x, T, H, E, k, counts, offsets, row_token, row_w,
                                slot_row, tiles, x_perm, acc_zero, zero_words, n_zero_words));
  QMOE_REQUIRE(barrier && (reinterpret_cast<uintptr_t>(chunk_hist) & 15u) == 0, QMOE_ERR_INVALID_ARGUMENT,
               "route_permute: null barrier or chunk_hist not 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T == 0) return route_empty(counts, offsets, tiles, E, zero_words, n_zero_words, s);
  const int64_t nchunks = (T + qmoe::kRouterChunk - 1) / qmoe::kRouterChunk;
  if (T > kRouterSmallMaxT && nchunks <= num_sms(0))
    return launch_route_permute(x, w_router, bias, T, H, E, k, normalize, topk_idx, topk_w, chunk_hist, counts,
                                offsets, row_token, row_w, slot_row, tiles, qmoe_max_tiles(T * k, E), x_perm,
                                acc_zero, zero_words, int(n_zero_words), barrier, s, false);
  QMOE_CHECK(launch_router(x, w_router, bias, T, H, E, k, normalize, nullptr, topk_idx, topk_w, chunk_hist, s));
  return launch_permute(topk_idx, topk_w, chunk_hist, x, T, H, E, k, counts, offsets, row_token, row_w, slot_row,
                        tiles, x_perm, acc_zero, s, zero_words, int(n_zero_words));
}

int qmoe_route_small(const void* x, const void* w_router, const float* bias, int64_t T, int64_t H, int64_t E,
                     int64_t k, int normalize, float* logits, int32_t* topk_idx, float* topk_w, int32_t* counts,
                     int32_t* offsets, int32_t* row_token, float* row_w, int32_t* slot_row, int32_t* tiles,
                     float* acc_zero, void* stream) {
  QMOE_CHECK(check_router_args(x, w_router, T, H, E, k, topk_idx, topk_w));
  QMOE_REQUIRE(logits && counts && offsets && row_token && row_w && slot_row && tiles, QMOE_ERR_INVALID_ARGUMENT,
               "route_small: null pointer");
  QMOE_REQUIRE(T <= qmoe::kRouteSmallMaxT, QMOE_ERR_UNSUPPORTED_SHAPE, "route_small: T=%lld > %d", (long long)T,
               qmoe::kRouteSmallMaxT);
  QMOE_REQUIRE(E <= qmoe::kRouteSmallMaxE, QMOE_ERR_UNSUPPORTED_SHAPE, "route_small: E=%lld > %d", (long long)E,
               qmoe::kRouteSmallMaxE);
  QMOE_REQUIRE(!acc_zero || aligned16(acc_zero), QMOE_ERR_MISALIGNED, "route_small: acc not 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (T == 0) return route_empty(counts, offsets, tiles, E, nullptr, 0, static_cast<cudaStream_t>(stream));
  return launch_route_small(x, w_router, bias, T, H, E, k, normalize, logits, topk_idx, topk_w, counts, offsets,
                            row_token, row_w, slot_row, tiles, qmoe_max_tiles(T * k, E), acc_zero,
                            static_cast<cudaStream_t>(stream));
}

size_t qmoe_grouped_gemm_gateup_split_workspace_size(void) { return qmoe::kSplitWorkspaceBytes; }

int qmoe_grouped_gemm_gateup_swiglu(const void* x, int64_t x_rows, const int32_t* gather_rows,
                                    const void* w_gate_up, const int32_t* tiles, int64_t max_tiles,
                                    int64_t max_tile_rows, int64_t R, int64_t H, int64_t I, int64_t E,
                                    void* act, void* split_ws, size_t split_ws_bytes, void* stream) {
  QMOE_REQUIRE(x && w_gate_up && tiles && act, QMOE_ERR_INVALID_ARGUMENT, "gate_up: null pointer");
  QMOE_REQUIRE(R >= 0 && R < (int64_t(1) << 31), QMOE_ERR_INVALID_ARGUMENT, "gate_up: bad R");
  QMOE_REQUIRE(!gather_rows || (x_rows > 0 && x_rows < (int64_t(1) << 31)), QMOE_ERR_INVALID_ARGUMENT,
               "gate_up: bad x_rows for a gather");
  QMOE_REQUIRE(H > 0 && H % qmoe::kBK == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "gate_up: H %% 64 != 0");
  QMOE_REQUIRE(I > 0 && I % qmoe::kBM == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "gate_up: I %% 128 != 0");
  QMOE_REQUIRE(E > 0 && E * 2 * I < (int64_t(1) << 31), QMOE_ERR_UNSUPPORTED_SHAPE, "gate_up: E too large");
  QMOE_REQUIRE(max_tiles >= 0 && max_tiles < (int64_t(1) << 24), QMOE_ERR_INVALID_ARGUMENT, "gate_up: bad max_tiles");
  QMOE_REQUIRE(aligned16(x) && aligned16(w_gate_up) && aligned16(act), QMOE_ERR_MISALIGNED,
               "gate_up: pointers must be 16-byte aligned");
  QMOE_REQUIRE(!split_ws || split_ws_bytes >= qmoe::kSplitWorkspaceBytes, QMOE_ERR_WORKSPACE_TOO_SMALL,
               "gate_up: split workspace %zu < required %zu bytes", split_ws_bytes, qmoe::kSplitWorkspaceBytes);
  QMOE_REQUIRE(!split_ws || aligned16(split_ws), QMOE_ERR_MISALIGNED, "gate_up: split workspace not 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (R == 0) return QMOE_OK;
  return launch_gemm_gateup(x, x_rows, gather_rows, w_gate_up, tiles, max_tiles, R, H, I, E, act, split_ws,
                            static_cast<cudaStream_t>(stream),
                            max_tile_rows >= 1 && max_tile_rows <= qmoe::kBNMax ? max_tile_rows : qmoe::kBNMax);
}

int qmoe_grouped_gemm_down_combine(const void* act, const void* w_down, const int32_t* tiles,
                                   int64_t max_tiles, int64_t max_tile_rows, int64_t flags,
                                   const int32_t* row_dst, const float* row_w,
                                   int64_t R, int64_t H, int64_t I, int64_t E, float* acc,
                                   int64_t n_acc, void* stream) {
  QMOE_REQUIRE(act && w_down && tiles && row_dst && row_w && acc, QMOE_ERR_INVALID_ARGUMENT,
               "down: null pointer");
  QMOE_REQUIRE(R >= 0 && R < (int64_t(1) << 31), QMOE_ERR_INVALID_ARGUMENT, "down: bad R");
  QMOE_REQUIRE(H > 0 && H % qmoe::kBM == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "down: H %% 128 != 0");
  QMOE_REQUIRE(I > 0 && I % qmoe::kBK == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "down: I %% 64 != 0");
  QMOE_REQUIRE(E > 0 && E * H < (int64_t(1) << 31), QMOE_ERR_UNSUPPORTED_SHAPE, "down: E too large");
  QMOE_REQUIRE(n_acc >= 0 && n_acc * H < (int64_t(1) << 40), QMOE_ERR_INVALID_ARGUMENT, "down: bad n_acc");
  QMOE_REQUIRE(max_tiles >= 0 && max_tiles < (int64_t(1) << 24), QMOE_ERR_INVALID_ARGUMENT, "down: bad max_tiles");
  QMOE_REQUIRE(aligned16(act) && aligned16(w_down), QMOE_ERR_MISALIGNED, "down: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (R == 0) return QMOE_OK;
  return launch_gemm_down(act, w_down, tiles, max_tiles, row_dst, row_w, R, H, I, E, acc, n_acc,
                          static_cast<cudaStream_t>(stream),
                          max_tile_rows >= 1 && max_tile_rows <= qmoe::kBNMax ? max_tile_rows : qmoe::kBNMax,
                          (flags & QMOE_GEMM_TILES_READY) ? qmoe::kGemmTilesReady : 0);
}

int qmoe_moe_experts(const void* x, int64_t x_rows, const int32_t* gather_rows, const void* w_gate_up,
                     const void* w_down, const int32_t* tiles, int64_t max_tiles, const int32_t* row_dst,
                     const float* row_w, int64_t R, int64_t H, int64_t I, int64_t E, void* act, float* acc,
                     int64_t n_acc, int32_t* done, void* stream) {
  QMOE_REQUIRE(x && w_gate_up && w_down && tiles && row_dst && row_w && act && acc && done,
               QMOE_ERR_INVALID_ARGUMENT, "moe_experts: null pointer");
  QMOE_REQUIRE(R >= 0 && R < (int64_t(1) << 31), QMOE_ERR_INVALID_ARGUMENT, "moe_experts: bad R");
  QMOE_REQUIRE(!gather_rows || (x_rows > 0 && x_rows < (int64_t(1) << 31)), QMOE_ERR_INVALID_ARGUMENT,
               "moe_experts: bad x_rows for a gather");
  QMOE_REQUIRE(H > 0 && H % qmoe::kBM == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "moe_experts: H %% 128 != 0");
  QMOE_REQUIRE(I > 0 && I % qmoe::kBM == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "moe_experts: I %% 128 != 0");
  QMOE_REQUIRE(E > 0 && E * 2 * I < (int64_t(1) << 31) && E * H < (int64_t(1) << 31), QMOE_ERR_UNSUPPORTED_SHAPE,
               "moe_experts: E too large");
  QMOE_REQUIRE(n_acc >= 0 && n_acc * H < (int64_t(1) << 40), QMOE_ERR_INVALID_ARGUMENT, "moe_experts: bad n_acc");
  QMOE_REQUIRE(max_tiles >= 0 && max_tiles < (int64_t(1) << 24), QMOE_ERR_INVALID_ARGUMENT,
               "moe_experts: bad max_tiles");
  QMOE_REQUIRE(aligned16(x) && aligned16(w_gate_up) && aligned16(w_down) && aligned16(act), QMOE_ERR_MISALIGNED,
               "moe_experts: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (R == 0) return QMOE_OK;
  return launch_moe_fused(x, x_rows, gather_rows, w_gate_up, w_down, tiles, max_tiles, row_dst, row_w, R, H, I, E,
                          act, acc, n_acc, done, static_cast<cudaStream_t>(stream));
}

int qmoe_masked_residual_add(const void* y, const float* mask, const void* residual, int64_t T, int64_t H,
                             void* out, void* stream) {
  QMOE_REQUIRE(y && out, QMOE_ERR_INVALID_ARGUMENT, "masked_residual_add: null pointer");
  QMOE_REQUIRE(T >= 0 && T < (int64_t(1) << 31), QMOE_ERR_INVALID_ARGUMENT, "masked_residual_add: bad T");
  QMOE_REQUIRE(H > 0 && H % 8 == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "masked_residual_add: H %% 8 != 0");
  QMOE_REQUIRE(aligned16(y) && aligned16(out) && (!residual || aligned16(residual)), QMOE_ERR_MISALIGNED,
               "masked_residual_add: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (T == 0) return QMOE_OK;
  const long long total = (long long)T * (H / 8);
  const int grid = int(std::min<long long>((total + 255) / 256, (long long)d->sms * 8));
  return launch_kernel(qmoe::masked_residual_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       true, "masked_residual_kernel", static_cast<const uint4*>(y), mask,
                       static_cast<const uint4*>(residual), static_cast<uint4*>(out), int(T), int(H / 8));
}

int qmoe_select_affinities(const float* affinities, const int32_t* idx, int64_t T, int64_t E, int64_t k,
                           int64_t normalize, float* w, void* stream) {
  QMOE_REQUIRE(affinities && idx && w, QMOE_ERR_INVALID_ARGUMENT, "select_affinities: null pointer");
  QMOE_REQUIRE(T >= 0 && T < (int64_t(1) << 31) && E >= 1 && T * E < (int64_t(1) << 40) && k >= 1 && k <= 32,
               QMOE_ERR_INVALID_ARGUMENT, "select_affinities: bad sizes");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (T == 0) return QMOE_OK;
  return launch_kernel(qmoe::select_affinities_kernel, dim3(int((T + 255) / 256)), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), true, "select_affinities_kernel", affinities, idx, int(T),
                       int(E), int(k), normalize ? 1 : 0, w);
}

int qmoe_greedy_pick(const void* logits, int64_t B, int64_t V, int32_t* tokens, int32_t* positions,
                     int32_t* lengths, void* stream) {
  QMOE_REQUIRE(logits && tokens, QMOE_ERR_INVALID_ARGUMENT, "greedy_pick: null pointer");
  QMOE_REQUIRE(B >= 0 && B < (int64_t(1) << 31) && V > 0 && V < (int64_t(1) << 31), QMOE_ERR_INVALID_ARGUMENT,
               "greedy_pick: bad sizes");
  QMOE_REQUIRE(V % 8 != 0 || aligned16(logits), QMOE_ERR_MISALIGNED, "greedy_pick: logits not 16-byte aligned");
  if (B == 0) return QMOE_OK;
  return launch_kernel(qmoe::greedy_pick_kernel, dim3(unsigned(B)), dim3(1024), 0, static_cast<cudaStream_t>(stream),
                       true, "greedy_pick_kernel", static_cast<const __nv_bfloat16*>(logits), int(V), tokens,
                       positions, lengths);
}

int qmoe_embedding_gather(const void* table, int64_t V, int64_t H, const int32_t* ids, int64_t n, void* out,
                          void* stream) {
  QMOE_REQUIRE(table && ids && out, QMOE_ERR_INVALID_ARGUMENT, "embedding: null pointer");
  QMOE_REQUIRE(V > 0 && V < (int64_t(1) << 31) && n >= 0 && n < (int64_t(1) << 31), QMOE_ERR_INVALID_ARGUMENT,
               "embedding: bad V or n");
  QMOE_REQUIRE(H > 0 && H % 8 == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "embedding: H %% 8 != 0");
  QMOE_REQUIRE(aligned16(table) && aligned16(out), QMOE_ERR_MISALIGNED, "embedding: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (n == 0) return QMOE_OK;
  const long long total = (long long)n * (H / 8);
  const int grid = int(std::min<long long>((total + 255) / 256, (long long)d->sms * 8));
  return launch_kernel(qmoe::embedding_gather_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       true, "embedding_gather_kernel", static_cast<const uint4*>(table), ids, int(n), int(V),
                       int(H / 8), static_cast<uint4*>(out));
}

int qmoe_combine_finalize(const float* acc, const void* residual, int64_t T, int64_t H, void* out,
                          void* stream) {
  QMOE_REQUIRE(acc && out, QMOE_ERR_INVALID_ARGUMENT, "finalize: null pointer");
  QMOE_REQUIRE(T >= 0 && H > 0 && H % 8 == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "finalize: H %% 8 != 0");
  QMOE_REQUIRE(aligned16(acc) && aligned16(out) && (!residual || aligned16(residual)),
               QMOE_ERR_MISALIGNED, "finalize: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  return launch_finalize(acc, residual, T, H, out, static_cast<cudaStream_t>(stream));
}

int64_t qmoe_blockwise_max_tiles(int64_t block_size, int64_t num_blocks) {
  if (block_size <= 0 || num_blocks <= 0) return 0;
  return num_blocks * ((block_size + qmoe::kTileRows - 1) / qmoe::kTileRows);
}

int qmoe_blockwise_prepare(const void* x, const float* affinities, int64_t aff_rows,
                           const int32_t* token_position_to_id, const int32_t* block_to_expert,
                           int64_t T, int64_t H, int64_t E, int64_t block_size, int64_t num_blocks,
                           void* x_perm, int32_t* row_dst, float* row_w, int32_t* tiles,
                           void* stream) {
  QMOE_REQUIRE(x && affinities && token_position_to_id && block_to_expert && x_perm && row_dst &&
                   row_w && tiles,
               QMOE_ERR_INVALID_ARGUMENT, "blockwise_prepare: null pointer");
  QMOE_REQUIRE(T >= 0 && T < (int64_t(1) << 31) && aff_rows >= 0, QMOE_ERR_INVALID_ARGUMENT,
               "blockwise_prepare: bad T / aff_rows");
  QMOE_REQUIRE(H > 0 && H % 8 == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "blockwise_prepare: H %% 8 != 0");
  QMOE_REQUIRE(E > 0, QMOE_ERR_INVALID_ARGUMENT, "blockwise_prepare: E <= 0");
  QMOE_REQUIRE(block_size >= 1 && block_size <= 8192, QMOE_ERR_UNSUPPORTED_SHAPE,
               "blockwise_prepare: block_size %lld not in [1, 8192]", (long long)block_size);
  QMOE_REQUIRE(num_blocks >= 0 && num_blocks * block_size < (int64_t(1) << 31),
               QMOE_ERR_INVALID_ARGUMENT, "blockwise_prepare: bad num_blocks");
  QMOE_REQUIRE(aligned16(x) && aligned16(x_perm), QMOE_ERR_MISALIGNED,
               "blockwise_prepare: x / x_perm must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (num_blocks == 0) return QMOE_OK;
  const int64_t max_tiles = qmoe_blockwise_max_tiles(block_size, num_blocks);
  const int smem = int(2 * sizeof(int) * block_size);
  QMOE_CHECK(set_smem(qmoe::blockwise_prepare_kernel, smem));
  qmoe::blockwise_prepare_kernel<<<int(num_blocks), qmoe::kBlockwiseThreads, smem,
                                   static_cast<cudaStream_t>(stream)>>>(
      token_position_to_id, block_to_expert, affinities, int(aff_rows),
      static_cast<const __nv_bfloat16*>(x), int(T), int(H), int(E), int(block_size),
      static_cast<__nv_bfloat16*>(x_perm), row_dst, row_w, tiles, int(max_tiles));
  return check_launch("blockwise_prepare_kernel");
}

int qmoe_linear(const void* x, const void* w, int64_t T, int64_t K, int64_t N, void* out, void* split_ws,
                size_t split_ws_bytes, void* stream) {
  QMOE_REQUIRE(x && w && out, QMOE_ERR_INVALID_ARGUMENT, "linear: null pointer");
  QMOE_REQUIRE(T >= 0 && T < (int64_t(1) << 31), QMOE_ERR_INVALID_ARGUMENT, "linear: bad T");
  QMOE_REQUIRE(K > 0 && K % qmoe::kBK == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "linear: K %% 64 != 0");
  QMOE_REQUIRE(N > 0 && N % qmoe::kBM == 0 && N < (int64_t(1) << 31), QMOE_ERR_UNSUPPORTED_SHAPE,
               "linear: N %% 128 != 0");
  QMOE_REQUIRE(aligned16(x) && aligned16(w) && aligned16(out), QMOE_ERR_MISALIGNED,
               "linear: pointers must be 16-byte aligned");
  QMOE_REQUIRE(!split_ws || split_ws_bytes >= qmoe::kSplitWorkspaceBytes, QMOE_ERR_WORKSPACE_TOO_SMALL,
               "linear: split workspace %zu < required %zu bytes", split_ws_bytes, qmoe::kSplitWorkspaceBytes);
  QMOE_REQUIRE(!split_ws || aligned16(split_ws), QMOE_ERR_MISALIGNED, "linear: split workspace not aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (T == 0) return QMOE_OK;
  return launch_linear(x, w, T, K, N, out, static_cast<cudaStream_t>(stream), split_ws);
}

int qmoe_rmsnorm(const void* x, int x_is_fp32, const void* residual, const float* weight,
                 int64_t rows, int64_t H, float eps, void* out, int out_is_fp32,
                 void* residual_out, void* stream) {
  QMOE_REQUIRE(x && weight && out, QMOE_ERR_INVALID_ARGUMENT, "rmsnorm: null pointer");
  QMOE_REQUIRE(!residual || (residual_out && !x_is_fp32), QMOE_ERR_INVALID_ARGUMENT,
               "rmsnorm: a residual needs residual_out and bf16 x");
  QMOE_REQUIRE(rows >= 0 && rows < (int64_t(1) << 31), QMOE_ERR_INVALID_ARGUMENT, "rmsnorm: bad rows");
  QMOE_REQUIRE(H > 0 && H % 4 == 0 && H <= 4096, QMOE_ERR_UNSUPPORTED_SHAPE,
               "rmsnorm: H must be a multiple of 4 and <= 4096");
  QMOE_REQUIRE(aligned16(x) && aligned16(weight) && aligned16(out) &&
                   (!residual || (aligned16(residual) && aligned16(residual_out))),
               QMOE_ERR_MISALIGNED, "rmsnorm: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (rows == 0) return QMOE_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = int((rows + 7) / 8);
  const auto* res = static_cast<const __nv_bfloat16*>(residual);
  auto* res_out = static_cast<__nv_bfloat16*>(residual_out);
  const int chunks = int((H + 127) / 128);
  if (x_is_fp32 && out_is_fp32)
    return launch_rmsnorm<float, float>(chunks, grid, s, static_cast<const float*>(x), nullptr, weight, int(rows),
                                        int(H), eps, static_cast<float*>(out), nullptr);
  if (x_is_fp32)
    return launch_rmsnorm<float, __nv_bfloat16>(chunks, grid, s, static_cast<const float*>(x), nullptr, weight,
                                                int(rows), int(H), eps, static_cast<__nv_bfloat16*>(out), nullptr);
  if (out_is_fp32)
    return launch_rmsnorm<__nv_bfloat16, float>(chunks, grid, s, static_cast<const __nv_bfloat16*>(x), res, weight,
                                                int(rows), int(H), eps, static_cast<float*>(out), res_out);
  return launch_rmsnorm<__nv_bfloat16, __nv_bfloat16>(chunks, grid, s, static_cast<const __nv_bfloat16*>(x), res,
                                                      weight, int(rows), int(H), eps,
                                                      static_cast<__nv_bfloat16*>(out), res_out);
}

int qmoe_qk_norm_rope(const void* qkv, const int32_t* positions, const int32_t* cache_slot,
                      const float* q_norm_w, const float* k_norm_w, const float* inv_freq, int64_t T,
                      int64_t nh, int64_t nkv, int64_t head_dim, float eps, void* q_out,
                      void* k_cache, void* v_cache, int64_t n_slots, int64_t max_seq, void* stream) {
  QMOE_REQUIRE(qkv && positions && q_norm_w && k_norm_w && inv_freq && q_out && k_cache && v_cache,
               QMOE_ERR_INVALID_ARGUMENT, "qk_norm_rope: null pointer");
  QMOE_REQUIRE(head_dim == qmoe::kQkHeadDim, QMOE_ERR_UNSUPPORTED_SHAPE,
               "qk_norm_rope: head_dim must be 128");
  QMOE_REQUIRE(nh > 0 && nkv > 0 && nh % nkv == 0, QMOE_ERR_INVALID_ARGUMENT, "qk_norm_rope: bad heads");
  QMOE_REQUIRE(nh + 2 * nkv <= qmoe::kQkWarps * qmoe::kQkMaxHeadsPerWarp, QMOE_ERR_UNSUPPORTED_SHAPE,
               "qk_norm_rope: more than %d heads", qmoe::kQkWarps * qmoe::kQkMaxHeadsPerWarp);
  QMOE_REQUIRE(T >= 0 && T * (nh + 2 * nkv) < (int64_t(1) << 31), QMOE_ERR_INVALID_ARGUMENT,
               "qk_norm_rope: bad T");
  QMOE_REQUIRE(n_slots > 0 && max_seq > 0, QMOE_ERR_INVALID_ARGUMENT, "qk_norm_rope: bad cache shape");
  QMOE_REQUIRE(aligned16(qkv) && aligned16(q_out) && aligned16(k_cache) && aligned16(v_cache) &&
                   aligned16(q_norm_w) && aligned16(k_norm_w),
               QMOE_ERR_MISALIGNED, "qk_norm_rope: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (T == 0) return QMOE_OK;
  // a CTA per token, each warp several heads
  return launch_kernel(qmoe::qk_norm_rope_kernel, dim3(unsigned(T)), dim3(32 * qmoe::kQkWarps), 0,
                       static_cast<cudaStream_t>(stream), true, "qk_norm_rope_kernel",
                       static_cast<const __nv_bfloat16*>(qkv), positions, cache_slot, q_norm_w, k_norm_w, inv_freq,
                       int(T), int(nh), int(nkv), eps, static_cast<__nv_bfloat16*>(q_out),
                       static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), int(max_seq),
                       int(n_slots));
}

int qmoe_attention_prefill(const void* q, const void* k_cache, const void* v_cache,
                           const int32_t* q_start, const int32_t* cache_slot, const int32_t* kv_start, int64_t B,
                           int64_t S, int64_t nh, int64_t nkv, int64_t head_dim, int64_t n_slots,
                           int64_t max_seq, float scale, void* out, void* stream) {
  QMOE_REQUIRE(q && k_cache && v_cache && q_start && out, QMOE_ERR_INVALID_ARGUMENT,
               "attention_prefill: null pointer");
  QMOE_REQUIRE(head_dim == qmoe::kFaD, QMOE_ERR_UNSUPPORTED_SHAPE, "attention_prefill: head_dim must be 128");
  QMOE_REQUIRE(nh > 0 && nkv > 0 && nh % nkv == 0 && nh <= 65535, QMOE_ERR_INVALID_ARGUMENT,
               "attention_prefill: bad heads");
  QMOE_REQUIRE(B >= 0 && B <= 65535 && S >= 0 && S <= max_seq && max_seq > 0 && max_seq < (int64_t(1) << 30) &&
                   n_slots > 0 && n_slots * nkv < (int64_t(1) << 31) && (cache_slot || B <= n_slots),
               QMOE_ERR_INVALID_ARGUMENT, "attention_prefill: bad sizes");
  const int64_t n_pairs = (S + 2 * qmoe::kFaRows - 1) / (2 * qmoe::kFaRows);  // CTAs per (sequence, head)
  QMOE_REQUIRE(B * S < (int64_t(1) << 31) && n_pairs * nh * B < (int64_t(1) << 31), QMOE_ERR_INVALID_ARGUMENT,
               "attention_prefill: too many queries");
  QMOE_REQUIRE(aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out),
               QMOE_ERR_MISALIGNED, "attention_prefill: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (B == 0 || S == 0) return QMOE_OK;
  // q (B*S, nh, 128): tokens outermost; caches (slots*nkv, max_seq, 128)
  CUtensorMap tq, tk, tv;
  QMOE_CHECK(make_tmap_bf16_3d(&tq, q, 128, uint64_t(nh), uint64_t(B * S), 256, uint64_t(nh) * 256, 64, 1,
                               qmoe::kFaRows));
  QMOE_CHECK(make_tmap_bf16_3d(&tk, k_cache, 128, uint64_t(max_seq), uint64_t(n_slots * nkv), 256,
                               uint64_t(max_seq) * 256, 64, qmoe::kFaRows, 1));
  QMOE_CHECK(make_tmap_bf16_3d(&tv, v_cache, 128, uint64_t(max_seq), uint64_t(n_slots * nkv), 256,
                               uint64_t(max_seq) * 256, 64, qmoe::kFaRows, 1));
  qmoe::FlashPrefillArgs args{};
  args.q_start = q_start;
  args.cache_slot = cache_slot;
  args.kv_start = kv_start;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.S = int(S);
  args.nh = int(nh);
  args.nkv = int(nkv);
  args.max_seq = int(max_seq);
  args.n_slots = int(n_slots);
  args.B = int(B);
  args.n_pairs = int(n_pairs);
  args.scale_log2 = scale * 1.4426950408889634f;
  QMOE_CHECK(set_smem(qmoe::flash_prefill_kernel, qmoe::kFaSmemBytes));
  return launch_kernel(qmoe::flash_prefill_kernel, dim3(unsigned(n_pairs * nh * B)), dim3(qmoe::kFaThreads),
                       size_t(qmoe::kFaSmemBytes), static_cast<cudaStream_t>(stream), true, "flash_prefill_kernel",
                       tq, tk, tv, args);
}

int64_t qmoe_attention_decode_splits(int64_t B, int64_t nkv, int64_t max_len) {
  if (B <= 0 || nkv <= 0 || max_len <= 0) return 1;
  const int sms = std::max(1, num_sms(0));
  // enough CTAs for two waves of the SMs, chunks of at least 128 keys
  int64_t want = (2 * int64_t(sms) + B * nkv - 1) / (B * nkv);
  int64_t most = (max_len + 127) / 128;
  return std::max<int64_t>(1, std::min(want, most));
}

size_t qmoe_attention_decode_workspace_size(int64_t B, int64_t nh, int64_t nsplit) {
  if (B <= 0 || nh <= 0 || nsplit <= 0) return 0;
  return size_t(B * nh * nsplit) * (qmoe::kAttnD + 2) * sizeof(float) + 256;
}

int qmoe_attention_decode(const void* q, const void* k_cache, const void* v_cache,
                          const int32_t* kv_len, const int32_t* cache_slot, const int32_t* kv_start, int64_t B,
                          int64_t nh,
                          int64_t nkv, int64_t head_dim, int64_t n_slots, int64_t max_seq, int64_t max_len,
                          int64_t nsplit, float scale, void* out, void* workspace,
                          size_t workspace_bytes, void* stream) {
  QMOE_REQUIRE(q && k_cache && v_cache && kv_len && out && workspace, QMOE_ERR_INVALID_ARGUMENT,
               "attention_decode: null pointer");
  QMOE_REQUIRE(head_dim == qmoe::kAttnD, QMOE_ERR_UNSUPPORTED_SHAPE, "attention_decode: head_dim must be 128");
  QMOE_REQUIRE(nkv > 0 && nh == nkv * qmoe::kDecodeGroup, QMOE_ERR_UNSUPPORTED_SHAPE,
               "attention_decode: needs 8 query heads per KV head");
  QMOE_REQUIRE(B >= 0 && B <= 65535 && nkv <= 65535 && max_len >= 0 && max_len <= max_seq && nsplit >= 1 &&
                   nsplit <= 65535 && n_slots > 0 && (cache_slot || B <= n_slots),
               QMOE_ERR_INVALID_ARGUMENT, "attention_decode: bad sizes");
  QMOE_REQUIRE(workspace_bytes >= qmoe_attention_decode_workspace_size(B, nh, nsplit),
               QMOE_ERR_WORKSPACE_TOO_SMALL, "attention_decode: workspace too small");
  QMOE_REQUIRE(aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out) &&
                   (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
               QMOE_ERR_MISALIGNED, "attention_decode: pointers must be 16-byte aligned (workspace 256)");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (B == 0) return QMOE_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* part_o = static_cast<float*>(workspace);
  float* part_ml = part_o + size_t(B * nh * nsplit) * qmoe::kAttnD;
  const int64_t chunk = std::max<int64_t>(64, ((max_len + nsplit - 1) / nsplit + 63) / 64 * 64);
  const int smem = 4 * qmoe::kAttnBK * qmoe::kAttnPad * 2 + 4 * qmoe::kDecodeGroup * (qmoe::kAttnD + 2) * 4;
  QMOE_CHECK(set_smem(qmoe::attn_decode_kernel, smem));
  const dim3 grid(static_cast<unsigned>(nsplit), static_cast<unsigned>(nkv), static_cast<unsigned>(B));
  QMOE_CHECK(launch_kernel(qmoe::attn_decode_kernel, grid, dim3(qmoe::kAttnThreads), size_t(smem), s, true,
                           "attn_decode_kernel", static_cast<const __nv_bfloat16*>(q),
                           static_cast<const __nv_bfloat16*>(k_cache), static_cast<const __nv_bfloat16*>(v_cache),
                           kv_len, cache_slot, kv_start, int(nh), int(nkv), int(max_seq), int(n_slots), int(chunk),
                           scale * 1.4426950408889634f, part_o, part_ml));
  return launch_kernel(qmoe::attn_decode_combine_kernel, dim3(unsigned((B * nh + 7) / 8)), dim3(256), 0, s, true,
                       "attn_decode_combine_kernel", static_cast<const float*>(part_o),
                       static_cast<const float*>(part_ml), int(B), int(nh), int(nsplit),
                       static_cast<__nv_bfloat16*>(out));
}

int qmoe_routing_histogram(const int32_t* topk_idx, int64_t T, int64_t k, int64_t E, int32_t* chunk_hist,
                           void* stream) {
  QMOE_REQUIRE(topk_idx && chunk_hist, QMOE_ERR_INVALID_ARGUMENT, "routing_histogram: null pointer");
  QMOE_REQUIRE(T >= 0 && T < (int64_t(1) << 31) / 32 && k >= 1 && k <= 32 && E >= 1 && E <= 256,
               QMOE_ERR_INVALID_ARGUMENT, "routing_histogram: bad sizes");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  const int nchunks = int((T + qmoe::kRouterChunk - 1) / qmoe::kRouterChunk);
  if (nchunks == 0) return QMOE_OK;
  qmoe::routing_hist_kernel<<<nchunks, qmoe::kEpThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      topk_idx, int(T), int(k), int(E), chunk_hist);
  return check_launch("routing_hist_kernel");
}

int qmoe_ep_pack(const int32_t* topk_idx, const float* topk_w, const void* x, int64_t T, int64_t H,
                 int64_t k, int64_t e_local, int64_t n_ranks, int32_t* chunk_hist, int32_t* send_counts,
                 void* send_x, int32_t* send_expert, float* send_w, int32_t* pair_pos, void* stream) {
  QMOE_REQUIRE(topk_idx && topk_w && x && chunk_hist && send_counts && send_x && send_expert && send_w &&
                   pair_pos,
               QMOE_ERR_INVALID_ARGUMENT, "ep_pack: null pointer");
  QMOE_REQUIRE(T >= 0 && T < (int64_t(1) << 31) / 32 && k >= 1 && k <= 32, QMOE_ERR_INVALID_ARGUMENT,
               "ep_pack: bad T / k");
  QMOE_REQUIRE(n_ranks >= 1 && n_ranks <= 256 && e_local >= 1, QMOE_ERR_INVALID_ARGUMENT,
               "ep_pack: bad n_ranks / e_local");
  QMOE_REQUIRE(H > 0 && H % 8 == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "ep_pack: H %% 8 != 0");
  QMOE_REQUIRE(aligned16(x) && aligned16(send_x), QMOE_ERR_MISALIGNED, "ep_pack: x / send_x not aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nchunks = int((T + qmoe::kRouterChunk - 1) / qmoe::kRouterChunk);
  if (nchunks == 0) {
    cudaError_t err = cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * size_t(n_ranks), s);
    if (err != cudaSuccess) return set_error(QMOE_ERR_CUDA, "ep_pack: %s", cudaGetErrorString(err));
    return QMOE_OK;
  }
  qmoe::ep_dest_hist_kernel<<<nchunks, qmoe::kEpThreads, 0, s>>>(topk_idx, int(T), int(k), int(e_local),
                                                                 int(n_ranks), chunk_hist);
  QMOE_CHECK(check_launch("ep_dest_hist_kernel"));
  qmoe::permute_scan_kernel<<<int(n_ranks), qmoe::kScanThreads, 0, s>>>(chunk_hist, nchunks, int(n_ranks),
                                                                        send_counts);
  QMOE_CHECK(check_launch("permute_scan_kernel"));
  qmoe::ep_pack_kernel<<<nchunks, qmoe::kEpThreads, 0, s>>>(
      topk_idx, topk_w, static_cast<const __nv_bfloat16*>(x), chunk_hist, send_counts, int(T), int(H),
      int(k), int(e_local), int(n_ranks), static_cast<__nv_bfloat16*>(send_x), send_expert, send_w,
      pair_pos);
  return check_launch("ep_pack_kernel");
}

int qmoe_ep_unpack(const void* y_back, const int32_t* pair_pos, const void* residual, int64_t T,
                   int64_t H, int64_t k, int64_t n_back, void* out, void* stream) {
  QMOE_REQUIRE(y_back && out, QMOE_ERR_INVALID_ARGUMENT, "ep_unpack: null pointer");
  QMOE_REQUIRE(T >= 0 && k >= 1 && k <= 32 && n_back >= 0, QMOE_ERR_INVALID_ARGUMENT, "ep_unpack: bad sizes");
  QMOE_REQUIRE(H > 0 && H % 256 == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "ep_unpack: H %% 256 != 0");
  QMOE_REQUIRE(aligned16(y_back) && aligned16(out) && (!residual || aligned16(residual)),
               QMOE_ERR_MISALIGNED, "ep_unpack: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  const int64_t warps = T * (H / 256);
  if (warps == 0) return QMOE_OK;
  qmoe::ep_unpack_kernel<<<int((warps + 7) / 8), qmoe::kEpThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(y_back), pair_pos, static_cast<const __nv_bfloat16*>(residual),
      int(T), int(H), int(k), int(n_back), static_cast<__nv_bfloat16*>(out));
  return check_launch("ep_unpack_kernel");
}

// ---------------------------------------------------------------------------
// CUDA IPC of caller-allocated buffers (the peer-memory EP path)
// ---------------------------------------------------------------------------
typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

int qmoe_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  QMOE_REQUIRE(ptr && handle_out && offset_out, QMOE_ERR_INVALID_ARGUMENT, "ipc_export: null pointer");
  static GetAddressRangeFn range_fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      range_fn = reinterpret_cast<GetAddressRangeFn>(p);
  });
  QMOE_REQUIRE(range_fn, QMOE_ERR_CUDA, "ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  QMOE_REQUIRE(r == CUDA_SUCCESS, QMOE_ERR_CUDA, "ipc_export: cuMemGetAddressRange failed (%d)", int(r));
  cudaIpcMemHandle_t h;
  cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  QMOE_REQUIRE(err == cudaSuccess, QMOE_ERR_CUDA, "ipc_export: %s", cudaGetErrorString(err));
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = int64_t(reinterpret_cast<uintptr_t>(ptr) - uintptr_t(base));
  return QMOE_OK;
}

int qmoe_ipc_import(const void* handle, int64_t offset, void** ptr_out, void** base_out) {
  QMOE_REQUIRE(handle && ptr_out && base_out && offset >= 0, QMOE_ERR_INVALID_ARGUMENT, "ipc_import: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t err = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  QMOE_REQUIRE(err == cudaSuccess, QMOE_ERR_CUDA, "ipc_import: %s", cudaGetErrorString(err));
  *base_out = base;
  *ptr_out = static_cast<uint8_t*>(base) + offset;
  return QMOE_OK;
}

int qmoe_ipc_close(void* base) {
  QMOE_REQUIRE(base, QMOE_ERR_INVALID_ARGUMENT, "ipc_close: null pointer");
  cudaError_t err = cudaIpcCloseMemHandle(base);
  QMOE_REQUIRE(err == cudaSuccess, QMOE_ERR_CUDA, "ipc_close: %s", cudaGetErrorString(err));
  return QMOE_OK;
}

int64_t qmoe_ep_ctrl_words(int64_t n_ranks, int64_t E) {
  if (n_ranks <= 0 || E <= 0) return 0;
  // both halves, the step counter, ep_wait_unpack's arrival count and the
  // local go words of ep_wait_unpack and ep_wait_expand
  return int64_t(qmoe::ep_step_word(int(n_ranks), int(E))) + 4;
}

int qmoe_ep_exchange_counts(const int32_t* counts, int* const* peer_ctrl, int* my_ctrl, int64_t me,
                            int64_t n_ranks, int64_t E, int64_t e_local, int64_t parity, int64_t epoch,
                            int32_t* dest_base, int32_t* tiles, int64_t max_tiles, int32_t* recv_rows,
                            int64_t cap_rows, int32_t* zero_words, int64_t n_zero_words, void* stream) {
  QMOE_REQUIRE(!zero_words == (n_zero_words == 0) && n_zero_words >= 0 && n_zero_words < (int64_t(1) << 24),
               QMOE_ERR_INVALID_ARGUMENT, "ep_exchange_counts: bad zero_words");
  QMOE_REQUIRE(counts && peer_ctrl && my_ctrl && dest_base && tiles && recv_rows, QMOE_ERR_INVALID_ARGUMENT,
               "ep_exchange_counts: null pointer");
  QMOE_REQUIRE(n_ranks >= 1 && n_ranks <= 32 && me >= 0 && me < n_ranks && E >= 1 && E <= 256 &&
                   e_local >= 1 && e_local * n_ranks == E && (parity == 0 || parity == 1) && epoch >= 0 &&
                   epoch < (int64_t(1) << 31) && max_tiles > 0 && cap_rows > 0 && cap_rows < (int64_t(1) << 31),
               QMOE_ERR_INVALID_ARGUMENT, "ep_exchange_counts: bad sizes");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  return launch_kernel(qmoe::ep_exchange_counts_kernel, dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       true, "ep_exchange_counts_kernel", counts, peer_ctrl, my_ctrl, int(me), int(n_ranks),
                       int(E), int(e_local), int(parity), int(epoch), dest_base, tiles, int(max_tiles),
                       recv_rows, int(cap_rows), zero_words, int(n_zero_words));
}

int qmoe_ep_dispatch(const void* x, const int32_t* topk_idx, const float* topk_w, const int32_t* slot_row,
                     const int32_t* offsets, const int32_t* dest_base, void* const* peer_tok,
                     void* const* peer_recv_meta, int64_t T, int64_t k, int64_t H, int64_t e_local, int64_t me,
                     int64_t n_ranks, int64_t parity, int64_t cap_rows, int64_t max_tokens, void* stream) {
  QMOE_REQUIRE((T == 0 || x) && topk_idx && topk_w && slot_row && offsets && dest_base && peer_tok &&
                   peer_recv_meta,
               QMOE_ERR_INVALID_ARGUMENT, "ep_dispatch: null pointer");
  QMOE_REQUIRE(T >= 0 && k >= 1 && k <= 32 && T * k < (int64_t(1) << 31) && H > 0 && H % 8 == 0 &&
                   e_local >= 1 && n_ranks >= 1 && n_ranks <= 32 && me >= 0 && me < n_ranks &&
                   (parity == 0 || parity == 1) && cap_rows > 0 && T <= max_tokens &&
                   2 * n_ranks * max_tokens < (int64_t(1) << 31),
               QMOE_ERR_INVALID_ARGUMENT, "ep_dispatch: bad sizes");
  QMOE_REQUIRE(aligned16(x), QMOE_ERR_MISALIGNED, "ep_dispatch: x not 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (T == 0) return QMOE_OK;
  const int grid = int(std::min<int64_t>((T * k + 7) / 8, 4 * int64_t(d->sms)));
  return launch_kernel(qmoe::ep_dispatch_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), true,
                       "ep_dispatch_kernel", static_cast<const __nv_bfloat16*>(x), topk_idx, topk_w, slot_row,
                       offsets, dest_base, reinterpret_cast<__nv_bfloat16* const*>(peer_tok),
                       reinterpret_cast<int4* const*>(peer_recv_meta), int(T), int(k), int(H), int(e_local),
                       int(me), int(n_ranks), int(parity), int(cap_rows), int(max_tokens));
}

int qmoe_ep_wait_expand(int* const* peer_ctrl, int* my_ctrl, int64_t n_ranks, int64_t E, int64_t me,
                        int64_t parity, int64_t epoch, const void* tok, int64_t tok_rows, const void* recv_meta,
                        void* recv_x, const int32_t* recv_rows, int64_t cap_rows, int64_t H, void* stream) {
  QMOE_REQUIRE(peer_ctrl && my_ctrl && tok && recv_meta && recv_x && recv_rows, QMOE_ERR_INVALID_ARGUMENT,
               "ep_wait_expand: null pointer");
  QMOE_REQUIRE(n_ranks >= 1 && n_ranks <= 32 && me >= 0 && me < n_ranks && (parity == 0 || parity == 1) &&
                   epoch >= 0 && epoch < (int64_t(1) << 31) && E >= 1 && tok_rows > 0 &&
                   tok_rows < (int64_t(1) << 31) && cap_rows > 0 && cap_rows < (int64_t(1) << 31) && H > 0 &&
                   H % 8 == 0,
               QMOE_ERR_INVALID_ARGUMENT, "ep_wait_expand: bad arguments");
  QMOE_REQUIRE(aligned16(tok) && aligned16(recv_x) && aligned16(recv_meta), QMOE_ERR_MISALIGNED,
               "ep_wait_expand: buffers not 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  return launch_kernel(qmoe::ep_wait_expand_kernel, dim3(d->sms), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       true, "ep_wait_expand_kernel", peer_ctrl, my_ctrl, int(n_ranks), int(E), int(me),
                       int(parity), int(epoch), static_cast<const __nv_bfloat16*>(tok), int(tok_rows),
                       static_cast<const int4*>(recv_meta), static_cast<__nv_bfloat16*>(recv_x), recv_rows,
                       int(cap_rows), int(H));
}

int qmoe_ep_signal_wait(int* const* peer_ctrl, int* my_ctrl, int64_t n_ranks, int64_t E, int64_t me,
                        int64_t parity, int64_t kind, int64_t epoch, void* stream) {
  QMOE_REQUIRE(peer_ctrl && my_ctrl, QMOE_ERR_INVALID_ARGUMENT, "ep_signal_wait: null pointer");
  QMOE_REQUIRE(n_ranks >= 1 && n_ranks <= 32 && me >= 0 && me < n_ranks && (parity == 0 || parity == 1) &&
                   kind >= 0 && kind <= 2 && epoch >= 0 && epoch < (int64_t(1) << 31) && E >= 1,
               QMOE_ERR_INVALID_ARGUMENT, "ep_signal_wait: bad arguments");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  return launch_kernel(qmoe::ep_signal_wait_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), true,
                       "ep_signal_wait_kernel", peer_ctrl, my_ctrl, int(n_ranks), int(E), int(me), int(parity),
                       int(kind), int(epoch));
}

int qmoe_ep_wait_unpack(int* const* peer_ctrl, int* my_ctrl, int64_t n_ranks, int64_t E, int64_t me,
                        int64_t parity, int64_t epoch, const void* y_back, const void* residual, int64_t T,
                        int64_t H, int64_t k, void* out, void* stream) {
  QMOE_REQUIRE(peer_ctrl && my_ctrl && (T == 0 || (y_back && out)), QMOE_ERR_INVALID_ARGUMENT,
               "ep_wait_unpack: null pointer");
  QMOE_REQUIRE(n_ranks >= 1 && n_ranks <= 32 && me >= 0 && me < n_ranks && (parity == 0 || parity == 1) &&
                   epoch >= 0 && epoch < (int64_t(1) << 31) && E >= 1 && T >= 0 && k >= 1 && k <= 32 &&
                   T * k < (int64_t(1) << 31),
               QMOE_ERR_INVALID_ARGUMENT, "ep_wait_unpack: bad arguments");
  QMOE_REQUIRE(H > 0 && H % 256 == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "ep_wait_unpack: H %% 256 != 0");
  QMOE_REQUIRE(aligned16(y_back) && aligned16(out) && (!residual || aligned16(residual)), QMOE_ERR_MISALIGNED,
               "ep_wait_unpack: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  // a warp per (token, 256-column slab), up to 8 CTAs per SM; at least one
  // CTA: the flags are waited for (and the step counter advanced) even when
  // T == 0
  const int64_t warps = T * (H / 256);
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>((warps + 7) / 8, 8 * int64_t(d->sms))));
  return launch_kernel(qmoe::ep_wait_unpack_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       true, "ep_wait_unpack_kernel", peer_ctrl, my_ctrl, int(n_ranks), int(E), int(me),
                       int(parity), int(epoch), static_cast<const __nv_bfloat16*>(y_back),
                       static_cast<const __nv_bfloat16*>(residual), int(T), int(H), int(k),
                       static_cast<__nv_bfloat16*>(out));
}

int qmoe_moe_experts_return(const void* x, const void* w_gate_up, const void* w_down, const int32_t* tiles,
                            int64_t max_tiles, const void* row_meta, void* const* peer_ret, int64_t ret_row0,
                            int64_t n_ret_rows, int64_t n_ranks, int64_t R, int64_t H, int64_t I, int64_t E,
                            void* act, int32_t* done, void* stream) {
  QMOE_REQUIRE(x && w_gate_up && w_down && tiles && row_meta && peer_ret && act && done, QMOE_ERR_INVALID_ARGUMENT,
               "moe_experts_return: null pointer");
  QMOE_REQUIRE(R >= 0 && R < (int64_t(1) << 31) && H > 0 && H % qmoe::kBM == 0 && I > 0 && I % qmoe::kBM == 0 &&
                   E > 0 && E * 2 * I < (int64_t(1) << 31) && E * H < (int64_t(1) << 31) && n_ret_rows > 0 &&
                   ret_row0 >= 0 && n_ranks >= 1 && max_tiles >= 0 && max_tiles < (int64_t(1) << 24),
               QMOE_ERR_INVALID_ARGUMENT, "moe_experts_return: bad sizes");
  QMOE_REQUIRE(aligned16(x) && aligned16(w_gate_up) && aligned16(w_down) && aligned16(act) && aligned16(row_meta),
               QMOE_ERR_MISALIGNED, "moe_experts_return: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (R == 0) return QMOE_OK;
  return launch_moe_fused(x, R, nullptr, w_gate_up, w_down, tiles, max_tiles, nullptr, nullptr, R, H, I, E, act,
                          nullptr, n_ret_rows, done, static_cast<cudaStream_t>(stream), nullptr, nullptr, row_meta,
                          peer_ret, ret_row0, n_ranks);
}

int qmoe_grouped_gemm_down_return(const void* act, const void* w_down, const int32_t* tiles, int64_t max_tiles,
                                  const void* row_meta, void* const* peer_ret, int64_t ret_row0,
                                  int64_t n_ret_rows, int64_t n_ranks, int64_t R, int64_t H, int64_t I,
                                  int64_t E, void* stream) {
  QMOE_REQUIRE(act && w_down && tiles && row_meta && peer_ret, QMOE_ERR_INVALID_ARGUMENT,
               "down_return: null pointer");
  QMOE_REQUIRE(R >= 0 && R < (int64_t(1) << 31) && H > 0 && H % qmoe::kBM == 0 && I > 0 && I % qmoe::kBK == 0 &&
                   E > 0 && E * H < (int64_t(1) << 31) && n_ret_rows > 0 && ret_row0 >= 0 && n_ranks >= 1 &&
                   max_tiles >= 0 && max_tiles < (int64_t(1) << 24),
               QMOE_ERR_INVALID_ARGUMENT, "down_return: bad sizes");
  QMOE_REQUIRE(aligned16(act) && aligned16(w_down) && aligned16(row_meta), QMOE_ERR_MISALIGNED,
               "down_return: pointers must be 16-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (R == 0) return QMOE_OK;
  using C = qmoe::GemmCfg<qmoe::kModeDownReturn>;
  CUtensorMap tmA, tmB;
  QMOE_CHECK(make_tmap_bf16(&tmA, w_down, uint64_t(I), uint64_t(E * H), qmoe::kBK, qmoe::kBM));
  QMOE_CHECK(make_tmap_bf16(&tmB, act, uint64_t(I), uint64_t(R), qmoe::kBK, qmoe::kBoxRows));
  qmoe::GemmArgs a{};
  a.tiles = tiles;
  a.max_tiles = int(max_tiles);
  a.n_mtiles = int(H / qmoe::kBM);
  a.num_kb = int(I / qmoe::kBK);
  a.k_splits = 1;
  a.a_rows_per_expert = int(H);
  a.acc_ld = int(H);
  a.n_acc = int(n_ret_rows);
  a.row_meta = static_cast<const int4*>(row_meta);
  a.peer_ret = reinterpret_cast<__nv_bfloat16* const*>(peer_ret);
  a.ret_row0 = int(ret_row0);
  a.n_ranks = int(n_ranks);
  const int64_t units = max_tiles * a.n_mtiles;
  const int grid = int(std::min<int64_t>(units, d->sms));
  if (grid <= 0) return QMOE_OK;
  QMOE_CHECK(set_smem(qmoe::grouped_gemm_kernel<qmoe::kModeDownReturn>, C::kSmemBytes));
  return launch_kernel(qmoe::grouped_gemm_kernel<qmoe::kModeDownReturn>, dim3(grid), dim3(qmoe::kGemmThreads),
                       C::kSmemBytes, static_cast<cudaStream_t>(stream), true, "grouped_gemm_kernel<down_return>",
                       tmA, tmB, tmB, a);
}

size_t qmoe_moe_forward_workspace_size(int64_t T, int64_t H, int64_t E, int64_t k, int64_t I) {
  if (T < 0 || H <= 0 || E <= 0 || k <= 0 || I <= 0) return 0;
  return fwd_layout(T, H, E, k, I).total;
}

int qmoe_moe_forward(const void* x, const void* w_router, const float* router_bias,
                     const void* w_gate_up, const void* w_down, const void* residual, int64_t T,
                     int64_t H, int64_t E, int64_t k, int64_t I, int normalize, void* out,
                     int32_t* topk_idx, float* topk_w, void* workspace, size_t workspace_bytes,
                     void* stream) {
  QMOE_REQUIRE(x && w_router && w_gate_up && w_down && out, QMOE_ERR_INVALID_ARGUMENT,
               "moe_forward: null pointer");
  QMOE_REQUIRE(T >= 0 && T < (int64_t(1) << 31) / 32, QMOE_ERR_INVALID_ARGUMENT, "moe_forward: bad T");
  QMOE_REQUIRE(H > 0 && H % 256 == 0 && H <= 4096, QMOE_ERR_UNSUPPORTED_SHAPE,
               "moe_forward: H=%lld must be a multiple of 256 and <= 4096", (long long)H);
  QMOE_REQUIRE(E >= 32 && E <= 256 && E % 32 == 0, QMOE_ERR_UNSUPPORTED_SHAPE,
               "moe_forward: E=%lld must be a multiple of 32 in [32, 256]", (long long)E);
  QMOE_REQUIRE(k >= 1 && k <= E && k <= 32, QMOE_ERR_INVALID_ARGUMENT, "moe_forward: k invalid");
  QMOE_REQUIRE(I > 0 && I % qmoe::kBM == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "moe_forward: I %% 128 != 0");
  QMOE_REQUIRE(E * 2 * I < (int64_t(1) << 31) && E * H < (int64_t(1) << 31), QMOE_ERR_UNSUPPORTED_SHAPE,
               "moe_forward: weights too large");
  QMOE_REQUIRE(aligned16(x) && aligned16(w_router) && aligned16(w_gate_up) && aligned16(w_down) &&
                   aligned16(out) && (!residual || aligned16(residual)),
               QMOE_ERR_MISALIGNED, "moe_forward: pointers must be 16-byte aligned");
  const FwdLayout L = fwd_layout(T, H, E, k, I);
  QMOE_REQUIRE(workspace || L.total == 0, QMOE_ERR_INVALID_ARGUMENT, "moe_forward: null workspace");
  QMOE_REQUIRE(workspace_bytes >= L.total, QMOE_ERR_WORKSPACE_TOO_SMALL,
               "moe_forward: workspace %zu < required %zu bytes", workspace_bytes, L.total);
  QMOE_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0, QMOE_ERR_MISALIGNED,
               "moe_forward: workspace must be 256-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (T == 0) return QMOE_OK;
  return moe_forward_on(x, w_router, router_bias, w_gate_up, w_down, residual, T, H, E, k, I, normalize, out,
                        topk_idx, topk_w, static_cast<uint8_t*>(workspace), L, static_cast<cudaStream_t>(stream));
}

size_t qmoe_moe_block_forward_workspace_size(int64_t T, int64_t H, int64_t E, int64_t k, int64_t I) {
  if (T < 0 || H <= 0 || E <= 0 || k <= 0 || I <= 0) return 0;
  return fwd_layout(T, H, E, k, I, true).total;
}

int qmoe_moe_block_forward(const void* x, const void* residual, const float* norm_weight, float eps,
                           const void* w_router, const float* router_bias, const void* w_gate_up,
                           const void* w_down, int64_t T, int64_t H, int64_t E, int64_t k, int64_t I,
                           int normalize, void* out, void* moe_in_out, void* residual_out, int32_t* topk_idx,
                           float* topk_w, void* workspace, size_t workspace_bytes, void* stream) {
  QMOE_REQUIRE(x && residual && norm_weight && w_router && w_gate_up && w_down && out, QMOE_ERR_INVALID_ARGUMENT,
               "moe_block_forward: null pointer");
  QMOE_REQUIRE(T >= 0 && T < (int64_t(1) << 31) / 32, QMOE_ERR_INVALID_ARGUMENT, "moe_block_forward: bad T");
  QMOE_REQUIRE(H > 0 && H % 256 == 0 && H <= 4096, QMOE_ERR_UNSUPPORTED_SHAPE,
               "moe_block_forward: H=%lld must be a multiple of 256 and <= 4096", (long long)H);
  QMOE_REQUIRE(E >= 32 && E <= 256 && E % 32 == 0, QMOE_ERR_UNSUPPORTED_SHAPE,
               "moe_block_forward: E=%lld must be a multiple of 32 in [32, 256]", (long long)E);
  QMOE_REQUIRE(k >= 1 && k <= E && k <= 32, QMOE_ERR_INVALID_ARGUMENT, "moe_block_forward: k invalid");
  QMOE_REQUIRE(I > 0 && I % qmoe::kBM == 0, QMOE_ERR_UNSUPPORTED_SHAPE, "moe_block_forward: I %% 128 != 0");
  QMOE_REQUIRE(E * 2 * I < (int64_t(1) << 31) && E * H < (int64_t(1) << 31), QMOE_ERR_UNSUPPORTED_SHAPE,
               "moe_block_forward: weights too large");
  QMOE_REQUIRE(aligned16(x) && aligned16(residual) && aligned16(norm_weight) && aligned16(w_router) &&
                   aligned16(w_gate_up) && aligned16(w_down) && aligned16(out) &&
                   (!moe_in_out || aligned16(moe_in_out)) && (!residual_out || aligned16(residual_out)),
               QMOE_ERR_MISALIGNED, "moe_block_forward: pointers must be 16-byte aligned");
  const FwdLayout L = fwd_layout(T, H, E, k, I, true);
  QMOE_REQUIRE(workspace || L.total == 0, QMOE_ERR_INVALID_ARGUMENT, "moe_block_forward: null workspace");
  QMOE_REQUIRE(workspace_bytes >= L.total, QMOE_ERR_WORKSPACE_TOO_SMALL,
               "moe_block_forward: workspace %zu < required %zu bytes", workspace_bytes, L.total);
  QMOE_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0, QMOE_ERR_MISALIGNED,
               "moe_block_forward: workspace must be 256-byte aligned");
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  if (T == 0) return QMOE_OK;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const AddNorm an{x, residual, norm_weight, eps, moe_in_out ? moe_in_out : ws + L.norm_h,
                   residual_out ? residual_out : ws + L.norm_res};
  return moe_forward_on(nullptr, w_router, router_bias, w_gate_up, w_down, nullptr, T, H, E, k, I, normalize, out,
                        topk_idx, topk_w, ws, L, static_cast<cudaStream_t>(stream), &an);
}

#ifdef QMOE_TRACE
// Trace build only (not part of the public header): copies the timeline
// stamps out and clears them.
QMOE_API int qmoe_trace_read(void* host, size_t bytes) {
  const size_t n = std::min(bytes, sizeof(qmoe::g_qmoe_trace));
  if (cudaMemcpyFromSymbol(host, qmoe::g_qmoe_trace, n) != cudaSuccess) return QMOE_ERR_CUDA;
  static unsigned long long zeros[qmoe::kTraceKernels * qmoe::kTraceCtas * qmoe::kTraceEvents];
  if (cudaMemcpyToSymbol(qmoe::g_qmoe_trace, zeros, sizeof(zeros)) != cudaSuccess) return QMOE_ERR_CUDA;
  return QMOE_OK;
}
#endif

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of qmoe_moe_forward (no counterpart in the
// reference).  Some callers cannot allocate device memory at the point where
// they run the layer: plugin "enqueue" hooks of inference runtimes may only
// queue work on the stream they are handed (a cudaMalloc there can
// synchronise the whole device), and embedders that own every byte of device
// memory hand this library no workspace.  This entry point takes its scratch
// from the fixed array below instead of a caller workspace.
//
//  - Size limit: kNoAllocScratchBytes (QMOE_NOALLOC_SCRATCH_BYTES, 8 MiB).
//    At Qwen3-30B-A3B shapes (H 2048, 128 experts, top-8, I 768) that holds
//    the scratch of up to 156 tokens per call -- decode-sized batches.
//    Larger calls are rejected with QMOE_ERR_WORKSPACE_TOO_SMALL before
//    anything is launched.
//  - The array lives in every GPU's memory as soon as the library's device
//    code is loaded on that GPU, and stays there until the process exits.
//  - Set-up: the first call on each device looks up the array's device
//    address with cudaGetSymbolAddress (which also loads the module on that
//    device); make that first call before any stream capture.  A failed
//    lookup is not remembered: the next call on that device retries it.
//  - All calls share the one array and it keeps the last call's contents.
//    Nothing in it needs to start at zero: the routing kernels rewrite every
//    index buffer and the permutation kernel zero-fills the fp32 combine
//    accumulator on each call.  Calls that overlap on the GPU (different
//    streams, or several host threads) race on the array: serialise them.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes = QMOE_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices];

// Device address of g_noalloc_scratch on the current device, looked up with
// that device current.  Only a successful lookup is kept: if the first one
// fails (e.g. it was made during a stream capture), the call returns the
// error, clears it from the runtime's per-thread error state, and the next
// call on that device tries again.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_error(QMOE_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices) return set_error(QMOE_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();  // do not leave the failure for the caller's next CUDA check
      return set_error(QMOE_ERR_CUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev,
                       cudaGetErrorString(err));
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return QMOE_OK;
}

}  // namespace

extern "C" int qmoe_moe_forward_noalloc(const void* x, const void* w_router,
                                        const float* router_bias, const void* w_gate_up,
                                        const void* w_down, const void* residual, int64_t T,
                                        int64_t H, int64_t E, int64_t k, int64_t I, int normalize,
                                        void* out, int32_t* topk_idx, float* topk_w, void* stream) {
  QMOE_REQUIRE(x && w_router && w_gate_up && w_down && out, QMOE_ERR_INVALID_ARGUMENT,
               "moe_forward_noalloc: null pointer");
  QMOE_REQUIRE(T >= 0 && T < (int64_t(1) << 31) / 32, QMOE_ERR_INVALID_ARGUMENT,
               "moe_forward_noalloc: bad T");
  QMOE_REQUIRE(H > 0 && H % 256 == 0 && H <= 4096, QMOE_ERR_UNSUPPORTED_SHAPE,
               "moe_forward_noalloc: H=%lld must be a multiple of 256 and <= 4096", (long long)H);
  QMOE_REQUIRE(E >= 32 && E <= 256 && E % 32 == 0, QMOE_ERR_UNSUPPORTED_SHAPE,
               "moe_forward_noalloc: E=%lld must be a multiple of 32 in [32, 256]", (long long)E);
  QMOE_REQUIRE(k >= 1 && k <= E && k <= 32, QMOE_ERR_INVALID_ARGUMENT, "moe_forward_noalloc: k invalid");
  QMOE_REQUIRE(I > 0 && I % qmoe::kBM == 0, QMOE_ERR_UNSUPPORTED_SHAPE,
               "moe_forward_noalloc: I %% 128 != 0");
  QMOE_REQUIRE(E * 2 * I < (int64_t(1) << 31) && E * H < (int64_t(1) << 31), QMOE_ERR_UNSUPPORTED_SHAPE,
               "moe_forward_noalloc: weights too large");
  QMOE_REQUIRE(aligned16(x) && aligned16(w_router) && aligned16(w_gate_up) && aligned16(w_down) &&
                   aligned16(out) && (!residual || aligned16(residual)),
               QMOE_ERR_MISALIGNED, "moe_forward_noalloc: pointers must be 16-byte aligned");
  const FwdLayout L = fwd_layout(T, H, E, k, I);
  QMOE_REQUIRE(L.total <= kNoAllocScratchBytes, QMOE_ERR_WORKSPACE_TOO_SMALL,
               "moe_forward_noalloc: %lld tokens need %zu bytes of scratch but the built-in scratch "
               "holds %zu; use qmoe_moe_forward with a caller workspace",
               (long long)T, L.total, kNoAllocScratchBytes);
  DeviceInfo* d = nullptr;
  QMOE_CHECK(device_info(&d));
  void* scratch = nullptr;
  QMOE_CHECK(noalloc_scratch(&scratch));
  if (T == 0) return QMOE_OK;
  return moe_forward_on(x, w_router, router_bias, w_gate_up, w_down, residual, T, H, E, k, I, normalize, out,
                        topk_idx, topk_w, static_cast<uint8_t*>(scratch), L, static_cast<cudaStream_t>(stream));
}
