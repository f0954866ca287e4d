// b200fa.cu -- host side of libb200fa.so: argument validation, TMA tensor
// maps, persistent-grid launch and the C ABI declared in include/b200fa.h.
//
// Replaces the reference CCE backends' native layers:
//   * shape/dtype checks of binding.py:87-98 and op_host/*.cpp:8-19
//     -> validate() below, returning negative codes instead of raising;
//   * ACLNN GetWorkspaceSize/launch pair (binding.py:20-26, 72-80) and the
//     host tiling Tile() (op_host/*.cpp:53-89) -> b200fa_fwd / _fwd_ex;
//   * PartitionContiguous (cce_task.h:28-35) -> b200fa_partition.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "b200fa.h"
#include "fa_kernel.cuh"

using namespace b200fa;

static_assert(kTimelineOffset == B200FA_WS_TIMELINE_OFFSET, "timeline offset mismatch");
static_assert(kTimelineBlocks == int(B200FA_TIMELINE_BLOCKS) && kTimelineRoles == int(B200FA_TIMELINE_ROLES),
              "timeline size mismatch");
static_assert(kBlockN == B200FA_BLOCK_KEYS, "capture block size mismatch");
static_assert(kFlagCapture == B200FA_FLAG_CAPTURE, "capture flag mismatch");
static_assert(kFlagTestBounds == B200FA_FLAG_TEST_BOUNDS, "test flag mismatch");
static_assert(kFlagCausal == B200FA_FLAG_CAUSAL, "causal flag mismatch");
static_assert(kDevTimeout == B200FA_DEV_TIMEOUT && kDevBounds == B200FA_DEV_BOUNDS && kDevPhase == B200FA_DEV_PHASE,
              "device status codes mismatch");

// Clusters of two CTAs: the pair that shares every tensor-core product.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    b200_fa_fp16_kernel(const __grid_constant__ FwdParams p) {
  attention_fwd_body<0, false>(p);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    b200_fa_fp32_kernel(const __grid_constant__ FwdParams p) {
  attention_fwd_body<1, false>(p);
}

// Debug-capture instantiations (B200FA_FLAG_CAPTURE).
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    b200_fa_fp16_capture_kernel(const __grid_constant__ FwdParams p) {
  attention_fwd_body<0, true>(p);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    b200_fa_fp32_capture_kernel(const __grid_constant__ FwdParams p) {
  attention_fwd_body<1, true>(p);
}

// Causal-mask kernels, defined in b200fa_causal.cu (B200FA_FLAG_CAUSAL).
__global__ void b200_fa_fp16_causal_kernel(const __grid_constant__ FwdParams p);
__global__ void b200_fa_fp32_causal_kernel(const __grid_constant__ FwdParams p);

// Test hook (b200fa_test_exp2): the softmax's two exponential forms on an
// array, pairwise as the softmax evaluates them -- exp2_poly2 (FMA pipe) into
// `poly`, MUFU ex2.approx into `mufu`.
__global__ void __launch_bounds__(256) exp2_probe_kernel(const float* x, float* poly, float* mufu, int64_t n) {
  const int64_t i = 2 * (int64_t(blockIdx.x) * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const bool two = i + 1 < n;
  const float a = x[i], b = two ? x[i + 1] : x[i];
  float pa, pb;
  f2_unpack(exp2_poly2(f2_pack(a, b)), pa, pb);
  poly[i] = pa;
  mufu[i] = ex2_approx(a);
  if (two) {
    poly[i + 1] = pb;
    mufu[i + 1] = ex2_approx(b);
  }
}

using KernelFn = void (*)(FwdParams);

KernelFn kernel_for(int variant, bool capture, bool causal) {
  if (capture) return variant == B200FA_VARIANT_FP16 ? b200_fa_fp16_capture_kernel : b200_fa_fp32_capture_kernel;
  if (causal) return variant == B200FA_VARIANT_FP16 ? b200_fa_fp16_causal_kernel : b200_fa_fp32_causal_kernel;
  return variant == B200FA_VARIANT_FP16 ? b200_fa_fp16_kernel : b200_fa_fp32_kernel;
}

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(static_cast<int>(e), "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
}

constexpr int64_t kMax31 = (int64_t(1) << 31) - 1;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Per-device facts read once: kernel attributes set, and how many CTA pairs
// can be resident at once (one per TPC whose two SMs are both available).
struct DeviceState {
  std::once_flag once;
  int pairs = 0;
  cudaError_t err = cudaSuccess;
};
DeviceState g_devices[64];

int device_setup(int dev, int* pairs) {
  if (dev < 0 || dev >= 64) return fail(B200FA_ERR_OPTIONS, "device ordinal %d out of range", dev);
  DeviceState& d = g_devices[dev];
  std::call_once(d.once, [&d] {
    cudaError_t e = cudaSuccess;
    for (int variant : {B200FA_VARIANT_FP16, B200FA_VARIANT_FP32})
      for (int kind = 0; kind < 3; ++kind)  // product, capture, causal
        if (e == cudaSuccess)
          e = cudaFuncSetAttribute(kernel_for(variant, kind == 1, kind == 2),
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(2, 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = kSmemBytes;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      e = cudaOccupancyMaxActiveClusters(&d.pairs, b200_fa_fp16_kernel, &cfg);
      if (e == cudaSuccess && d.pairs < 1) e = cudaErrorInvalidConfiguration;
    }
    d.err = e;
  });
  if (d.err != cudaSuccess) return cuda_fail(d.err, "device setup");
  *pairs = d.pairs;
  return B200FA_OK;
}

// Persistent grid: one CTA pair per resident slot, at most one per item;
// `max_ctas` (when set) caps the CTAs, rounded down to whole pairs (>= 1).
int grid_ctas(int pairs, int32_t max_ctas, int64_t items) {
  int64_t n = pairs;
  if (max_ctas > 0 && max_ctas / 2 < n) n = max_ctas / 2 > 0 ? max_ctas / 2 : 1;
  if (n > B200FA_MAX_CTAS / 2) n = B200FA_MAX_CTAS / 2;
  if (items < n) n = items;
  return int(2 * n);
}

int validate_shape(int64_t B, int64_t Hq, int64_t Hkv, int64_t Nq, int64_t Nk, int64_t D) {
  if (D != kHeadDim) return fail(B200FA_ERR_HEAD_DIM, "head dim must be 128, got %lld", (long long)D);
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Nq <= 0 || Nk <= 0)
    return fail(B200FA_ERR_SHAPE, "invalid attention geometry B=%lld Hq=%lld Hkv=%lld Nq=%lld Nk=%lld",
                (long long)B, (long long)Hq, (long long)Hkv, (long long)Nq, (long long)Nk);
  if (Hq % Hkv != 0)
    return fail(B200FA_ERR_GROUPING, "Hq (%lld) must be a multiple of Hkv (%lld)", (long long)Hq, (long long)Hkv);
  if (Nq > kMax31 || Nk > kMax31 || B * Hq > kMax31 || B * Hkv > kMax31)
    return fail(B200FA_ERR_TOO_LARGE, "Nq, Nk and B*H must be below 2^31");
  const int64_t units = B * Hq * ceil_div<int64_t>(Nq, kBlockM);
  if (units > kMax31) return fail(B200FA_ERR_TOO_LARGE, "work unit count %lld exceeds 2^31-1", (long long)units);
  return B200FA_OK;
}

int encode_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t planes, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (!fn) return fail(B200FA_ERR_NO_DRIVER, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[3] = {cuuint64_t(kHeadDim), cuuint64_t(rows), cuuint64_t(planes)};
  const cuuint64_t strides[2] = {cuuint64_t(kHeadDim * 2), cuuint64_t(rows) * kHeadDim * 2};
  const cuuint32_t box[3] = {64, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200FA_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return B200FA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The caller's options as a full struct: NULL means defaults, and the
// 16-byte layout without the capture fields is accepted as well.
constexpr uint32_t kOptionsV1Bytes = 16;
int read_options(const b200fa_options* in, b200fa_options* out) {
  *out = b200fa_options{sizeof(b200fa_options), 0u, 0u, 0, nullptr, 0};
  if (in == nullptr) return B200FA_OK;
  if (in->struct_size == sizeof(b200fa_options)) {
    *out = *in;
  } else if (in->struct_size == kOptionsV1Bytes) {
    std::memcpy(out, in, kOptionsV1Bytes);
    out->struct_size = sizeof(b200fa_options);
    out->capture = nullptr;
    out->capture_bytes = 0;
  } else {
    return fail(B200FA_ERR_OPTIONS, "b200fa_options.struct_size mismatch");
  }
  return B200FA_OK;
}

int64_t capture_bytes(int64_t B, int64_t Hq, int64_t Nq, int64_t Nk) {
  // four scalar planes (m, l, alpha, z) + the O plane (kHeadDim floats per record)
  return int64_t(4 + kHeadDim) * 4 * B * Hq * ceil_div<int64_t>(Nk, kBlockN) * Nq;
}

// Capture buffer checks (B200FA_FLAG_CAPTURE).
int check_capture(const b200fa_options& o, int64_t B, int64_t Hq, int64_t Nq, int64_t Nk) {
  if ((o.flags & B200FA_FLAG_CAPTURE) == 0) return B200FA_OK;
  if (o.flags & B200FA_FLAG_CAUSAL)
    return fail(B200FA_ERR_OPTIONS, "B200FA_FLAG_CAPTURE is not supported together with B200FA_FLAG_CAUSAL");
  const uint64_t need = uint64_t(capture_bytes(B, Hq, Nq, Nk));
  if (o.capture == nullptr || (reinterpret_cast<uintptr_t>(o.capture) & 15u) != 0 || o.capture_bytes < need)
    return fail(B200FA_ERR_OPTIONS, "B200FA_FLAG_CAPTURE needs a 16-byte aligned buffer of at least %llu bytes",
                (unsigned long long)need);
  return B200FA_OK;
}

// Argument checks shared by b200fa_fwd_ex and b200fa_fwd_noalloc, in the
// order both report them: pointers, shape, variant, scale, unit range,
// alignment.
int check_args(const void* q, const void* k, const void* v, const void* o, int64_t B, int64_t Hq, int64_t Hkv,
               int64_t Nq, int64_t Nk, int64_t D, float scale, int32_t variant, int64_t unit_begin,
               int64_t unit_end) {
  if (!q || !k || !v || !o) return fail(B200FA_ERR_NULL, "q, k, v and o must be device pointers");
  int rc = validate_shape(B, Hq, Hkv, Nq, Nk, D);
  if (rc != B200FA_OK) return rc;
  if (variant != B200FA_VARIANT_FP16 && variant != B200FA_VARIANT_FP32)
    return fail(B200FA_ERR_VARIANT, "unknown variant %d", variant);
  if (!std::isfinite(scale) || !(scale > 0.f)) return fail(B200FA_ERR_SCALE, "scale must be finite and positive");
  const int64_t units = B * Hq * ceil_div<int64_t>(Nq, kBlockM);
  if (unit_begin < 0 || unit_end > units || unit_begin > unit_end)
    return fail(B200FA_ERR_UNIT_RANGE, "unit range [%lld, %lld) outside [0, %lld)", (long long)unit_begin,
                (long long)unit_end, (long long)units);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(B200FA_ERR_ALIGNMENT, "tensor pointers must be 16-byte aligned");
  return B200FA_OK;
}

// Options (NULL = defaults) and the capture buffer check; *items = work items
// of the unit range (0: nothing to launch).
int read_call_options(const b200fa_options* opts, int64_t B, int64_t Hq, int64_t Nq, int64_t Nk, int64_t unit_begin,
                      int64_t unit_end, b200fa_options* o_full, int64_t* items) {
  int rc = read_options(opts, o_full);
  if (rc != B200FA_OK) return rc;
  if ((rc = check_capture(*o_full, B, Hq, Nq, Nk)) != B200FA_OK) return rc;
  *items = plan_count<int64_t>(ceil_div<int64_t>(Nq, kBlockM), unit_begin, unit_end);
  return B200FA_OK;
}

// Tensor maps and kernel parameters of one call; `ws` is the device scratch
// (status header, trace records, timeline) the kernel writes.
int fill_params(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t Hq, int64_t Hkv, int64_t Nq,
                int64_t Nk, float scale, int64_t unit_begin, int64_t unit_end, int64_t items,
                const b200fa_options& opts, void* ws, FwdParams* p) {
  std::memset(p, 0, sizeof(*p));
  int rc;
  if ((rc = encode_map(&p->tm_q, q, Nq, B * Hq, kBlockM)) != B200FA_OK) return rc;
  if ((rc = encode_map(&p->tm_k, k, Nk, B * Hkv, kKBoxRows)) != B200FA_OK) return rc;
  if ((rc = encode_map(&p->tm_v, v, Nk, B * Hkv, kBlockN)) != B200FA_OK) return rc;
  if ((rc = encode_map(&p->tm_o, o, Nq, B * Hq, kBlockM)) != B200FA_OK) return rc;
  p->Hq = int32_t(Hq);
  p->Hkv = int32_t(Hkv);
  p->group = int32_t(Hq / Hkv);
  p->nqb = int32_t(ceil_div<int64_t>(Nq, kBlockM));
  p->n_kv = int32_t(ceil_div<int64_t>(Nk, kBlockN));
  p->nk_tail = int32_t(Nk - int64_t(p->n_kv - 1) * kBlockN);
  p->unit_begin = int32_t(unit_begin);
  p->unit_end = int32_t(unit_end);
  p->num_items = int32_t(items);
  p->scale_log2 = float(double(scale) * 1.4426950408889634074);
  p->flags = opts.flags;
  p->timeout_ns = uint64_t(opts.timeout_us ? opts.timeout_us : 2000000u) * 1000ull;
  p->ws = static_cast<uint32_t*>(ws);
  p->capture = (opts.flags & B200FA_FLAG_CAPTURE) ? opts.capture : nullptr;
  p->heads = int32_t(B * Hq);
  p->nq = int32_t(Nq);
  return B200FA_OK;
}

int launch(int32_t variant, const FwdParams& p, int grid, void* stream, const char* where) {
  kernel_for(variant, p.capture != nullptr, (p.flags & kFlagCausal) != 0)<<<grid, kThreads, kSmemBytes,
                                                                          static_cast<cudaStream_t>(stream)>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, where);
  return B200FA_OK;
}

}  // namespace

extern "C" {

int64_t b200fa_num_units(int64_t B, int64_t Hq, int64_t Nq) {
  if (B <= 0 || Hq <= 0 || Nq <= 0) return fail(B200FA_ERR_SHAPE, "non-positive size");
  return B * Hq * ceil_div<int64_t>(Nq, kBlockM);
}

int b200fa_partition(int64_t total, int32_t parts, int32_t index, int64_t* begin, int64_t* end) {
  if (!begin || !end) return fail(B200FA_ERR_NULL, "begin/end must not be NULL");
  if (total < 0 || parts <= 0 || index < 0 || index >= parts)
    return fail(B200FA_ERR_UNIT_RANGE, "bad partition total=%lld parts=%d index=%d", (long long)total, parts, index);
  const int64_t base = total / parts, rem = total % parts;
  *begin = index * base + (index < rem ? index : rem);
  *end = *begin + base + (index < rem ? 1 : 0);
  return B200FA_OK;
}

int64_t b200fa_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Nq, int64_t Nk, int64_t D,
                              int32_t variant) {
  const int rc = validate_shape(B, Hq, Hkv, Nq, Nk, D);
  if (rc != B200FA_OK) return rc;
  if (variant != B200FA_VARIANT_FP16 && variant != B200FA_VARIANT_FP32)
    return fail(B200FA_ERR_VARIANT, "unknown variant %d", variant);
  return int64_t(B200FA_WS_TIMELINE_OFFSET) + int64_t(B200FA_WS_TIMELINE_BYTES);
}

int64_t b200fa_plan_item(int64_t B, int64_t Hq, int64_t Nq, int64_t unit_begin, int64_t unit_end, int64_t index,
                         int64_t* bh, int64_t* qblock, int64_t* count) {
  const int64_t units = b200fa_num_units(B, Hq, Nq);
  if (units < 0) return units;
  if (unit_begin < 0 || unit_end > units || unit_begin > unit_end)
    return fail(B200FA_ERR_UNIT_RANGE, "unit range [%lld, %lld) outside [0, %lld)", (long long)unit_begin,
                (long long)unit_end, (long long)units);
  const int64_t nqb = ceil_div<int64_t>(Nq, kBlockM);
  const int64_t n = plan_count<int64_t>(nqb, unit_begin, unit_end);
  if (index >= 0 && index < n && bh && qblock && count) plan_decode<int64_t>(nqb, unit_begin, unit_end, index, *bh, *qblock, *count);
  return n;
}

int b200fa_fwd_ex(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t Hq, int64_t Hkv,
                  int64_t Nq, int64_t Nk, int64_t D, float scale, int32_t variant, int64_t unit_begin,
                  int64_t unit_end, void* workspace, uint64_t ws_bytes, void* stream, const b200fa_options* opts) {
  g_last_error[0] = '\0';
  int rc = check_args(q, k, v, o, B, Hq, Hkv, Nq, Nk, D, scale, variant, unit_begin, unit_end);
  if (rc != B200FA_OK) return rc;
  const uint64_t ws_need = uint64_t(B200FA_WS_TIMELINE_OFFSET) + uint64_t(B200FA_WS_TIMELINE_BYTES);
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0 || ws_bytes < ws_need)
    return fail(B200FA_ERR_WORKSPACE, "workspace must be 256-byte aligned and at least %llu bytes",
                (unsigned long long)ws_need);
  b200fa_options o_full;
  int64_t items = 0;
  if ((rc = read_call_options(opts, B, Hq, Nq, Nk, unit_begin, unit_end, &o_full, &items)) != B200FA_OK) return rc;
  if (items == 0) return B200FA_OK;  // empty shard: nothing to launch

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int pairs = 0;
  if ((rc = device_setup(dev, &pairs)) != B200FA_OK) return rc;
  FwdParams p;
  if ((rc = fill_params(q, k, v, o, B, Hq, Hkv, Nq, Nk, scale, unit_begin, unit_end, items, o_full, workspace, &p)) !=
      B200FA_OK)
    return rc;
  return launch(variant, p, grid_ctas(pairs, o_full.max_ctas, items), stream, "kernel launch");
}

int b200fa_fwd(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t Hq, int64_t Hkv, int64_t Nq,
               int64_t Nk, int64_t D, float scale, int32_t variant, int64_t unit_begin, int64_t unit_end,
               void* workspace, uint64_t ws_bytes, void* stream) {
  return b200fa_fwd_ex(q, k, v, o, B, Hq, Hkv, Nq, Nk, D, scale, variant, unit_begin, unit_end, workspace, ws_bytes,
                       stream, nullptr);
}

int b200fa_read_status(const void* workspace, void* stream, uint32_t* status) {
  if (!workspace || !status) return fail(B200FA_ERR_NULL, "workspace and status must not be NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  e = cudaMemcpy(status, workspace, 4 * sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy status");
  return B200FA_OK;
}

int b200fa_reset_status(void* workspace, void* stream) {
  if (!workspace) return fail(B200FA_ERR_NULL, "workspace must not be NULL");
  const cudaError_t e = cudaMemsetAsync(workspace, 0, B200FA_WS_HEADER_BYTES, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync status");
  return B200FA_OK;
}

const char* b200fa_kernel_name(int32_t variant) {
  if (variant == B200FA_VARIANT_FP16) return "b200_fa_fp16_kernel";
  if (variant == B200FA_VARIANT_FP32) return "b200_fa_fp32_kernel";
  return nullptr;
}

int64_t b200fa_capture_bytes(int64_t B, int64_t Hq, int64_t Nq, int64_t Nk) {
  if (B <= 0 || Hq <= 0 || Nq <= 0 || Nk <= 0) return fail(B200FA_ERR_SHAPE, "non-positive size");
  return capture_bytes(B, Hq, Nq, Nk);
}

const char* b200fa_last_error_string(void) { return g_last_error; }

int b200fa_test_exp2(const float* x, float* poly, float* mufu, int64_t n, void* stream) {
  g_last_error[0] = '\0';
  if (!x || !poly || !mufu) return fail(B200FA_ERR_NULL, "x, poly and mufu must be device pointers");
  if (n < 0 || n > kMax31) return fail(B200FA_ERR_SHAPE, "n must be in [0, 2^31)");
  if (n == 0) return B200FA_OK;
  const int64_t pairs = (n + 1) / 2;
  const int blocks = int((pairs + 255) / 256);
  exp2_probe_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, poly, mufu, n);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "exp2 test kernel launch");
  return B200FA_OK;
}

const char* b200fa_version(void) { return "b200fa 0.1 sm_100a"; }

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point (b200fa_fwd_noalloc).  For callers that cannot
// hand the library a workspace -- a C/FFI host without a device allocator, a
// runtime that owns the whole device pool, a path that must not call
// cudaMalloc because it can synchronize the device.  The kernel's scratch
// (status header + trace records) lives in this file-scope device array
// instead: one copy per device that loads the library, kept until exit.
namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[B200FA_NOALLOC_SCRATCH_BYTES];

struct NoAllocScratch {
  std::once_flag once;
  void* ptr = nullptr;
  cudaError_t err = cudaSuccess;
};
NoAllocScratch g_noalloc[64];

// Device address of device `dev`'s copy of g_noalloc_scratch.  In host code
// the array's name is only a host-side stand-in, so the address is resolved
// once per device, with that device current, and cached.
int noalloc_scratch(int dev, void** out) {
  if (dev < 0 || dev >= 64) return fail(B200FA_ERR_OPTIONS, "device ordinal %d out of range", dev);
  NoAllocScratch& s = g_noalloc[dev];
  std::call_once(s.once, [&s] { s.err = cudaGetSymbolAddress(&s.ptr, g_noalloc_scratch); });
  if (s.err != cudaSuccess) return cuda_fail(s.err, "cudaGetSymbolAddress(g_noalloc_scratch)");
  *out = s.ptr;
  return B200FA_OK;
}

}  // namespace

extern "C" int b200fa_fwd_noalloc(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t Hq,
                                  int64_t Hkv, int64_t Nq, int64_t Nk, int64_t D, float scale, int32_t variant,
                                  int64_t unit_begin, int64_t unit_end, void* stream, const b200fa_options* opts,
                                  void** scratch_out) {
  g_last_error[0] = '\0';
  int rc = check_args(q, k, v, o, B, Hq, Hkv, Nq, Nk, D, scale, variant, unit_begin, unit_end);
  if (rc != B200FA_OK) return rc;
  b200fa_options o_full;
  int64_t items = 0;
  if ((rc = read_call_options(opts, B, Hq, Nq, Nk, unit_begin, unit_end, &o_full, &items)) != B200FA_OK) return rc;
  if (o_full.flags & B200FA_FLAG_TIMELINE)
    return fail(B200FA_ERR_WORKSPACE,
                "b200fa_fwd_noalloc does not support B200FA_FLAG_TIMELINE: the timeline needs %u bytes of scratch "
                "and the static scratch holds %u; use b200fa_fwd_ex with a workspace",
                unsigned(B200FA_WS_TIMELINE_BYTES), unsigned(B200FA_NOALLOC_SCRATCH_BYTES));

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int pairs = 0;
  if ((rc = device_setup(dev, &pairs)) != B200FA_OK) return rc;
  void* scratch = nullptr;
  if ((rc = noalloc_scratch(dev, &scratch)) != B200FA_OK) return rc;
  if (scratch_out) *scratch_out = scratch;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (items == 0) {
    // Nothing to launch; the status read through scratch_out must still
    // describe this call, not an earlier one.
    e = cudaMemsetAsync(scratch, 0, B200FA_WS_HEADER_BYTES, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(noalloc status header)");
    return B200FA_OK;
  }
  const int grid = grid_ctas(pairs, o_full.max_ctas, items);
  const uint64_t need = uint64_t(B200FA_WS_HEADER_BYTES) +
                        ((o_full.flags & B200FA_FLAG_TRACE) ? uint64_t(B200FA_WS_TRACE_BYTES) * uint64_t(grid) : 0u);
  if (need > B200FA_NOALLOC_SCRATCH_BYTES)
    return fail(B200FA_ERR_WORKSPACE,
                "b200fa_fwd_noalloc: this call needs %llu bytes of scratch (trace records for %d CTAs) but the "
                "static scratch holds %u (trace for at most %u CTAs); set max_ctas <= %u or drop B200FA_FLAG_TRACE",
                (unsigned long long)need, grid, (unsigned)B200FA_NOALLOC_SCRATCH_BYTES,
                (unsigned)B200FA_NOALLOC_TRACE_CTAS, (unsigned)B200FA_NOALLOC_TRACE_CTAS);

  FwdParams p;
  if ((rc = fill_params(q, k, v, o, B, Hq, Hkv, Nq, Nk, scale, unit_begin, unit_end, items, o_full, scratch, &p)) !=
      B200FA_OK)
    return rc;
  // The array keeps the previous call's contents: the status header must start
  // at zero for this call.  Trace records are rewritten by every CTA that runs.
  e = cudaMemsetAsync(scratch, 0, B200FA_WS_HEADER_BYTES, st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(noalloc status header)");
  return launch(variant, p, grid, stream, "kernel launch (noalloc)");
}
