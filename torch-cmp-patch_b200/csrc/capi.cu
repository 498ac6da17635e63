// capi.cu -- the extern "C" entry points declared in include/cmpx_b200.h.
//
// This layer replaces the argument handling of the reference's pybind functions
// (custom_attention_forward src/main.cpp:1603-1774, custom_bmm_forward src/main.cpp:363-441):
// it validates the descriptor, picks the tile-table entry (a fixed function of dtype / shape /
// layout -- the reference decided at run time by racing its kernel against stock,
// cmpext3/autoselect.py:290-364), and launches on the caller's stream.  It never allocates,
// never synchronises on the hot path, and returns a status instead of throwing.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <mutex>

#include "cmpx_internal.h"
#include "cmpx_ptx.cuh"

namespace cmpx {

// Device status word (one per device: every device that loads the module has its own copy).
__device__ unsigned int g_dev_flags;

namespace {

constexpr int kMaxDevices = 64;

struct DeviceState {
  std::once_flag once;
  int status = CMPX_ERR_DEVICE;
  unsigned int* flags = nullptr;
  int num_sms = 0;
};
DeviceState g_devices[kMaxDevices];

unsigned long long wait_timeout_ns() {
  static const unsigned long long v = [] {
    const char* s = std::getenv("CMPX_WAIT_TIMEOUT_MS");
    long long ms = s ? std::atoll(s) : 0;
    if (ms <= 0) ms = 2000;
    return static_cast<unsigned long long>(ms) * 1000000ull;
  }();
  return v;
}

// Resolves the per-device state once (with that device current): checks for sm_100 and looks
// up the device address of the status word.
int device_ctx(LaunchCtx* ctx, cudaStream_t stream) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CMPX_ERR_DEVICE;
  DeviceState& ds = g_devices[dev];
  std::call_once(ds.once, [&] {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return;
    if (prop.major != 10) return;  // sm_100 family only: the kernels are built for sm_100a
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_dev_flags) != cudaSuccess) return;
    ds.flags = static_cast<unsigned int*>(ptr);
    ds.num_sms = prop.multiProcessorCount;
    ds.status = CMPX_OK;
  });
  if (ds.status != CMPX_OK) {
    cudaGetLastError();
    return ds.status;
  }
  ctx->stream = stream;
  ctx->dev_flags = ds.flags;
  ctx->timeout_ns = wait_timeout_ns();
  ctx->num_sms = ds.num_sms;
  return CMPX_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

bool attn_desc_valid(const cmpx_attn_desc* d) {
  if (!d || !d->q || !d->k || !d->v || !d->o) return false;
  if (d->batch < 0 || d->heads < 0 || d->len_q < 0 || d->len_k < 0 || d->head_dim <= 0) return false;
  if (!std::isfinite(d->scale)) return false;
  // grouped-query attention: heads_kv (0 = heads) must divide heads
  if (d->heads_kv < 0 || (d->heads_kv > 0 && (d->heads_kv > d->heads || d->heads % d->heads_kv != 0)))
    return false;
  if (d->mask) {  // strides: 0 (broadcast) or positive; the key stride must be 1
    for (int i = 0; i < 3; ++i)
      if (d->mask_stride[i] < 0) return false;
    if (d->mask_stride[3] != 1) return false;
    if (d->mask_kind != CMPX_MASK_BOOL && d->mask_kind != CMPX_MASK_ADD) return false;
  }
  return true;
}

bool bmm_desc_valid(const cmpx_bmm_desc* d) {
  if (!d || !d->a || !d->b || !d->c) return false;
  if (d->batch < 0 || d->m < 0 || d->n < 0 || d->k < 0) return false;
  return true;
}

// Shape checks shared by every attention kernel (beyond what each kernel's own plan checks).
int attn_common_checks(const cmpx_attn_desc* d) {
  if (!attn_desc_valid(d)) return CMPX_ERR_INVALID_ARGUMENT;
  if (d->scale == 0.0) return CMPX_ERR_UNSUPPORTED_SHAPE;  // uniform softmax: left to stock
  if (d->len_k == 0 && d->len_q > 0) return CMPX_ERR_UNSUPPORTED_SHAPE;  // empty softmax
  if (d->len_q > (1ll << 31) - 1024 || d->len_k > (1ll << 31) - 1024) return CMPX_ERR_UNSUPPORTED_SHAPE;
  if (d->causal != 0 && d->causal != 1) return CMPX_ERR_INVALID_ARGUMENT;
  return CMPX_OK;
}

const char* attn_plan_impl(const cmpx_attn_desc* d, int* st) {
  *st = attn_common_checks(d);
  if (*st != CMPX_OK) return "none";
  if (d->dtype == CMPX_F32) return attn_f32_plan(d, st);
  if (d->dtype == CMPX_F16 || d->dtype == CMPX_BF16) return fmha_sm100_plan(d, st);
  *st = CMPX_ERR_UNSUPPORTED_DTYPE;
  return "none";
}

const char* bmm_plan_impl(const cmpx_bmm_desc* d, int* st) {
  if (!bmm_desc_valid(d)) {
    *st = CMPX_ERR_INVALID_ARGUMENT;
    return "none";
  }
  if (d->dtype == CMPX_F16 || d->dtype == CMPX_BF16) return bmm_sm100_plan(d, st);
  if (d->dtype == CMPX_F32) return bmm_x3_plan(d, st);
  *st = CMPX_ERR_UNSUPPORTED_DTYPE;
  return "none";
}

const char* linear_plan_impl(const cmpx_linear_desc* d, int* st) {
  if (!d || !d->x || !d->w || !d->y) {
    *st = CMPX_ERR_INVALID_ARGUMENT;
    return "none";
  }
  if (d->dtype == CMPX_F16 || d->dtype == CMPX_BF16) return linear_sm100_plan(d, st);
  if (d->dtype == CMPX_F32) return linear_x3_plan(d, st);
  *st = CMPX_ERR_UNSUPPORTED_DTYPE;
  return "none";
}

void copy_name(const char* name, char* buf, size_t len) {
  if (!buf || len == 0) return;
  std::strncpy(buf, name, len - 1);
  buf[len - 1] = '\0';
}

__global__ void wait_selftest_kernel(unsigned long long timeout_ns, unsigned int* dev_flags) {
  __shared__ __align__(8) unsigned long long bar_storage;
  __shared__ int abort_word;
  const uint32_t bar = smem_u32(&bar_storage);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    abort_word = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const WaitCtl ctl{reinterpret_cast<volatile int*>(&abort_word), dev_flags, timeout_ns};
    mbar_wait(bar, 0, ctl);  // nothing arrives: returns false after timeout_ns, flag raised
  }
  __syncthreads();
}

}  // namespace

bool encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i] == 0 ? 1 : dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstride[i] = strides_bytes[i];
  const CUresult r = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), gdim,
                        gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int launch_wait_selftest(uint64_t timeout_ns, const LaunchCtx& ctx) {
  wait_selftest_kernel<<<1, 32, 0, ctx.stream>>>(timeout_ns, ctx.dev_flags);
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

// SM count of the current device (148, a B200's, when no device can be queried: sizes computed
// from it are upper bounds that a launch on fewer SMs checks again).
int current_num_sms() {
  int dev = -1;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
    LaunchCtx ctx;
    if (device_ctx(&ctx, nullptr) == CMPX_OK && ctx.num_sms > 0) return ctx.num_sms;
  }
  cudaGetLastError();
  return 148;
}

}  // namespace cmpx

using namespace cmpx;

extern "C" {

int cmpx_abi_version(void) { return CMPX_ABI_VERSION; }

const char* cmpx_status_str(int status) {
  switch (status) {
    case CMPX_OK: return "ok";
    case CMPX_ERR_INVALID_ARGUMENT: return "invalid argument";
    case CMPX_ERR_UNSUPPORTED_SHAPE: return "unsupported shape (outside the tile table)";
    case CMPX_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case CMPX_ERR_MISALIGNED: return "pointer or stride not 16-byte aligned for TMA";
    case CMPX_ERR_WORKSPACE: return "workspace missing or too small";
    case CMPX_ERR_LAUNCH: return "kernel launch or tensor-map encode failed";
    case CMPX_ERR_DEVICE: return "no usable sm_100 device is current";
    case CMPX_ERR_DEVICE_TIMEOUT: return "a device-side wait timed out";
    default: return "unknown status";
  }
}

size_t cmpx_attn_workspace_size(const cmpx_attn_desc* desc) {
  // The persistent 16-bit kernels keep two work counters (next item, CTAs finished); a non-causal
  // call whose last wave of items is partial also parks the split items' partial results.  An fp32
  // call needs workspace only for such a split (and runs without it when given none).
  if (!desc) return 0;
  if (desc->dtype == CMPX_F32) return attn_tf32x3_workspace_bytes(desc, current_num_sms());
  if (desc->dtype != CMPX_F16 && desc->dtype != CMPX_BF16) return 0;
  return fmha_workspace_bytes(desc, current_num_sms());
}

int cmpx_attn_plan(const cmpx_attn_desc* desc, char* buf, size_t buf_len) {
  int st = CMPX_OK;
  const char* name = attn_plan_impl(desc, &st);
  copy_name(st == CMPX_OK ? name : "none", buf, buf_len);
  return st;
}

int cmpx_bmm_plan(const cmpx_bmm_desc* desc, char* buf, size_t buf_len) {
  int st = CMPX_OK;
  const char* name = bmm_plan_impl(desc, &st);
  copy_name(st == CMPX_OK ? name : "none", buf, buf_len);
  return st;
}

int cmpx_linear_plan(const cmpx_linear_desc* desc, char* buf, size_t buf_len) {
  int st = CMPX_OK;
  const char* name = linear_plan_impl(desc, &st);
  copy_name(st == CMPX_OK ? name : "none", buf, buf_len);
  return st;
}

int cmpx_linear(const cmpx_linear_desc* desc, void* stream) {
  int st = CMPX_OK;
  linear_plan_impl(desc, &st);
  if (st != CMPX_OK) return st;
  if (desc->m == 0) return CMPX_OK;
  LaunchCtx ctx;
  st = device_ctx(&ctx, static_cast<cudaStream_t>(stream));
  if (st != CMPX_OK) return st;
  if (desc->dtype == CMPX_F32) return launch_linear_x3(desc, ctx);
  return launch_linear_sm100(desc, ctx);
}

int cmpx_attn_fwd(const cmpx_attn_desc* desc, void* stream) {
  int st = CMPX_OK;
  attn_plan_impl(desc, &st);
  if (st != CMPX_OK) return st;
  if (desc->batch == 0 || desc->heads == 0 || desc->len_q == 0) return CMPX_OK;
  if ((desc->dtype == CMPX_F16 || desc->dtype == CMPX_BF16) &&
      (!desc->workspace || desc->workspace_bytes < fmha_workspace_min(desc) ||
       (reinterpret_cast<uintptr_t>(desc->workspace) & 15u) != 0))
    return CMPX_ERR_WORKSPACE;
  LaunchCtx ctx;
  st = device_ctx(&ctx, static_cast<cudaStream_t>(stream));
  if (st != CMPX_OK) return st;
  if (desc->dtype == CMPX_F32) return launch_attn_f32(desc, ctx);
  return launch_fmha_sm100(desc, ctx);
}

int cmpx_bmm(const cmpx_bmm_desc* desc, void* stream) {
  int st = CMPX_OK;
  bmm_plan_impl(desc, &st);
  if (st != CMPX_OK) return st;
  if (desc->batch == 0 || desc->m == 0 || desc->n == 0) return CMPX_OK;
  LaunchCtx ctx;
  st = device_ctx(&ctx, static_cast<cudaStream_t>(stream));
  if (st != CMPX_OK) return st;
  if (desc->dtype == CMPX_F32) return launch_bmm_x3(desc, ctx);
  return launch_bmm_sm100(desc, ctx);
}

size_t cmpx_bmm_workspace_size(const cmpx_bmm_desc* desc) {
  if (!desc || desc->dtype != CMPX_F32) return 0;
  return bmm_x3_workspace_bytes(desc);
}

int cmpx_bmm_ws(const cmpx_bmm_desc* desc, void* workspace, size_t workspace_bytes, void* stream) {
  int st = CMPX_OK;
  bmm_plan_impl(desc, &st);
  // an fp32 B stored MN-major is served through the workspace (launch_bmm_x3 decides)
  const bool f32_mn = st == CMPX_ERR_MISALIGNED && desc->dtype == CMPX_F32 &&
                      bmm_x3_workspace_bytes(desc) > 0 && workspace_bytes >= bmm_x3_workspace_bytes(desc);
  if (st != CMPX_OK && !f32_mn) return st;
  if (desc->batch == 0 || desc->m == 0 || desc->n == 0) return CMPX_OK;
  LaunchCtx ctx;
  st = device_ctx(&ctx, static_cast<cudaStream_t>(stream));
  if (st != CMPX_OK) return st;
  if (desc->dtype == CMPX_F32) return launch_bmm_x3(desc, ctx, workspace, workspace_bytes);
  return launch_bmm_sm100(desc, ctx);
}

size_t cmpx_linear_workspace_size(const cmpx_linear_desc* desc) {
  if (!desc || desc->dtype != CMPX_F32) return 0;
  return linear_x3_workspace_bytes(desc);
}

int cmpx_linear_ws(const cmpx_linear_desc* desc, void* workspace, size_t workspace_bytes, void* stream) {
  int st = CMPX_OK;
  linear_plan_impl(desc, &st);
  if (st != CMPX_OK) return st;
  if (desc->m == 0) return CMPX_OK;
  LaunchCtx ctx;
  st = device_ctx(&ctx, static_cast<cudaStream_t>(stream));
  if (st != CMPX_OK) return st;
  if (desc->dtype == CMPX_F32) return launch_linear_x3(desc, ctx, workspace, workspace_bytes);
  return launch_linear_sm100(desc, ctx);
}

int cmpx_bmm_small(const cmpx_bmm_desc* desc, void* stream) {
  int st = CMPX_OK;
  bmm_small_plan(desc, &st);
  if (st != CMPX_OK) return st;
  if (desc->batch == 0 || desc->m == 0 || desc->n == 0) return CMPX_OK;
  LaunchCtx ctx;
  st = device_ctx(&ctx, static_cast<cudaStream_t>(stream));
  if (st != CMPX_OK) return st;
  return launch_bmm_small(desc, ctx);
}

int cmpx_bmm_small_plan(const cmpx_bmm_desc* desc, char* buf, size_t buf_len) {
  int st = CMPX_OK;
  const char* name = bmm_small_plan(desc, &st);
  copy_name(st == CMPX_OK ? name : "none", buf, buf_len);
  return st;
}

int cmpx_softmax_rows(const cmpx_softmax_desc* desc, void* stream) {
  int st = CMPX_OK;
  softmax_rows_plan(desc, &st);
  if (st != CMPX_OK) return st;
  if (desc->rows == 0) return CMPX_OK;
  LaunchCtx ctx;
  st = device_ctx(&ctx, static_cast<cudaStream_t>(stream));
  if (st != CMPX_OK) return st;
  return launch_softmax_rows(desc, ctx);
}

int cmpx_bmm_rowstats(const cmpx_bmm_desc* desc, float* stats, void* stream) {
  int st = CMPX_OK;
  bmm_rowstats_plan(desc, stats, &st);
  if (st != CMPX_OK) return st;
  if (desc->batch == 0 || desc->m == 0 || desc->n == 0) return CMPX_OK;
  LaunchCtx ctx;
  st = device_ctx(&ctx, static_cast<cudaStream_t>(stream));
  if (st != CMPX_OK) return st;
  return launch_bmm_rowstats(desc, stats, ctx);
}

int cmpx_bmm_rowstats_plan(const cmpx_bmm_desc* desc, const float* stats, char* buf, size_t buf_len) {
  int st = CMPX_OK;
  const char* name = bmm_rowstats_plan(desc, stats, &st);
  copy_name(st == CMPX_OK ? name : "none", buf, buf_len);
  return st;
}

int cmpx_softmax_product(const cmpx_bmm_desc* desc, const float* stats, void* y, void* stream) {
  int st = CMPX_OK;
  softmax_product_plan(desc, stats, y, &st);
  if (st != CMPX_OK) return st;
  if (desc->batch == 0 || desc->m == 0) return CMPX_OK;
  LaunchCtx ctx;
  st = device_ctx(&ctx, static_cast<cudaStream_t>(stream));
  if (st != CMPX_OK) return st;
  return launch_softmax_product(desc, stats, y, ctx);
}

int cmpx_softmax_product_plan(const cmpx_bmm_desc* desc, const float* stats, const void* y, char* buf,
                              size_t buf_len) {
  int st = CMPX_OK;
  const char* name = softmax_product_plan(desc, stats, y, &st);
  copy_name(st == CMPX_OK ? name : "none", buf, buf_len);
  return st;
}

int cmpx_device_status(unsigned int* flags) {
  if (!flags) return CMPX_ERR_INVALID_ARGUMENT;
  LaunchCtx ctx;
  const int st = device_ctx(&ctx, nullptr);
  if (st != CMPX_OK) return st;
  if (cudaDeviceSynchronize() != cudaSuccess) return CMPX_ERR_DEVICE;
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_dev_flags, sizeof(v)) != cudaSuccess) return CMPX_ERR_DEVICE;
  const unsigned int zero = 0;
  if (cudaMemcpyToSymbol(g_dev_flags, &zero, sizeof(zero)) != cudaSuccess) return CMPX_ERR_DEVICE;
  *flags = v;
  return CMPX_OK;
}

int cmpx_selftest_wait_timeout(uint64_t timeout_ns, void* stream) {
  LaunchCtx ctx;
  const int st = device_ctx(&ctx, static_cast<cudaStream_t>(stream));
  if (st != CMPX_OK) return st;
  if (timeout_ns == 0 || timeout_ns > 10ull * 1000000000ull) return CMPX_ERR_INVALID_ARGUMENT;
  return launch_wait_selftest(timeout_ns, ctx);
}

}  // extern "C"
