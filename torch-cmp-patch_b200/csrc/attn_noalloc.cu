// attn_noalloc.cu -- an attention entry point for callers that cannot allocate device memory.
//
// cmpx_attn_fwd needs a small device workspace (the work counters of the persistent 16-bit
// kernel), and its callers hand one in.  Some callers have no way to get one at the moment of the
// call: a serving process whose memory pool owns the whole device and forbids further cudaMalloc,
// code that runs inside an allocator's own callback, or a real-time / certified stack that only
// allocates at start-up (cudaMalloc may also synchronise the device, which such callers cannot
// afford).  cmpx_attn_fwd_noalloc serves them: it uses a fixed scratch array that lives in the
// library's own device memory and allocates nothing per call.
//
// The scratch array below is a file-scope __device__ variable: every GPU that loads this library
// holds its 256 bytes until the process exits.  In host code its name is only a stand-in for the
// device object, so the host never passes it to a kernel directly: on the first call on each
// device (with that device current) cudaGetSymbolAddress turns it into a device address, which
// every later call on that device reuses.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "cmpx_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 256;  // the most scratch one call may use
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct ScratchSlot {
  std::once_flag once;
  cudaError_t status = cudaErrorUnknown;
  void* ptr = nullptr;
};
ScratchSlot g_scratch[kMaxDevices];

// Device address of the scratch array on the current device (resolved once per device).
void* scratch_on_current_device(int* status) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *status = CMPX_ERR_DEVICE;
    return nullptr;
  }
  ScratchSlot& slot = g_scratch[dev];
  std::call_once(slot.once, [&] {
    void* p = nullptr;
    slot.status = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (slot.status == cudaSuccess) slot.ptr = p;
  });
  if (slot.status != cudaSuccess || !slot.ptr) {
    cudaGetLastError();
    *status = CMPX_ERR_DEVICE;
    return nullptr;
  }
  *status = CMPX_OK;
  return slot.ptr;
}

}  // namespace

extern "C" CMPX_API int cmpx_attn_fwd_noalloc(const cmpx_attn_desc* desc, void* stream) {
  if (!desc) return CMPX_ERR_INVALID_ARGUMENT;
  // The 16-bit kernels run with their minimum workspace (the work counters; no tail split).  A
  // boolean mask is packed to bits in the workspace, which the fixed scratch has no room for.
  const bool sixteen = desc->dtype == CMPX_F16 || desc->dtype == CMPX_BF16;
  if (sixteen && desc->mask) return CMPX_ERR_WORKSPACE;
  const size_t need = sixteen ? cmpx::kAttnWorkspaceMin : 0;
  if (need > kNoAllocScratchBytes) return CMPX_ERR_WORKSPACE;  // beyond the fixed scratch
  cmpx_attn_desc d = *desc;  // the caller's workspace fields are ignored
  d.workspace = nullptr;
  d.workspace_bytes = 0;
  const int plan_status = cmpx_attn_plan(&d, nullptr, 0);  // reject bad calls before any device work
  if (plan_status != CMPX_OK) return plan_status;
  if (need > 0) {
    int st = CMPX_OK;
    void* scratch = scratch_on_current_device(&st);
    if (st != CMPX_OK) return st;
    // The array keeps whatever the previous call left in it: clear the counters this call
    // relies on starting at zero (an enqueued memset, not an allocation).
    if (cudaMemsetAsync(scratch, 0, need, static_cast<cudaStream_t>(stream)) != cudaSuccess) {
      cudaGetLastError();
      return CMPX_ERR_LAUNCH;
    }
    d.workspace = scratch;
    d.workspace_bytes = kNoAllocScratchBytes;
  }
  return cmpx_attn_fwd(&d, stream);
}
