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
// every later call on that device reuses.  A lookup that fails is not kept, so the next call on
// that device looks the address up again.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>

#include "cmpx_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 256;  // the most scratch one call may use
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array, per device; null until a lookup on that device succeeded.
// A failed lookup (e.g. one made while the stream was being captured) is not remembered: the next
// call on that device tries again.
std::atomic<void*> g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mutex;

// Device address of the scratch array on the current device.
void* scratch_on_current_device(int* status) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    *status = CMPX_ERR_DEVICE;
    return nullptr;
  }
  void* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    p = g_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (!p) {
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        *status = CMPX_ERR_DEVICE;
        return nullptr;
      }
      g_scratch_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *status = CMPX_OK;
  return p;
}

}  // namespace

extern "C" CMPX_API int cmpx_attn_fwd_noalloc(const cmpx_attn_desc* desc, void* stream) {
  if (!desc) return CMPX_ERR_INVALID_ARGUMENT;
  cmpx_attn_desc d = *desc;  // the caller's workspace fields are ignored
  d.workspace = nullptr;
  d.workspace_bytes = 0;
  const int plan_status = cmpx_attn_plan(&d, nullptr, 0);  // reject bad calls before any device work
  if (plan_status != CMPX_OK) return plan_status;
  // The 16-bit kernels run with their minimum workspace: the work counters (no tail split), plus a
  // boolean mask packed to bits, for which the fixed scratch has no room.  fp32 needs none.
  const bool sixteen = d.dtype == CMPX_F16 || d.dtype == CMPX_BF16;
  const size_t need = sixteen ? cmpx::fmha_workspace_min(&d) : 0;
  if (need > kNoAllocScratchBytes) return CMPX_ERR_WORKSPACE;  // beyond the fixed scratch
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
