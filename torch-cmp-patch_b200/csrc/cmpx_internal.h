// cmpx_internal.h -- host-side declarations shared by the C-ABI layer and the kernel files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/cmpx_b200.h"

namespace cmpx {

// Per-call launch context filled in by the C-ABI layer.
struct LaunchCtx {
  cudaStream_t stream;
  unsigned int* dev_flags;         // device status word of the current device
  unsigned long long timeout_ns;   // bound on every in-kernel wait
  int num_sms;
};

// Encodes a tiled TMA descriptor (driver entry point resolved at run time).
// dims/strides_bytes are innermost-first; strides_bytes has rank-1 entries.
bool encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle);

// ---- attention ----
// Tile-table lookups: return a static name and whether the kernel supports the call.
const char* fmha_sm100_plan(const cmpx_attn_desc* d, int* status);
int launch_fmha_sm100(const cmpx_attn_desc* d, const LaunchCtx& ctx);

const char* attn_f32_plan(const cmpx_attn_desc* d, int* status);
int launch_attn_f32(const cmpx_attn_desc* d, const LaunchCtx& ctx);

// ---- batched matmul ----
const char* bmm_sm100_plan(const cmpx_bmm_desc* d, int* status);
int launch_bmm_sm100(const cmpx_bmm_desc* d, const LaunchCtx& ctx);

const char* bmm_f32_plan(const cmpx_bmm_desc* d, int* status);
int launch_bmm_f32(const cmpx_bmm_desc* d, const LaunchCtx& ctx);

// ---- self test ----
int launch_wait_selftest(uint64_t timeout_ns, const LaunchCtx& ctx);

}  // namespace cmpx
