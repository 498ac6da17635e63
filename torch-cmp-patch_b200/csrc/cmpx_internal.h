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

// 4-D TMA map over a [B, H, L, D] 16-bit tensor with element strides st = {b, h, l} (D
// contiguous): box = 64 head-dim elements (128 bytes, 128-byte swizzle) x box_rows rows.
bool make_bhsd_map(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, int64_t D, int64_t L,
                   int64_t H, int64_t B, const int64_t* st, uint32_t box_rows);

// ---- attention ----
// Key/value heads of a call (heads_kv = 0 means one per query head) and the query-head group size.
inline int64_t attn_heads_kv(const cmpx_attn_desc* d) { return d->heads_kv > 0 ? d->heads_kv : d->heads; }
inline int attn_group(const cmpx_attn_desc* d) {
  const int64_t hk = attn_heads_kv(d);
  return hk > 0 ? static_cast<int>(d->heads / hk) : 1;
}

// SM count of the current device (148, a B200's, when no device can be queried).
int current_num_sms();

// Smallest workspace the 16-bit attention kernels accept: their two work counters.
constexpr size_t kAttnWorkspaceMin = 256;

// Tile-table lookups: return a static name and whether the kernel supports the call.
const char* fmha_sm100_plan(const cmpx_attn_desc* d, int* status);
// Workspace for the fastest schedule of a 16-bit call on num_sms SMs (>= kAttnWorkspaceMin: the
// tail split's partial results on top of the counters; a workspace of at least kAttnWorkspaceMin
// but below this runs unsplit).
size_t fmha_workspace_bytes(const cmpx_attn_desc* d, int num_sms);
// Smallest workspace a 16-bit call accepts: the work counters, plus the packed mask if it has one.
size_t fmha_workspace_min(const cmpx_attn_desc* d);
int launch_fmha_sm100(const cmpx_attn_desc* d, const LaunchCtx& ctx);
// Short key sequences (non-causal, 1 <= Lk <= 128): one key tile, Q tiles streamed.
bool fmha_short_eligible(const cmpx_attn_desc* d);
const char* fmha_short_name(const cmpx_attn_desc* d);
int launch_fmha_short(const cmpx_attn_desc* d, const LaunchCtx& ctx);

const char* attn_f32_plan(const cmpx_attn_desc* d, int* status);
int launch_attn_f32(const cmpx_attn_desc* d, const LaunchCtx& ctx);
// fp32 on the tensor cores (3xTF32), head_dim <= 64 with 16-byte aligned pointers / strides.
bool attn_tf32x3_eligible(const cmpx_attn_desc* d);
int launch_attn_tf32x3(const cmpx_attn_desc* d, const LaunchCtx& ctx);
// workspace of an fp32 call's tail split (0: the call runs without one)
size_t attn_tf32x3_workspace_bytes(const cmpx_attn_desc* d, int num_sms);
bool attn_tf32x3_tail_split(const cmpx_attn_desc* d, int num_sms);

// ---- batched matmul ----
const char* bmm_sm100_plan(const cmpx_bmm_desc* d, int* status);
int launch_bmm_sm100(const cmpx_bmm_desc* d, const LaunchCtx& ctx);
// fp32 on the tensor cores (3xTF32), K-major operands.
const char* bmm_x3_plan(const cmpx_bmm_desc* d, int* status);
// ws: the split-operand workspace (bmm_x3_workspace_bytes); null or smaller: the converter path.
int launch_bmm_x3(const cmpx_bmm_desc* d, const LaunchCtx& ctx, void* ws = nullptr, size_t ws_bytes = 0);
size_t bmm_x3_workspace_bytes(const cmpx_bmm_desc* d);
// Many tiny products (the reference's M*K*N <= 32768 route): one thread or warp per output element.
const char* bmm_small_plan(const cmpx_bmm_desc* d, int* status);
int launch_bmm_small(const cmpx_bmm_desc* d, const LaunchCtx& ctx);
// The GEMM of a linear layer: x [m, k] times W^T with W [n, k] read in place as a K-major B.
cmpx_bmm_desc linear_as_bmm(const cmpx_linear_desc* d);


// ---- linear (the bmm GEMM with batch 1, W read as a K-major B, bias in the epilogue) ----
const char* linear_sm100_plan(const cmpx_linear_desc* d, int* status);
int launch_linear_sm100(const cmpx_linear_desc* d, const LaunchCtx& ctx);
const char* linear_x3_plan(const cmpx_linear_desc* d, int* status);
int launch_linear_x3(const cmpx_linear_desc* d, const LaunchCtx& ctx, void* ws = nullptr, size_t ws_bytes = 0);
size_t linear_x3_workspace_bytes(const cmpx_linear_desc* d);

// ---- row softmax (einsum-attention chain) ----
const char* softmax_rows_plan(const cmpx_softmax_desc* d, int* status);
int launch_softmax_rows(const cmpx_softmax_desc* d, const LaunchCtx& ctx);
// the 16-bit product with per-row, per-64-column (max, sum) statistics (rowstats.cuh)
const char* bmm_rowstats_plan(const cmpx_bmm_desc* d, const void* stats, int* status);
int launch_bmm_rowstats(const cmpx_bmm_desc* d, float* stats, const LaunchCtx& ctx);
// softmax over the last dimension of a 16-bit product A B, recomputed from A and B (K-major,
// k <= 128) and the product's row statistics
const char* softmax_product_plan(const cmpx_bmm_desc* d, const void* stats, const void* y, int* status);
int launch_softmax_product(const cmpx_bmm_desc* d, const float* stats, void* y, const LaunchCtx& ctx);

// ---- self test ----
int launch_wait_selftest(uint64_t timeout_ns, const LaunchCtx& ctx);

}  // namespace cmpx
