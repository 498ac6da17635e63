// attn_fwd_f32.cu -- routing of fp32 scaled-dot-product attention (fp32 inputs, fp32 accumulation).
//
// The accuracy contract for fp32 inputs is 1e-4 relative to stock fp32 SDPA, which rules out
// single-pass TF32 tensor-core products (10-bit mantissa).  Every fp32 call with head_dim <= 128
// (the reference kernel's own range, src/cuda/fp32_attention.cu:8 MAX_DIM) and 16-byte aligned
// operands runs the tensor-core 3xTF32 kernel (attn_tf32x3_sm100.cu; 64-key tiles for D <= 64,
// 32-key tiles for D <= 128), which replaces attention_fp32_strict_kernel
// (src/cuda/fp32_attention.cu:35-198).  The binding copies operands that are not 16-byte aligned
// into padded buffers, so the remaining declines are head_dim > 128.
#include <cuda_runtime.h>


#include "cmpx_internal.h"

namespace cmpx {

const char* attn_f32_plan(const cmpx_attn_desc* d, int* status) {
  *status = CMPX_OK;
  if (d->dtype != CMPX_F32) {
    *status = CMPX_ERR_UNSUPPORTED_DTYPE;
    return "none";
  }
  if (d->head_dim < 1 || d->head_dim > 128) {
    *status = CMPX_ERR_UNSUPPORTED_SHAPE;
    return "none";
  }
  if (d->len_q > (int64_t)64 * 65535 || d->batch * d->heads > (1ll << 31) - 1) {
    *status = CMPX_ERR_UNSUPPORTED_SHAPE;
    return "none";
  }
  if (attn_tf32x3_eligible(d)) {
    // "+tail-split": the schedule a call given cmpx_attn_workspace_size() bytes runs
    static const char* const names[2][2][3] = {
        {{"attn_tf32x3_sm100<D64,128q,64kv,persistent>", "attn_tf32x3_sm100<D64,128q,64kv,persistent+mask>",
          "attn_tf32x3_sm100<D64,128q,64kv,persistent+addmask>"},
         {"attn_tf32x3_sm100<D128,128q,32kv,persistent>", "attn_tf32x3_sm100<D128,128q,32kv,persistent+mask>",
          "attn_tf32x3_sm100<D128,128q,32kv,persistent+addmask>"}},
        {{"attn_tf32x3_sm100<D64,128q,64kv,persistent+tail-split>",
          "attn_tf32x3_sm100<D64,128q,64kv,persistent+mask+tail-split>",
          "attn_tf32x3_sm100<D64,128q,64kv,persistent+addmask+tail-split>"},
         {"attn_tf32x3_sm100<D128,128q,32kv,persistent+tail-split>",
          "attn_tf32x3_sm100<D128,128q,32kv,persistent+mask+tail-split>",
          "attn_tf32x3_sm100<D128,128q,32kv,persistent+addmask+tail-split>"}}};
    const int mk = !d->mask ? 0 : d->mask_kind == CMPX_MASK_BOOL ? 1 : 2;
    const int split = attn_tf32x3_tail_split(d, current_num_sms()) ? 1 : 0;
    return names[split][d->head_dim <= 64 ? 0 : 1][mk];
  }
  // Operands the 3xTF32 kernel cannot read with TMA (strides or pointers not 16-byte aligned; the
  // ctypes binding copies such inputs to padded buffers before it gets here).
  *status = CMPX_ERR_MISALIGNED;
  return "none";
}

int launch_attn_f32(const cmpx_attn_desc* d, const LaunchCtx& ctx) {
  int st = CMPX_OK;
  attn_f32_plan(d, &st);
  if (st != CMPX_OK) return st;
  if (d->len_q == 0) return CMPX_OK;
  return launch_attn_tf32x3(d, ctx);
}

}  // namespace cmpx
