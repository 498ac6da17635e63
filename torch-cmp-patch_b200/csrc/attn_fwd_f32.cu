// attn_fwd_f32.cu -- routing of fp32 scaled-dot-product attention (fp32 inputs, fp32 accumulation).
//
// The accuracy contract for fp32 inputs is 1e-4 relative to stock fp32 SDPA, which rules out
// single-pass TF32 tensor-core products (10-bit mantissa).  Calls with head_dim <= 64 and 16-byte
// aligned operands run the tensor-core 3xTF32 kernel (attn_tf32x3_sm100.cu), which replaces
// attention_fp32_strict_kernel (src/cuda/fp32_attention.cu:35-198).  The other fp32 calls are not
// in the tile table: on B200 stock torch beats a CUDA-core fp32 kernel for them.
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
    if (!d->mask) return "attn_tf32x3_sm100<D64,128q,64kv,persistent>";
    return d->mask_kind == CMPX_MASK_BOOL ? "attn_tf32x3_sm100<D64,128q,64kv,persistent+mask>"
                                          : "attn_tf32x3_sm100<D64,128q,64kv,persistent+addmask>";
  }
  // Head dims above 64, or operands the 3xTF32 kernel cannot read with TMA: stock torch is faster
  // than a CUDA-core fp32 kernel on B200 (measured: 20 vs 47 TFLOP/s at D = 128), so these calls
  // are left to it -- what the reference's own runtime selection did for fp32 attention.
  *status = CMPX_ERR_UNSUPPORTED_SHAPE;
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
