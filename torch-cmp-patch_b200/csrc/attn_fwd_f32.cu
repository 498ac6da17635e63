// attn_fwd_f32.cu -- fp32 scaled-dot-product attention forward (fp32 inputs, fp32 accumulation).
//
// The accuracy contract for fp32 inputs is 1e-4 relative to stock fp32 SDPA, which rules out
// single-pass TF32 tensor-core products (10-bit mantissa).  This kernel keeps every product and
// sum in fp32 FMA on the CUDA cores.  It replaces attention_fp32_strict_kernel
// (src/cuda/fp32_attention.cu:35-198: one thread per query row, D-long dot products per key,
// register-spilling row buffers, reciprocal through fp16) with a tiled online-softmax kernel:
//
//   * a CTA owns 64 query rows of one (batch, head); 256 threads as a 16 x 16 grid, thread
//     (ty, tx) computes the 4 x 4 block of scores rows ty*4.., keys tx*4.. of each 64-key tile;
//   * Q^T and K^T tiles sit in shared memory head-dim-major so each step of the dot product is
//     two float4 loads and 16 FMAs;
//   * row max / row sum across the 16 threads of a row with warp shuffles; running m, l per row;
//   * P goes through shared memory (key-major) and O += P V accumulates 4 rows x 4*NC columns
//     per thread; O is rescaled by exp2(m_old - m_new) whenever the row max moves;
//   * causal masking (top-left aligned) and the ragged last key tile are masked to -inf.
// Supports any head_dim <= 128 and arbitrary batch/head/row strides (contiguous head dim).  Calls
// with head_dim <= 64 and 16-byte aligned operands go to the tensor-core 3xTF32 kernel instead
// (attn_tf32x3_sm100.cu); this kernel serves the rest.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "cmpx_internal.h"

namespace cmpx {

struct F32AttnParams {
  const float* q;
  const float* k;
  const float* v;
  float* o;
  long long qs[3], ks[3], vs[3], os[3];
  int heads, len_q, len_k, head_dim, causal;
  int group;  // query heads per key/value head (grouped-query attention)
  float scale_log2;
};

__device__ __forceinline__ float f32_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int DP>
struct F32Cfg {
  static constexpr int BQ = 64, BK = 64;
  static constexpr int LDT = 64 + 4;       // row pitch of the transposed Q/K tiles
  static constexpr int LDV = DP + 4;       // row pitch of the V tile
  static constexpr int LDP = 64 + 4;       // row pitch of P^T
  static constexpr int NC = DP / 64;       // float4 column groups of O per thread
  static constexpr int SMEM_FLOATS = DP * LDT /*Q^T*/ + DP * LDT /*K^T*/ + BK * LDV /*V*/ + BK * LDP /*P^T*/;
  static constexpr int SMEM_BYTES = SMEM_FLOATS * 4;
};

template <int DP>
__global__ void __launch_bounds__(256) attn_fwd_f32_kernel(const F32AttnParams p) {
  using C = F32Cfg<DP>;
  extern __shared__ float4 smem_f4[];
  float* smem = reinterpret_cast<float*>(smem_f4);
  float* sQt = smem;                        // [DP][LDT]  Q^T (scaled by scale*log2e)
  float* sKt = sQt + DP * C::LDT;           // [DP][LDT]  K^T
  float* sV = sKt + DP * C::LDT;            // [BK][LDV]
  float* sPt = sV + C::BK * C::LDV;         // [BK][LDP]  P^T

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int bh = blockIdx.x;
  const int b = bh / p.heads, h = bh - (bh / p.heads) * p.heads;
  const int q0 = (gridDim.y - 1 - blockIdx.y) * C::BQ;  // later (heavier causal) rows first
  const int D = p.head_dim;

  const float* qb = p.q + b * p.qs[0] + h * p.qs[1];
  const float* kb = p.k + b * p.ks[0] + (h / p.group) * p.ks[1];
  const float* vb = p.v + b * p.vs[0] + (h / p.group) * p.vs[1];
  float* ob = p.o + b * p.os[0] + h * p.os[1];

  // Q tile, transposed, pre-multiplied by scale*log2(e) so scores come out in the exp2 domain.
  for (int idx = tid; idx < C::BQ * DP; idx += 256) {
    const int r = idx / DP, d = idx - (idx / DP) * DP;
    float x = 0.f;
    if (q0 + r < p.len_q && d < D) x = qb[(long long)(q0 + r) * p.qs[2] + d] * p.scale_log2;
    sQt[d * C::LDT + r] = x;
  }

  float m_run[4], l_run[4], acc[4][4 * C::NC];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 4 * C::NC; ++c) acc[i][c] = 0.f;
  }

  const int kv_end = p.causal ? min(p.len_k, q0 + C::BQ) : p.len_k;
  for (int kv0 = 0; kv0 < kv_end; kv0 += C::BK) {
    __syncthreads();  // previous tile's readers are done with sKt / sV / sPt
    for (int idx = tid; idx < C::BK * DP; idx += 256) {
      const int r = idx / DP, d = idx - (idx / DP) * DP;
      float kx = 0.f, vx = 0.f;
      if (kv0 + r < p.len_k && d < D) {
        kx = kb[(long long)(kv0 + r) * p.ks[2] + d];
        vx = vb[(long long)(kv0 + r) * p.vs[2] + d];
      }
      sKt[d * C::LDT + r] = kx;
      sV[r * C::LDV + d] = vx;
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) s[i][jj] = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; ++d) {
      const float4 qv = *reinterpret_cast<const float4*>(&sQt[d * C::LDT + ty * 4]);
      const float4 kv = *reinterpret_cast<const float4*>(&sKt[d * C::LDT + tx * 4]);
      const float qa[4] = {qv.x, qv.y, qv.z, qv.w};
      const float ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) s[i][jj] = fmaf(qa[i], ka[jj], s[i][jj]);
    }

    float alpha[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qrow = q0 + ty * 4 + i;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int kv = kv0 + tx * 4 + jj;
        if (kv >= p.len_k || (p.causal && kv > qrow)) s[i][jj] = -INFINITY;
      }
      float mx = fmaxf(fmaxf(s[i][0], s[i][1]), fmaxf(s[i][2], s[i][3]));
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_run[i], mx);
      const float mb = (m_new == -INFINITY) ? 0.f : m_new;
      alpha[i] = f32_ex2(m_run[i] - mb);
      m_run[i] = m_new;
      float rs = 0.f;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        s[i][jj] = f32_ex2(s[i][jj] - mb);
        rs += s[i][jj];
      }
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l_run[i] = l_run[i] * alpha[i] + rs;
#pragma unroll
      for (int c = 0; c < 4 * C::NC; ++c) acc[i][c] *= alpha[i];
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj)
      *reinterpret_cast<float4*>(&sPt[(tx * 4 + jj) * C::LDP + ty * 4]) =
          make_float4(s[0][jj], s[1][jj], s[2][jj], s[3][jj]);
    __syncthreads();

    const int kmax = min(C::BK, kv_end - kv0);
#pragma unroll 4
    for (int kk = 0; kk < kmax; ++kk) {
      const float4 pv = *reinterpret_cast<const float4*>(&sPt[kk * C::LDP + ty * 4]);
      const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
      for (int c = 0; c < C::NC; ++c) {
        const float4 vv = *reinterpret_cast<const float4*>(&sV[kk * C::LDV + c * 64 + tx * 4]);
        const float va[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[i][c * 4 + e] = fmaf(pa[i], va[e], acc[i][c * 4 + e]);
      }
    }
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qrow = q0 + ty * 4 + i;
    if (qrow >= p.len_q) continue;
    const float inv = 1.f / l_run[i];
    float* orow = ob + (long long)qrow * p.os[2];
#pragma unroll
    for (int c = 0; c < C::NC; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = c * 64 + tx * 4 + e;
        if (d < D) orow[d] = acc[i][c * 4 + e] * inv;
      }
  }
}

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
  if (attn_tf32x3_eligible(d)) return "attn_tf32x3_sm100<D64,128q,64kv,persistent>";
  return d->head_dim <= 64 ? "attn_f32_simt<D64,64q,64kv>" : "attn_f32_simt<D128,64q,64kv>";
}

namespace {
template <int DP>
int launch_f32_typed(const cmpx_attn_desc* d, const LaunchCtx& ctx) {
  using C = F32Cfg<DP>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(reinterpret_cast<const void*>(&attn_fwd_f32_kernel<DP>),
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return CMPX_ERR_LAUNCH;
  F32AttnParams p;
  p.q = static_cast<const float*>(d->q);
  p.k = static_cast<const float*>(d->k);
  p.v = static_cast<const float*>(d->v);
  p.o = static_cast<float*>(d->o);
  for (int i = 0; i < 3; ++i) {
    p.qs[i] = d->q_stride[i];
    p.ks[i] = d->k_stride[i];
    p.vs[i] = d->v_stride[i];
    p.os[i] = d->o_stride[i];
  }
  p.heads = static_cast<int>(d->heads);
  p.group = attn_group(d);
  p.len_q = static_cast<int>(d->len_q);
  p.len_k = static_cast<int>(d->len_k);
  p.head_dim = static_cast<int>(d->head_dim);
  p.causal = d->causal ? 1 : 0;
  p.scale_log2 = static_cast<float>(d->scale * 1.4426950408889634);
  dim3 grid(static_cast<unsigned>(d->batch * d->heads),
            static_cast<unsigned>((d->len_q + C::BQ - 1) / C::BQ));
  attn_fwd_f32_kernel<DP><<<grid, 256, C::SMEM_BYTES, ctx.stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}
}  // namespace

int launch_attn_f32(const cmpx_attn_desc* d, const LaunchCtx& ctx) {
  int st = CMPX_OK;
  attn_f32_plan(d, &st);
  if (st != CMPX_OK) return st;
  if (d->len_q == 0) return CMPX_OK;
  if (attn_tf32x3_eligible(d)) return launch_attn_tf32x3(d, ctx);
  return d->head_dim <= 64 ? launch_f32_typed<64>(d, ctx) : launch_f32_typed<128>(d, ctx);
}

}  // namespace cmpx
