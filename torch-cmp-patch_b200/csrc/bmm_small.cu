// bmm_small.cu -- batched products of many tiny matrices (fp32 / fp16 / bf16, B200 sm_100a).
//
// The reference routes a 3-D bmm / matmul whose per-item product is small (M*K*N <= 32768 by
// default: FEM element blocks, tiny heads) away from its tiled GEMM, to an eager broadcast multiply
// and sum over a [batch, M, K, N] intermediate (cmpext3/__init__.py:440-464), because a tiled GEMM
// wastes almost all of its tile on such shapes.  This kernel computes the same products directly,
// with no intermediate tensor: every output element is one dot product of length K in fp32
// (products exact in fp32, one rounding to the output type at the end), reading A and B in place
// through their strides (transposed and otherwise strided views need no copy).
//
//   * K < 128: one thread per output element.  Consecutive threads take consecutive columns of a
//     row, so the B loads of a warp are contiguous along N and the A loads are shared by the threads
//     of one row (L1 hits).
//   * K >= 128 (then M*N <= 256 per item): one warp per output element, the lanes striding along K
//     (contiguous A loads), then a shuffle reduction.
//
// The work is a few FLOP per byte at these sizes, so both forms are bound by the loads; grids are
// grid-stride loops sized to the SM count.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "cmpx_internal.h"

namespace cmpx {
namespace {

constexpr int kWarpK = 128;  // K from which one warp (rather than one thread) computes an element

struct SmallParams {
  const void* a;
  const void* b;
  void* c;
  int64_t m, n, k, total;  // total = batch * m * n output elements
  int64_t as0, as1, as2, bs0, bs1, bs2, cs0, cs1, cs2;
};

template <int DT>
__device__ __forceinline__ float ld(const void* base, int64_t i) {
  if constexpr (DT == CMPX_F32) return __ldg(static_cast<const float*>(base) + i);
  if constexpr (DT == CMPX_F16) return __half2float(__ldg(static_cast<const __half*>(base) + i));
  return __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(base) + i));
}

template <int DT>
__device__ __forceinline__ void st(void* base, int64_t i, float v) {
  if constexpr (DT == CMPX_F32) static_cast<float*>(base)[i] = v;
  else if constexpr (DT == CMPX_F16) static_cast<__half*>(base)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
}

// Output element o of the flattened [batch, m, n] result -> (item, row, column).
__device__ __forceinline__ void split(const SmallParams& p, int64_t o, int64_t& item, int64_t& r, int64_t& c) {
  const int64_t mn = p.m * p.n;
  item = o / mn;
  const int64_t rem = o - item * mn;
  r = rem / p.n;
  c = rem - r * p.n;
}

template <int DT>
__global__ void __launch_bounds__(256) bmm_small_thread_kernel(const SmallParams p) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t o = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < p.total; o += stride) {
    int64_t item, r, c;
    split(p, o, item, r, c);
    const int64_t a0 = item * p.as0 + r * p.as1, b0 = item * p.bs0 + c * p.bs2;
    float acc0 = 0.f, acc1 = 0.f;
    int64_t kk = 0;
    for (; kk + 2 <= p.k; kk += 2) {
      acc0 = fmaf(ld<DT>(p.a, a0 + kk * p.as2), ld<DT>(p.b, b0 + kk * p.bs1), acc0);
      acc1 = fmaf(ld<DT>(p.a, a0 + (kk + 1) * p.as2), ld<DT>(p.b, b0 + (kk + 1) * p.bs1), acc1);
    }
    if (kk < p.k) acc0 = fmaf(ld<DT>(p.a, a0 + kk * p.as2), ld<DT>(p.b, b0 + kk * p.bs1), acc0);
    st<DT>(p.c, item * p.cs0 + r * p.cs1 + c * p.cs2, acc0 + acc1);
  }
}

template <int DT>
__global__ void __launch_bounds__(256) bmm_small_warp_kernel(const SmallParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t o = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; o < p.total; o += nwarps) {
    int64_t item, r, c;
    split(p, o, item, r, c);
    const int64_t a0 = item * p.as0 + r * p.as1, b0 = item * p.bs0 + c * p.bs2;
    float acc = 0.f;
    for (int64_t kk = lane; kk < p.k; kk += 32) acc = fmaf(ld<DT>(p.a, a0 + kk * p.as2), ld<DT>(p.b, b0 + kk * p.bs1), acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) st<DT>(p.c, item * p.cs0 + r * p.cs1 + c * p.cs2, acc);
  }
}

template <int DT>
int launch_dt(const SmallParams& p, const LaunchCtx& ctx) {
  const int sms = std::max(1, ctx.num_sms);
  if (p.k >= kWarpK) {
    const int64_t blocks = std::min<int64_t>((p.total * 32 + 255) / 256, static_cast<int64_t>(sms) * 16);
    bmm_small_warp_kernel<DT><<<static_cast<int>(std::max<int64_t>(1, blocks)), 256, 0, ctx.stream>>>(p);
  } else {
    const int64_t blocks = std::min<int64_t>((p.total + 255) / 256, static_cast<int64_t>(sms) * 16);
    bmm_small_thread_kernel<DT><<<static_cast<int>(std::max<int64_t>(1, blocks)), 256, 0, ctx.stream>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

}  // namespace

const char* bmm_small_plan(const cmpx_bmm_desc* d, int* status) {
  *status = CMPX_OK;
  if (!d || d->batch < 0 || d->m < 0 || d->n < 0 || d->k < 0) {
    *status = CMPX_ERR_INVALID_ARGUMENT;
    return "none";
  }
  if (d->dtype != CMPX_F32 && d->dtype != CMPX_F16 && d->dtype != CMPX_BF16) {
    *status = CMPX_ERR_UNSUPPORTED_DTYPE;
    return "none";
  }
  const bool empty = d->batch == 0 || d->m == 0 || d->n == 0;
  if (!empty && (!d->c || (d->k > 0 && (!d->a || !d->b)))) {
    *status = CMPX_ERR_INVALID_ARGUMENT;
    return "none";
  }
  for (int i = 0; i < 3; ++i)
    if (d->a_stride[i] < 0 || d->b_stride[i] < 0 || d->c_stride[i] < 0) {
      *status = CMPX_ERR_INVALID_ARGUMENT;
      return "none";
    }
  static const char* const names[3][2] = {{"bmm_small<f32,thread-per-element>", "bmm_small<f32,warp-per-element>"},
                                          {"bmm_small<f16,thread-per-element>", "bmm_small<f16,warp-per-element>"},
                                          {"bmm_small<bf16,thread-per-element>", "bmm_small<bf16,warp-per-element>"}};
  return names[d->dtype][d->k >= kWarpK ? 1 : 0];
}

int launch_bmm_small(const cmpx_bmm_desc* d, const LaunchCtx& ctx) {
  SmallParams p;
  p.a = d->a;
  p.b = d->b;
  p.c = d->c;
  p.m = d->m;
  p.n = d->n;
  p.k = d->k;
  p.total = d->batch * d->m * d->n;
  p.as0 = d->a_stride[0];
  p.as1 = d->a_stride[1];
  p.as2 = d->a_stride[2];
  p.bs0 = d->b_stride[0];
  p.bs1 = d->b_stride[1];
  p.bs2 = d->b_stride[2];
  p.cs0 = d->c_stride[0];
  p.cs1 = d->c_stride[1];
  p.cs2 = d->c_stride[2];
  switch (d->dtype) {
    case CMPX_F32: return launch_dt<CMPX_F32>(p, ctx);
    case CMPX_F16: return launch_dt<CMPX_F16>(p, ctx);
    default: return launch_dt<CMPX_BF16>(p, ctx);
  }
}

}  // namespace cmpx
