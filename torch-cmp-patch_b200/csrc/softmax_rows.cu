// softmax_rows.cu -- row softmax over the last dimension (fp16 / bf16 / fp32), B200 sm_100a.
//
// y[r, :] = exp(x[r, :] - max) / sum(exp(x[r, :] - max)), computed in fp32 and rounded once to
// the output dtype -- the value torch.softmax(x, dim=-1) returns.  Serves the einsum-attention
// chain (scores einsum -> softmax -> values einsum, cmpext3/einsum_ops.py:69-121 of the
// reference), whose softmax over the [.., L, L] score tensor is a pure HBM stream: read the row,
// write the row.
//
//   * one warp per row (grid-stride over rows), 16-byte vector loads: a row of up to 2048 16-bit
//     (1024 fp32) values is held in registers, so it is read from HBM once; its exponentials stay
//     in registers between the sum and the store;
//   * longer rows, or rows whose pointers / strides are not 16-byte aligned: two passes with
//     scalar loads (online max and sum, then exp and store), reading the row twice.
// Exponentials: ex2.approx of (x - max) * log2(e) (fp32, relative error ~2^-22).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>

#include "cmpx_internal.h"
#include "cmpx_ptx.cuh"

namespace cmpx {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

template <int DT>
__device__ __forceinline__ float to_f32(uint32_t bits16) {
  if (DT == CMPX_BF16) return __uint_as_float(bits16 << 16);
  __half_raw hr;
  hr.x = static_cast<unsigned short>(bits16);
  return __half2float(__half(hr));
}

// 16-byte chunk -> EPC floats
template <int DT>
__device__ __forceinline__ void unpack(const uint4& v, float* f) {
  if (DT == CMPX_F32) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  } else {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = to_f32<DT>(w[i] & 0xFFFFu);
      f[2 * i + 1] = to_f32<DT>(w[i] >> 16);
    }
  }
}

template <int DT>
__device__ __forceinline__ uint4 pack(const float* f) {
  uint4 v;
  if (DT == CMPX_F32) {
    v.x = __float_as_uint(f[0]);
    v.y = __float_as_uint(f[1]);
    v.z = __float_as_uint(f[2]);
    v.w = __float_as_uint(f[3]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = DT == CMPX_BF16 ? pack_bf16x2(f[2 * i], f[2 * i + 1]) : pack_f16x2(f[2 * i], f[2 * i + 1]);
    v = make_uint4(w[0], w[1], w[2], w[3]);
  }
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Register-resident rows: CHUNKS 16-byte chunks per lane (row length <= CHUNKS * 32 * EPC).
template <int DT, int CHUNKS>
__global__ void __launch_bounds__(256) softmax_rows_reg_kernel(const uint8_t* __restrict__ x,
                                                               uint8_t* __restrict__ y, int64_t rows,
                                                               int cols, int64_t xs_bytes,
                                                               int64_t ys_bytes) {
  constexpr int EPC = DT == CMPX_F32 ? 4 : 8;  // elements per 16-byte chunk
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int nchunks = cols / EPC;
  for (int64_t r = warp0; r < rows; r += nwarps) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + r * xs_bytes);
    uint4* yr = reinterpret_cast<uint4*>(y + r * ys_bytes);
    uint4 v[CHUNKS];
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      const int idx = c * 32 + lane;
      if (idx < nchunks) v[c] = __ldg(xr + idx);
    }
    float e[CHUNKS * EPC];
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      if (c * 32 + lane < nchunks) {
        unpack<DT>(v[c], e + c * EPC);
#pragma unroll
        for (int i = 0; i < EPC; ++i) m = fmaxf(m, e[c * EPC + i]);
      }
    }
    m = warp_max(m);
    // A row of -inf keeps m = -inf: the result is NaN, as torch's is.  The exponent is the exact
    // difference x - m times log2(e), not fma(x, log2e, -m*log2e): the rounded product m*log2e
    // would carry an error of |m| * 2^-24 into every exponent of a row with large scores.
    float l = 0.f;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      if (c * 32 + lane < nchunks) {
#pragma unroll
        for (int i = 0; i < EPC; ++i) {
          e[c * EPC + i] = ex2_approx((e[c * EPC + i] - m) * kLog2e);
          l += e[c * EPC + i];
        }
      }
    }
    l = warp_sum(l);
    const float inv = 1.f / l;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      const int idx = c * 32 + lane;
      if (idx < nchunks) {
        float o[EPC];
#pragma unroll
        for (int i = 0; i < EPC; ++i) o[i] = e[c * EPC + i] * inv;
        yr[idx] = pack<DT>(o);
      }
    }
  }
}

template <int DT>
__device__ __forceinline__ float load_elt(const uint8_t* p, int64_t i) {
  if (DT == CMPX_F32) return reinterpret_cast<const float*>(p)[i];
  return to_f32<DT>(reinterpret_cast<const unsigned short*>(p)[i]);
}

template <int DT>
__device__ __forceinline__ void store_elt(uint8_t* p, int64_t i, float v) {
  if (DT == CMPX_F32) {
    reinterpret_cast<float*>(p)[i] = v;
  } else if (DT == CMPX_BF16) {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  }
}

// Any row length / alignment: online max + sum, then exp and store (the row is read twice).
template <int DT>
__global__ void __launch_bounds__(256) softmax_rows_stream_kernel(const uint8_t* __restrict__ x,
                                                                  uint8_t* __restrict__ y, int64_t rows,
                                                                  int64_t cols, int64_t xs_bytes,
                                                                  int64_t ys_bytes) {
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = warp0; r < rows; r += nwarps) {
    const uint8_t* xr = x + r * xs_bytes;
    uint8_t* yr = y + r * ys_bytes;
    float m = -INFINITY, l = 0.f;  // running max and sum of exp(x - m) of this lane's elements
    for (int64_t c = lane; c < cols; c += 32) {
      const float v = load_elt<DT>(xr, c);
      if (v > m) {
        l = l * ex2_approx((m - v) * kLog2e) + 1.f;  // m = -inf: l is 0 and ex2(-inf) = 0
        m = v;
      } else if (v != -INFINITY) {  // -inf adds nothing (and -inf - -inf would be NaN)
        l += ex2_approx((v - m) * kLog2e);
      }
    }
    const float mr = warp_max(m);
    l = (m == -INFINITY) ? 0.f : l * ex2_approx((m - mr) * kLog2e);
    l = warp_sum(l);
    const float inv = 1.f / l;
    for (int64_t c = lane; c < cols; c += 32)
      store_elt<DT>(yr, c, ex2_approx((load_elt<DT>(xr, c) - mr) * kLog2e) * inv);
  }
}

template <int DT>
int launch_dt(const cmpx_softmax_desc* d, const LaunchCtx& ctx) {
  constexpr int ES = DT == CMPX_F32 ? 4 : 2;
  constexpr int EPC = 16 / ES;
  const uint8_t* x = static_cast<const uint8_t*>(d->x);
  uint8_t* y = static_cast<uint8_t*>(d->y);
  const int64_t xs = d->x_row_stride * ES, ys = d->y_row_stride * ES;
  const int threads = 256;
  const int64_t warps_needed = d->rows;
  const int64_t max_blocks = static_cast<int64_t>(std::max(1, ctx.num_sms)) * 8;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min((warps_needed + 7) / 8, max_blocks)));
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0) &&
                       (xs % 16 == 0) && (ys % 16 == 0) && (d->cols % EPC == 0);
  const int64_t chunks = d->cols / EPC;
  if (aligned && chunks <= 8 * 32) {
    const int c = static_cast<int>(d->cols);
    if (chunks <= 32)
      softmax_rows_reg_kernel<DT, 1><<<blocks, threads, 0, ctx.stream>>>(x, y, d->rows, c, xs, ys);
    else if (chunks <= 64)
      softmax_rows_reg_kernel<DT, 2><<<blocks, threads, 0, ctx.stream>>>(x, y, d->rows, c, xs, ys);
    else if (chunks <= 128)
      softmax_rows_reg_kernel<DT, 4><<<blocks, threads, 0, ctx.stream>>>(x, y, d->rows, c, xs, ys);
    else
      softmax_rows_reg_kernel<DT, 8><<<blocks, threads, 0, ctx.stream>>>(x, y, d->rows, c, xs, ys);
  } else {
    softmax_rows_stream_kernel<DT><<<blocks, threads, 0, ctx.stream>>>(x, y, d->rows, d->cols, xs, ys);
  }
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

}  // namespace

const char* softmax_rows_plan(const cmpx_softmax_desc* d, int* status) {
  *status = CMPX_OK;
  if (!d || !d->x || !d->y || d->rows < 0 || d->cols < 0 || d->x_row_stride < d->cols ||
      d->y_row_stride < d->cols) {
    *status = CMPX_ERR_INVALID_ARGUMENT;
    return "none";
  }
  if (d->dtype != CMPX_F32 && d->dtype != CMPX_F16 && d->dtype != CMPX_BF16) {
    *status = CMPX_ERR_UNSUPPORTED_DTYPE;
    return "none";
  }
  if (d->cols == 0 && d->rows > 0) {
    *status = CMPX_ERR_UNSUPPORTED_SHAPE;
    return "none";
  }
  const int es = d->dtype == CMPX_F32 ? 4 : 2;
  const int epc = 16 / es;
  const bool aligned = (reinterpret_cast<uintptr_t>(d->x) % 16 == 0) && (reinterpret_cast<uintptr_t>(d->y) % 16 == 0) &&
                       ((d->x_row_stride * es) % 16 == 0) && ((d->y_row_stride * es) % 16 == 0) &&
                       (d->cols % epc == 0);
  return aligned && d->cols / epc <= 256 ? "softmax_rows<warp per row, row in registers>"
                                        : "softmax_rows<warp per row, two passes>";
}

int launch_softmax_rows(const cmpx_softmax_desc* d, const LaunchCtx& ctx) {
  if (d->rows == 0) return CMPX_OK;
  if (d->dtype == CMPX_F32) return launch_dt<CMPX_F32>(d, ctx);
  if (d->dtype == CMPX_F16) return launch_dt<CMPX_F16>(d, ctx);
  return launch_dt<CMPX_BF16>(d, ctx);
}

}  // namespace cmpx
