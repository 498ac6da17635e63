// Row statistics of a softmax over 16-bit scores: shared by the bmm kernel that writes the scores
// (and their per-64-column statistics) and the fused softmax that consumes them.
//
// The statistics of a run of columns of one row are (max, sum): max = the largest 16-bit score,
// sum = sum over the run of 2^((v - max) * log2 e), every v being the score as stored (rounded to
// the 16-bit type).  Runs combine as (max(m1, m2), s1 * 2^((m1 - m) log2 e) + s2 * 2^(...)); a run
// of -inf only is (-inf, 0).  The softmax of the row is then 2^(v log2 e - max log2 e - log2 sum).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "cmpx_ptx.cuh"

namespace cmpx {

constexpr float kRowLog2e = 1.4426950408889634f;

template <bool BF16>
__device__ __forceinline__ uint32_t pack16(float lo, float hi) {
  return BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}
// The two values of a packed 16-bit pair, back in fp32 (exact).
template <bool BF16>
__device__ __forceinline__ void unpack16(uint32_t v, float& lo, float& hi) {
  if (BF16) {
    lo = __uint_as_float(v << 16);
    hi = __uint_as_float(v & 0xFFFF0000u);
  } else {
    const __half2 h = *reinterpret_cast<const __half2*>(&v);
    lo = __low2float(h);
    hi = __high2float(h);
  }
}

// Folds 32 consecutive 16-bit scores of one row (packed in pairs; columns col0 .. col0 + 31,
// those at or past n excluded) into the running statistics (cm, cs).
template <bool BF16>
__device__ __forceinline__ void rowstats32(const uint32_t (&pk)[16], int col0, int n, float& cm, float& cs) {
  float v[32];
#pragma unroll
  for (int e = 0; e < 16; ++e) unpack16<BF16>(pk[e], v[2 * e], v[2 * e + 1]);
  if (col0 + 32 > n) {
#pragma unroll
    for (int e = 0; e < 32; ++e)
      if (col0 + e >= n) v[e] = -INFINITY;
  }
  float a8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) a8[e] = fmax3(v[e], v[8 + e], v[16 + e]);
#pragma unroll
  for (int e = 0; e < 8; ++e) a8[e] = fmaxf(a8[e], v[24 + e]);
  const float mx = fmax3(fmax3(a8[0], a8[1], a8[2]), fmax3(a8[3], a8[4], a8[5]), fmaxf(a8[6], a8[7]));
  if (mx > cm) {
    if (cm != -INFINITY) cs *= ex2_approx((cm - mx) * kRowLog2e);
    cm = mx;
  }
  if (cm == -INFINITY) return;
  // 2^(v log2e - cm log2e): two columns per packed FMA, the sum in two packed accumulators
  const uint64_t l2 = f2_pack(kRowLog2e, kRowLog2e), nm = f2_pack(-cm * kRowLog2e, -cm * kRowLog2e);
  uint64_t sa = f2_pack(0.f, 0.f), sb = sa;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    float x0, x1;
    f2_unpack(f2_fma(f2_pack(v[2 * e], v[2 * e + 1]), l2, nm), x0, x1);
    if (e & 1)
      sb = f2_add(sb, f2_pack(ex2_approx(x0), ex2_approx(x1)));
    else
      sa = f2_add(sa, f2_pack(ex2_approx(x0), ex2_approx(x1)));
  }
  float s0, s1;
  f2_unpack(f2_add(sa, sb), s0, s1);
  cs += s0 + s1;
}

// Combines statistics (m2, s2) into (m, s).
__device__ __forceinline__ void rowstats_merge(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m2 > m) {
    s = (m == -INFINITY ? 0.f : s * ex2_approx((m - m2) * kRowLog2e)) + s2;
    m = m2;
  } else {
    s += s2 * ex2_approx((m2 - m) * kRowLog2e);
  }
}

}  // namespace cmpx
