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

// Pair-native helpers: a packed 16-bit pair and the two fp32 values it holds, as one 64-bit
// register pair (the operand of the packed f32x2 arithmetic), so that no value is moved between
// registers to form a pair.
template <bool BF16>
__device__ __forceinline__ uint64_t unpack16x2(uint32_t w) {
  uint64_t r;
  if (BF16)
    asm("{\n\t.reg .b32 lo, hi;\n\tshl.b32 lo, %1, 16;\n\tand.b32 hi, %1, 0xffff0000;\n\tmov.b64 %0, {lo, hi};\n\t}"
        : "=l"(r) : "r"(w));
  else
    asm("{\n\t.reg .b16 l, h;\n\t.reg .f32 lo, hi;\n\tmov.b32 {l, h}, %1;\n\tcvt.f32.f16 lo, l;\n\t"
        "cvt.f32.f16 hi, h;\n\tmov.b64 %0, {lo, hi};\n\t}"
        : "=l"(r) : "r"(w));
  return r;
}
// Rounds a pair of fp32 values to the packed 16-bit pair (round to nearest even).
template <bool BF16>
__device__ __forceinline__ uint32_t pack16x2(uint64_t v) {
  uint32_t r;
  if (BF16)
    asm("{\n\t.reg .f32 lo, hi;\n\tmov.b64 {lo, hi}, %1;\n\tcvt.rn.bf16x2.f32 %0, hi, lo;\n\t}" : "=r"(r) : "l"(v));
  else
    asm("{\n\t.reg .f32 lo, hi;\n\tmov.b64 {lo, hi}, %1;\n\tcvt.rn.f16x2.f32 %0, hi, lo;\n\t}" : "=r"(r) : "l"(v));
  return r;
}
// 2^x of both halves of a pair.
__device__ __forceinline__ uint64_t ex2x2(uint64_t x) {
  uint64_t r;
  asm("{\n\t.reg .f32 lo, hi;\n\tmov.b64 {lo, hi}, %1;\n\tex2.approx.ftz.f32 lo, lo;\n\tex2.approx.ftz.f32 hi, hi;\n\t"
      "mov.b64 %0, {lo, hi};\n\t}"
      : "=l"(r) : "l"(x));
  return r;
}
// Element-wise max of two packed 16-bit pairs (exact; a NaN loses to a number, as fmaxf).
template <bool BF16>
__device__ __forceinline__ uint32_t hmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  if (BF16)
    asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else
    asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Folds 64 consecutive 16-bit scores of one row (packed in pairs; columns col0 .. col0 + 63,
// those at or past n excluded) into the running statistics (cm, cs).
template <bool BF16>
__device__ __forceinline__ void rowstats64(uint32_t (&pk)[32], int col0, int n, float& cm, float& cs) {
  if (col0 + 64 > n) {  // the run's tail past n: -inf, which adds nothing
    const uint32_t ninf = BF16 ? 0xff80u : 0xfc00u;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      if (col0 + 2 * e >= n) pk[e] = (pk[e] & 0xffff0000u) | ninf;
      if (col0 + 2 * e + 1 >= n) pk[e] = (pk[e] & 0x0000ffffu) | (ninf << 16);
    }
  }
  uint32_t t[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) t[e] = hmax2<BF16>(pk[e], pk[e + 16]);
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
    for (int e = 0; e < w; ++e) t[e] = hmax2<BF16>(t[e], t[e + w]);
  float lo, hi;
  f2_unpack(unpack16x2<BF16>(t[0]), lo, hi);
  const float mx = fmaxf(lo, hi);
  if (mx > cm) {
    if (cm != -INFINITY) cs *= ex2_approx((cm - mx) * kRowLog2e);
    cm = mx;
  }
  if (cm == -INFINITY) return;
  // 2^(v log2e - cm log2e), two columns per packed FMA, the sum in four packed accumulators
  const uint64_t l2 = f2_pack(kRowLog2e, kRowLog2e), nm = f2_pack(-cm * kRowLog2e, -cm * kRowLog2e);
  uint64_t acc[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] = f2_pack(0.f, 0.f);
#pragma unroll
  for (int e = 0; e < 32; ++e) acc[e & 3] = f2_add(acc[e & 3], ex2x2(f2_fma(unpack16x2<BF16>(pk[e]), l2, nm)));
  float s0, s1;
  f2_unpack(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])), s0, s1);
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
