// bmm_x3_sm100.cu -- fp32 batched matmul C[b] = A[b] @ B[b] (+ bias) on the tensor cores (B200 sm_100a).
//
// Replaces the reference's fp32 GEMM (gemm_fp32_ga100_kernel, src/cuda/fp32_matmul.cu:31-184,
// launched per batch item from custom_bmm_forward, src/main.cpp:363-441: FMUL/FADD on the CUDA
// cores) for fp32 calls of cmpext3.ops.bmm and, with a bias, cmpext3.ops.linear.  One TF32 product
// keeps 10 mantissa bits (~1e-3 per element), short of the fp32 contract, so every product is
// split the 3xTF32 way: x = x_hi + x_lo with x_hi the value truncated to TF32 (exact) and
// x_lo = x - x_hi (exact in fp32), and a b ~= a_hi b_hi + a_hi b_lo + a_lo b_hi (the dropped
// a_lo b_lo is ~2^-22 relative).
//
//   * one persistent launch: a CTA per SM walks the 128 x 128 output tiles of every batch item in
//     bands of 16 row tiles (as the 16-bit GEMM);
//   * operands are K-major (A rows and B columns contiguous along K, read in place through rank-3
//     TMA maps); 32-element (128-byte) K blocks stream through a 3-stage ring of 64 KB stages:
//     A and B as loaded (their hi parts) and their lo parts;
//   * split operands (a caller workspace, cmpx_bmm_ws / cmpx_linear_ws): x3_lo_kernel writes lo(A)
//     and lo(B) once per call, K-major (x3_lo_t_kernel also hi(B) for a B stored MN-major), and
//     warp 0 loads them beside A and B, four tiles per stage; the converter warps then idle.  The
//     split done per stage in shared memory (below) is what bounds the GEMM otherwise: 4096^3 runs
//     at 226 TFLOP/s split against 136;
//   * warp 0: TMA; warps 2-9 ("converter", without a workspace or after the pass flagged a NaN it
//     cannot keep): per stage, lo = x - trunc(x) for both tiles.  The hi part is the word as
//     loaded: the tensor core's TF32 read of an fp32 word keeps its top 19 bits (measured: the same
//     results as explicitly truncated operands).  Only an inf / NaN word is rewritten in place (a
//     NaN whose payload sits in the dropped bits would read as inf);
//     warp 1: 12 tcgen05.mma kind::tf32 per stage (4 K-steps of 8 x 3 products) into
//     one of two TMEM tile buffers, so tile i+1's products overlap tile i's epilogue.  A buffer is
//     two accumulators: hi*hi, and the two cross terms, ~2^-11 smaller.  The tensor core's fp32
//     accumulation loses a little on every add into a large sum (measured: error growing linearly
//     with K), so the cross terms are summed apart from the large one and the two meet once, in
//     the epilogue: a third of the adds into the large sum;
//   * warps 10-17: TMEM -> fp32 sum of the two accumulators (+ bias) -> swizzled shared staging ->
//     TMA stores (clipped at M, N).
// Every wait is bounded (cmpx_ptx.cuh); a CTA that gives up drains its copies and MMAs, frees TMEM,
// raises the device status word and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "cmpx_internal.h"
#include "cmpx_ptx.cuh"

namespace cmpx {

struct X3GemmCfg {
  static constexpr int BM = 128, BN = 128, BK = 32;  // BK fp32 = one 128-byte swizzle row
  static constexpr int TILE = 128 * 128;             // 16 KB: a 128-row A or B tile of one K block
  static constexpr int A_HI = 0, A_LO = TILE, B_HI = 2 * TILE, B_LO = 3 * TILE;
  static constexpr int STAGE_BYTES = 4 * TILE;       // 64 KB
  static constexpr int STAGES = 3;
  static constexpr int SLOT_BYTES = 32 * 128;        // one epilogue warp's 32 rows x 32 fp32
  static constexpr int EPI_WARPS = 8;
  static constexpr int OFF_STAGING = STAGES * STAGE_BYTES;
  static constexpr int OFF_BAR = OFF_STAGING + EPI_WARPS * SLOT_BYTES;
  static constexpr int B_FULL = 0, B_CONV = STAGES, B_EMPTY = 2 * STAGES;  // [STAGES] each
  static constexpr int B_ACCF = 3 * STAGES, B_ACCE = 3 * STAGES + 2;       // [2] each
  static constexpr int B_DRAIN = 3 * STAGES + 4;
  static constexpr int NBAR = 3 * STAGES + 5;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // +1024: runtime alignment slack
  // Two tile buffers, each a main accumulator (hi*hi) and a cross-term one (hi*lo + lo*hi).
  static constexpr int TMEM_COLS = 4 * BN;
  static constexpr int THREADS = 576;  // warp 0 TMA, 1 MMA, 2-9 converter, 10-17 epilogue
  static constexpr int CONV_THREADS = 256;
  static constexpr int W_EPI = 10;
  // Longest K one launch accumulates: the tensor core's fp32 accumulation error grows with K
  // (measured rel-to-peak vs float64: 1e-5 at K = 4096, 2e-5 at 8192, 9e-5 at 32768).  Longer
  // products run as several launches over K chunks of at most this length: the first stores C,
  // the others add their fp32 partial products into it (TMA reduce-add), so the error stays that
  // of one chunk.
  static constexpr int MAX_K = 8192;
};
static_assert(X3GemmCfg::SMEM_BYTES <= 232448, "shared memory");

struct X3GemmParams {
  int m, n, k;
  int n_kblocks;
  int tiles_m, tiles_n, n_tiles;
  const float* bias;  // [n] added to every row (linear), or null
  int accumulate;     // 1: add the product into C (a later K chunk), 0: store it
  // Split operands (pre = 1): the lo parts of A and B were written once per call by x3_lo_kernel
  // and are loaded by TMA beside the operands, so the converter warps have nothing to do; unless
  // that pass raised *special (a NaN the tensor core would read as inf), in which case the
  // converter path runs (it rewrites such words in shared memory).
  int pre;
  const unsigned int* special;
  unsigned long long timeout_ns;
  unsigned int* dev_flags;
};

__device__ __forceinline__ bool x3_special(uint32_t bits) { return (bits & 0x7F800000u) == 0x7F800000u; }
// The exact remainder below the TF32 part; 0 for inf / NaN.
__device__ __forceinline__ uint32_t x3_lo(uint32_t bits) {
  return x3_special(bits) ? 0u : __float_as_uint(__uint_as_float(bits) - __uint_as_float(bits & 0xFFFFE000u));
}
// The word the tensor core is given as the TF32 part of an inf / NaN (a NaN stays a NaN).
__device__ __forceinline__ uint32_t x3_hi_special(uint32_t bits) {
  return x3_special(bits) && (bits & 0x007FFFFFu) ? 0x7FC00000u : bits;
}
// A NaN whose payload sits only in the 13 bits TF32 drops: the tensor core would read it as inf.
__device__ __forceinline__ bool x3_nan_low(uint32_t bits) {
  return x3_special(bits) && (bits & 0x007FFFFFu) != 0u && (bits & 0x007FE000u) == 0u;
}

// The lo parts of one K-major operand, once per call: x is `batch` items of `rows` rows of k
// elements (row_stride / batch_stride elements apart, contiguous along k, 16-byte aligned rows);
// lo is [batch][rows][k_pad] packed, x3_lo of each element and zero past k.  The hi part is the
// operand itself, as the converter path uses it.  A block walks whole rows, a thread one float4.
struct X3LoParams {
  const float* x;
  long long batch_stride, row_stride;
  int rows, k, k_pad, batch;
  float* lo;
  unsigned int* special;
};

// The same for a B stored MN-major (element (z, kk, j) at x + z * batch_stride + kk * row_stride + j,
// contiguous along n): both parts written K-major, hi = the word itself, through a shared-memory
// 32 x 32 transpose, so the GEMM reads B from the workspace and no transposed copy of B is made.
struct X3LoTParams {
  const float* x;
  long long batch_stride, row_stride;
  int n, k, k_pad, tiles_j, tiles_k;
  float* hi;
  float* lo;
  unsigned int* special;
};

__global__ void __launch_bounds__(256) x3_lo_t_kernel(const X3LoTParams p) {
  __shared__ uint32_t t[32][33];
  const int z = blockIdx.y;
  const int tile = blockIdx.x, tj = tile % p.tiles_j, tk = tile / p.tiles_j;
  const int j0 = tj * 32, kk0 = tk * 32;
  const float* src = p.x + z * p.batch_stride;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int kk = kk0 + i, j = j0 + threadIdx.x;
    t[i][threadIdx.x] = (kk < p.k && j < p.n) ? __float_as_uint(__ldg(src + kk * p.row_stride + j)) : 0u;
  }
  __syncthreads();
  bool bad = false;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int j = j0 + i, kk = kk0 + threadIdx.x;
    if (j < p.n && kk < p.k_pad) {
      const uint32_t w = t[threadIdx.x][i];
      const size_t o = (static_cast<size_t>(z) * p.n + j) * p.k_pad + kk;
      p.hi[o] = __uint_as_float(w);
      p.lo[o] = __uint_as_float(x3_lo(w));
      bad |= x3_nan_low(w);
    }
  }
  if (bad) atomicOr(p.special, 1u);
}

__global__ void __launch_bounds__(256) x3_lo_kernel(const X3LoParams p) {
  const int quads = p.k_pad >> 2;
  const long long n_rows = static_cast<long long>(p.batch) * p.rows;
  bool bad = false;
  for (long long rr = blockIdx.x; rr < n_rows; rr += gridDim.x) {
    const long long z = rr / p.rows, r = rr - z * p.rows;
    const float* src = p.x + z * p.batch_stride + r * p.row_stride;
    float4* dst = reinterpret_cast<float4*>(p.lo + rr * p.k_pad);
    for (int q = threadIdx.x; q < quads; q += blockDim.x) {
      const int k0 = q * 4;
      uint32_t w[4];
      if (k0 + 4 <= p.k) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(src + k0));
        w[0] = __float_as_uint(v.x); w[1] = __float_as_uint(v.y); w[2] = __float_as_uint(v.z); w[3] = __float_as_uint(v.w);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = k0 + e < p.k ? __float_as_uint(__ldg(src + k0 + e)) : 0u;
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) bad |= x3_nan_low(w[e]);
      dst[q] = make_float4(__uint_as_float(x3_lo(w[0])), __uint_as_float(x3_lo(w[1])), __uint_as_float(x3_lo(w[2])),
                           __uint_as_float(x3_lo(w[3])));
    }
  }
  if (bad) atomicOr(p.special, 1u);
}

__global__ void __launch_bounds__(576, 1)
    bmm_x3_sm100_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_alo,
                        const __grid_constant__ CUtensorMap tm_blo, const X3GemmParams p) {
  using C = X3GemmCfg;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  auto bar = [&](int i) -> uint32_t { return base + C::OFF_BAR + 8u * i; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  auto stage = [&](int it) -> uint32_t { return base + (it % C::STAGES) * C::STAGE_BYTES; };
  // Tile t -> (batch item z, first row m0, first column n0): bands of kBand row tiles, m fastest
  // inside a band, so the CTAs busy at one moment share a band of A and a few column tiles of B.
  constexpr int kBand = 16;
  auto decode = [&](int t, int& z, int& m0, int& n0) {
    const int per_item = p.tiles_m * p.tiles_n;
    z = t / per_item;
    const int r = t - z * per_item;
    const int band = r / (kBand * p.tiles_n);
    const int first_m = band * kBand;
    const int rows = min(kBand, p.tiles_m - first_m);
    const int w = r - band * kBand * p.tiles_n;
    m0 = (first_m + w % rows) * C::BM;
    n0 = (w / rows) * C::BN;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar(C::B_FULL + s), 1);
      mbar_init(bar(C::B_CONV + s), C::CONV_THREADS);
      mbar_init(bar(C::B_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(C::B_ACCF + b), 1);
      mbar_init(bar(C::B_ACCE + b), C::EPI_WARPS);
    }
    mbar_init(bar(C::B_DRAIN), 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
    tmem_relinquish();
  }
  const bool pre = p.pre != 0 && p.special[0] == 0u;  // (written by the previous kernel on this stream)
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_c);
    if (pre) {
      tma_prefetch_desc(&tm_alo);
      tma_prefetch_desc(&tm_blo);
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const WaitCtl ctl{abort_flag, p.dev_flags, p.timeout_ns};

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;  // K blocks issued so far over all of this CTA's tiles (ring position)
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.n_tiles; t += gridDim.x) {
        int z, m0, n0;
        decode(t, z, m0, n0);
        for (int kb = 0; kb < p.n_kblocks; ++kb, ++it) {
          const int st = it % C::STAGES;
          if (!(ok = mbar_wait(bar(C::B_EMPTY + st), (static_cast<uint32_t>(it / C::STAGES) & 1u) ^ 1u, ctl))) break;
          const uint32_t s = stage(it);
          mbar_arrive_expect_tx(bar(C::B_FULL + st), (pre ? 4 : 2) * C::TILE);
          tma_load_3d(s + C::A_HI, &tm_a, bar(C::B_FULL + st), kb * C::BK, m0, z);
          tma_load_3d(s + C::B_HI, &tm_b, bar(C::B_FULL + st), kb * C::BK, n0, z);
          if (pre) {
            tma_load_3d(s + C::A_LO, &tm_alo, bar(C::B_FULL + st), kb * C::BK, m0, z);
            tma_load_3d(s + C::B_LO, &tm_blo, bar(C::B_FULL + st), kb * C::BK, n0, z);
          }
        }
      }
      if (*abort_flag) {
        // Let every copy still in flight land before shared memory goes away.
        for (int i = max(0, it - C::STAGES); i < it; ++i)
          mbar_wait_drain(bar(C::B_FULL + i % C::STAGES), static_cast<uint32_t>(i / C::STAGES) & 1u,
                          p.timeout_ns);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (warp-uniform)
    constexpr uint32_t kIdesc = idesc_tf32(128, C::BN, 0, 0);  // K-major A and B
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x, i = 0; ok && t < p.n_tiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      if (!(ok = mbar_wait_all(bar(C::B_ACCE + b), (static_cast<uint32_t>(i >> 1) & 1u) ^ 1u, ctl))) break;
      tc_fence_after_sync();
      const uint32_t d_main = tmem + b * 2 * C::BN, d_cross = d_main + C::BN;
      for (int kb = 0; kb < p.n_kblocks; ++kb, ++it) {
        const int st = it % C::STAGES;
        if (!(ok = mbar_wait_all(bar((pre ? C::B_FULL : C::B_CONV) + st), static_cast<uint32_t>(it / C::STAGES) & 1u,
                                 ctl)))
          break;
        tc_fence_after_sync();
        const uint32_t s = stage(it);
        const uint64_t dah = smem_desc_sw128(s + C::A_HI, 16, 1024);
        const uint64_t dal = smem_desc_sw128(s + C::A_LO, 16, 1024);
        const uint64_t dbh = smem_desc_sw128(s + C::B_HI, 16, 1024);
        const uint64_t dbl = smem_desc_sw128(s + C::B_LO, 16, 1024);
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // K-steps of 8 fp32 = 32 bytes along the swizzled row
          const uint64_t ko = static_cast<uint64_t>((k * 32) >> 4);
          const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
          umma_ss_tf32_w(d_cross, dah + ko, dbl + ko, kIdesc, acc);
          umma_ss_tf32_w(d_cross, dal + ko, dbh + ko, kIdesc, 1u);
          umma_ss_tf32_w(d_main, dah + ko, dbh + ko, kIdesc, acc);
        }
        umma_commit_w(bar(C::B_EMPTY + st));
      }
      if (ok) umma_commit_w(bar(C::B_ACCF + b));
    }
  } else if (warp < C::W_EPI) {
    // ------------------------------------------------------------------ converter (warps 2-9)
    // Both tiles of a stage are 1024 16-byte units each, their lo parts 16 KB further on: unit v
    // of 2048 is tile v / 1024, and hi / lo are elementwise, so the swizzled layout carries over.
    const int tid = threadIdx.x - 64;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && !pre && t < p.n_tiles; t += gridDim.x) {  // (split operands: idle)
      for (int kb = 0; kb < p.n_kblocks; ++kb, ++it) {
        const int st = it % C::STAGES;
        if (!(ok = mbar_wait_all(bar(C::B_FULL + st), static_cast<uint32_t>(it / C::STAGES) & 1u, ctl))) break;
        const uint32_t s = stage(it);
#pragma unroll 4
        for (int v = tid; v < 2048; v += C::CONV_THREADS) {
          const uint32_t hi_addr = s + (v >> 10) * (2 * C::TILE) + (v & 1023) * 16;
          uint32_t x0, x1, x2, x3;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(x0), "=r"(x1), "=r"(x2), "=r"(x3)
                       : "r"(hi_addr));
          st_shared_v4(hi_addr + C::TILE, x3_lo(x0), x3_lo(x1), x3_lo(x2), x3_lo(x3));
          if (x3_special(x0) | x3_special(x1) | x3_special(x2) | x3_special(x3))
            st_shared_v4(hi_addr, x3_hi_special(x0), x3_hi_special(x1), x3_hi_special(x2), x3_hi_special(x3));
        }
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core's reads
        mbar_arrive(bar(C::B_CONV + st));
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 10..17)
    // Warp w reads TMEM lane quarter w % 4 (the quarter its warp index may address) and the
    // 32-column chunks c = half, half + 2 of each tile, through its own 4 KB staging slot: a
    // chunk waits until the store of the slot's previous chunk has read it.
    const int quarter = warp & 3;
    const int half = (warp - C::W_EPI) >> 2;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t slot = base + C::OFF_STAGING + (warp - C::W_EPI) * C::SLOT_BYTES;
    bool ok = true;
    bool stored = false;
    for (int t = blockIdx.x, i = 0; ok && t < p.n_tiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      int z, m0, n0;
      decode(t, z, m0, n0);
      if (!(ok = mbar_wait_all(bar(C::B_ACCF + b), static_cast<uint32_t>(i >> 1) & 1u, ctl))) break;
      tc_fence_after_sync();
      const int r0 = m0 + quarter * 32;
#pragma unroll 1
      for (int c = half; c < C::BN / 32; c += 2) {
        uint32_t acc[32], cross[32];
        tmem_ld32(t_lane + b * 2 * C::BN + c * 32, acc);
        tmem_ld32(t_lane + b * 2 * C::BN + C::BN + c * 32, cross);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = __float_as_uint(__uint_as_float(acc[j]) + __uint_as_float(cross[j]));
        if (c + 2 >= C::BN / 32) {
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(C::B_ACCE + b));  // accumulator b read
        }
        const int col0 = n0 + c * 32;
        if (p.bias) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < p.n) acc[j] = __float_as_uint(__uint_as_float(acc[j]) + __ldg(p.bias + col0 + j));
        }
        if (stored) {  // the slot's previous chunk must have been read by its store
          if (lane == 0) bulk_wait_group_read0();
          __syncwarp();
        }
#pragma unroll
        for (int q = 0; q < 8; ++q)
          st_shared_v4(slot + lane * 128 + ((q ^ (lane & 7)) << 4), acc[4 * q], acc[4 * q + 1],
                       acc[4 * q + 2], acc[4 * q + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (r0 < p.m && col0 < p.n) {
            if (p.accumulate)
              tma_reduce_add_3d(&tm_c, slot, col0, r0, z);
            else
              tma_store_3d(&tm_c, slot, col0, r0, z);
          }
          bulk_commit_group();
        }
        __syncwarp();
        stored = true;
      }
    }
    if (lane == 0) bulk_wait_group0();  // every store of this warp complete before exit
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    if (*abort_flag) {
      __syncwarp();
      umma_commit_w(bar(C::B_DRAIN));  // same election as the MMAs: tracks all of them
      if (lane == 0) mbar_wait_drain(bar(C::B_DRAIN), 0, p.timeout_ns);
      __syncwarp();
    }
    tc_fence_after_sync();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// --------------------------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------------------------
namespace {

// A positive element stride whose fp32 byte stride TMA accepts (a multiple of 16 bytes).
inline bool s16f(int64_t s) { return s > 0 && ((s * 4) % 16) == 0 && (s * 4) < (1ll << 40); }

// The byte stride of a dimension that holds one index: any multiple of 16 serves (never stepped).
inline uint64_t unit_stride(int64_t s, int64_t extent, int64_t fallback_elems) {
  if (extent == 1 && !s16f(s)) return static_cast<uint64_t>((fallback_elems * 4 + 15) / 16 * 16);
  return static_cast<uint64_t>(s) * 4;
}

constexpr const char* kX3Name = "bmm_x3tf32_sm100<f32,128x128x32,3st,persistent>";
constexpr const char* kX3ChunkName = "bmm_x3tf32_sm100<f32,128x128x32,3st,persistent+k-chunks>";

// Workspace of the split-operand schedule: bytes [0, 256) are left as they are (the attention
// calls' zero-kept counters, so one workspace serves both), the pass's special-value flag at 256,
// lo(A) from 512, lo(B) after it, each [batch][rows][k_pad] fp32 with k_pad = k rounded up to 4.
struct X3Ws {
  size_t bytes = 0, off_alo = 0, off_blo = 0, off_bhi = 0;  // off_bhi: MN-major B only
  int64_t k_pad = 0;
};

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Split operands pay when each operand tile is read by enough output tiles and the product is long
// enough for the converter's shared-memory traffic to be what bounds a tile: the pass moves every
// element of A and B three more times (read, lo written, lo read by the GEMM).  Measured on a B200
// (converter -> split, TFLOP/s): 1024^3 48 -> 63, 16384 x 1024 x 1024 135 -> 195, 4096^3 136 -> 226;
// but 4 x 1024 x 256 x 1024 83 -> 70 and 64 x 2048 x 64 x 2048 121 -> 112 (a few K blocks per tile:
// the epilogue, not the converter, sets the pace).  Hence m n / (m + n) >= 512 and k >= 512.
inline X3Ws x3_ws_layout(const cmpx_bmm_desc* d, bool b_mn = false) {
  X3Ws w;
  const double m = static_cast<double>(d->m), n = static_cast<double>(d->n);
  if (d->m < 1 || d->n < 1 || d->k < 512 || m * n / (m + n) < 512.0) return w;
  w.k_pad = (d->k + 3) / 4 * 4;
  w.off_alo = 512;
  w.off_blo = w.off_alo + align256(static_cast<size_t>(d->batch) * d->m * w.k_pad * 4);
  w.bytes = w.off_blo + align256(static_cast<size_t>(d->batch) * d->n * w.k_pad * 4);
  if (b_mn) {
    w.off_bhi = w.bytes;
    w.bytes = w.off_bhi + align256(static_cast<size_t>(d->batch) * d->n * w.k_pad * 4);
  }
  return w;
}

// An fp32 product whose only departure from the plan's layouts is an MN-major B (a row-major
// [k, n] matrix, contiguous along n, rows 16-byte aligned): served through the workspace, where the
// pass writes B's hi and lo parts K-major.
inline bool x3_b_mn_ok(const cmpx_bmm_desc* d) {
  if (d->dtype != CMPX_F32 || d->k < 1 || d->m > (int64_t)128 * 65535 || d->n > (1ll << 31) - 256 ||
      d->batch > 65535 || d->k > (1ll << 31) - 64)
    return false;
  const void* ptrs[3] = {d->a, d->b, d->c};
  for (const void* ptr : ptrs)
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) return false;
  const bool a_ok = d->a_stride[2] == 1 && (d->m == 1 || s16f(d->a_stride[1]));
  const bool b_ok = d->b_stride[2] == 1 && (d->k == 1 || s16f(d->b_stride[1]));
  const bool c_ok = d->c_stride[2] == 1 && (d->m == 1 || s16f(d->c_stride[1]));
  const bool batch_ok = d->batch == 1 || (s16f(d->a_stride[0]) && s16f(d->b_stride[0]) && s16f(d->c_stride[0]));
  return a_ok && b_ok && c_ok && batch_ok;
}

}  // namespace

const char* bmm_x3_plan(const cmpx_bmm_desc* d, int* status) {
  *status = CMPX_OK;
  if (d->dtype != CMPX_F32) {
    *status = CMPX_ERR_UNSUPPORTED_DTYPE;
    return "none";
  }
  if (d->k < 1 || d->m > (int64_t)128 * 65535 || d->n > (1ll << 31) - 256 || d->batch > 65535 ||
      d->k > (1ll << 31) - 64) {
    *status = CMPX_ERR_UNSUPPORTED_SHAPE;
    return "none";
  }
  const void* ptrs[3] = {d->a, d->b, d->c};
  for (const void* ptr : ptrs)
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) {
      *status = CMPX_ERR_MISALIGNED;
      return "none";
    }
  // K-major operands only: A contiguous along K (rows 16-byte aligned), B contiguous along K
  // (columns 16-byte aligned); C rows contiguous and 16-byte aligned.
  const bool a_ok = d->a_stride[2] == 1 && (d->m == 1 || s16f(d->a_stride[1]));
  const bool b_ok = d->b_stride[1] == 1 && (d->n == 1 || s16f(d->b_stride[2]));
  const bool c_ok = d->c_stride[2] == 1 && (d->m == 1 || s16f(d->c_stride[1]));
  const bool batch_ok = d->batch == 1 || (s16f(d->a_stride[0]) && s16f(d->b_stride[0]) && s16f(d->c_stride[0]));
  if (!a_ok || !b_ok || !c_ok || !batch_ok) {
    *status = CMPX_ERR_MISALIGNED;
    return "none";
  }
  return d->k > X3GemmCfg::MAX_K ? kX3ChunkName : kX3Name;
}

namespace {

// The split operands of one launch: lo(A) and lo(B) (already offset to the launch's first k) with
// their row pitch, and the pass's flag; null lo pointers: the converter path.
struct X3Pre {
  const float* lo_a = nullptr;
  const float* lo_b = nullptr;
  int64_t k_pad = 0;
  const unsigned int* special = nullptr;
};

int launch_x3_once(const cmpx_bmm_desc* d, const LaunchCtx& ctx, const float* bias, int accumulate, const X3Pre& pre) {
  using C = X3GemmCfg;
  const uint64_t M = d->m, N = d->n, K = d->k, Z = d->batch;
  CUtensorMap ta, tb, tc, talo, tblo;
  {
    const uint64_t dims[3] = {K, M, Z};
    const uint64_t st[2] = {unit_stride(d->a_stride[1], d->m, d->k),
                            unit_stride(d->a_stride[0], d->batch, d->m * d->k)};
    const uint32_t box[3] = {32, 128, 1};
    if (!encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, d->a, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return CMPX_ERR_LAUNCH;
  }
  {
    const uint64_t dims[3] = {K, N, Z};
    const uint64_t st[2] = {unit_stride(d->b_stride[2], d->n, d->k),
                            unit_stride(d->b_stride[0], d->batch, d->n * d->k)};
    const uint32_t box[3] = {32, 128, 1};
    if (!encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, d->b, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return CMPX_ERR_LAUNCH;
  }
  {
    const uint64_t dims[3] = {N, M, Z};
    const uint64_t st[2] = {unit_stride(d->c_stride[1], d->m, d->n),
                            unit_stride(d->c_stride[0], d->batch, d->m * d->n)};
    const uint32_t box[3] = {32, 32, 1};
    if (!encode_tmap(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, d->c, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return CMPX_ERR_LAUNCH;
  }
  const bool use_pre = pre.lo_a != nullptr;
  if (use_pre) {
    const uint32_t box[3] = {32, 128, 1};
    const uint64_t da[3] = {K, M, Z}, sa[2] = {static_cast<uint64_t>(pre.k_pad) * 4, M * pre.k_pad * 4};
    const uint64_t db[3] = {K, N, Z}, sb[2] = {static_cast<uint64_t>(pre.k_pad) * 4, N * pre.k_pad * 4};
    if (!encode_tmap(&talo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, pre.lo_a, da, sa, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&tblo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, pre.lo_b, db, sb, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return CMPX_ERR_LAUNCH;
  } else {
    talo = ta;  // (not read)
    tblo = tb;
  }
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(reinterpret_cast<const void*>(&bmm_x3_sm100_kernel),
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return CMPX_ERR_LAUNCH;
  X3GemmParams p;
  p.m = static_cast<int>(M);
  p.n = static_cast<int>(N);
  p.k = static_cast<int>(K);
  p.n_kblocks = static_cast<int>((K + C::BK - 1) / C::BK);
  p.tiles_m = static_cast<int>((M + C::BM - 1) / C::BM);
  p.tiles_n = static_cast<int>((N + C::BN - 1) / C::BN);
  const int64_t n_tiles = static_cast<int64_t>(p.tiles_m) * p.tiles_n * static_cast<int64_t>(Z);
  if (n_tiles > (1ll << 31) - 1) return CMPX_ERR_UNSUPPORTED_SHAPE;
  p.n_tiles = static_cast<int>(n_tiles);
  p.bias = bias;
  p.accumulate = accumulate;
  p.pre = use_pre ? 1 : 0;
  p.special = use_pre ? pre.special : ctx.dev_flags;  // (read only when pre = 1)
  p.timeout_ns = ctx.timeout_ns;
  p.dev_flags = ctx.dev_flags;
  const int grid = static_cast<int>(std::min<int64_t>(n_tiles, std::max(1, ctx.num_sms)));
  bmm_x3_sm100_kernel<<<grid, C::THREADS, C::SMEM_BYTES, ctx.stream>>>(ta, tb, tc, talo, tblo, p);
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

// The product over K in chunks of at most MAX_K (equal lengths, multiples of 32): one launch per
// chunk on the caller's stream, the first storing C (and adding the bias), the others adding into
// it.  A and B are K-major, so a chunk is the same operand from element k0 on: its pointers move
// by k0 elements (16-byte aligned, k0 being a multiple of 32).
int launch_x3_lo(const float* x, long long batch_stride, long long row_stride, int64_t rows, const cmpx_bmm_desc* d,
                 int64_t k_pad, float* lo, unsigned int* special, const LaunchCtx& ctx) {
  X3LoParams q;
  q.x = x;
  q.batch_stride = batch_stride;
  q.row_stride = row_stride;
  q.rows = static_cast<int>(rows);
  q.k = static_cast<int>(d->k);
  q.k_pad = static_cast<int>(k_pad);
  q.batch = static_cast<int>(d->batch);
  q.lo = lo;
  q.special = special;
  const int64_t n_rows = rows * d->batch;
  const int threads = static_cast<int>(std::min<int64_t>(256, std::max<int64_t>(32, (k_pad / 4 + 31) / 32 * 32)));
  const int grid = static_cast<int>(std::min<int64_t>(n_rows, std::max(1, ctx.num_sms) * 32));
  x3_lo_kernel<<<grid, threads, 0, ctx.stream>>>(q);
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

int launch_x3(const cmpx_bmm_desc* d_in, const LaunchCtx& ctx, const float* bias, void* ws, size_t ws_bytes,
              bool b_mn = false) {
  using C = X3GemmCfg;
  X3Pre pre;
  cmpx_bmm_desc dd = *d_in;  // (MN-major B: B is read from the workspace, K-major)
  const cmpx_bmm_desc* d = &dd;
  const X3Ws lay = x3_ws_layout(d, b_mn);
  if (lay.bytes > 0 && ws && ws_bytes >= lay.bytes && (reinterpret_cast<uintptr_t>(ws) & 15u) == 0) {
    uint8_t* w = static_cast<uint8_t*>(ws);
    unsigned int* special = reinterpret_cast<unsigned int*>(w + 256);
    float* lo_a = reinterpret_cast<float*>(w + lay.off_alo);
    float* lo_b = reinterpret_cast<float*>(w + lay.off_blo);
    if (cudaMemsetAsync(special, 0, 16, ctx.stream) != cudaSuccess) return CMPX_ERR_LAUNCH;
    int st = launch_x3_lo(static_cast<const float*>(d->a), d->a_stride[0], d->a_stride[1], d->m, d, lay.k_pad, lo_a,
                          special, ctx);
    if (st == CMPX_OK && !b_mn)
      st = launch_x3_lo(static_cast<const float*>(d->b), d->b_stride[0], d->b_stride[2], d->n, d, lay.k_pad, lo_b,
                        special, ctx);
    if (st == CMPX_OK && b_mn) {
      float* hi_b = reinterpret_cast<float*>(w + lay.off_bhi);
      X3LoTParams q;
      q.x = static_cast<const float*>(d->b);
      q.batch_stride = d->b_stride[0];
      q.row_stride = d->b_stride[1];
      q.n = static_cast<int>(d->n);
      q.k = static_cast<int>(d->k);
      q.k_pad = static_cast<int>(lay.k_pad);
      q.tiles_j = static_cast<int>((d->n + 31) / 32);
      q.tiles_k = static_cast<int>((lay.k_pad + 31) / 32);
      q.hi = hi_b;
      q.lo = lo_b;
      q.special = special;
      const int64_t tiles = static_cast<int64_t>(q.tiles_j) * q.tiles_k;
      if (tiles > (1ll << 31) - 1) return CMPX_ERR_UNSUPPORTED_SHAPE;
      x3_lo_t_kernel<<<dim3(static_cast<unsigned>(tiles), static_cast<unsigned>(d->batch)), dim3(32, 8), 0,
                       ctx.stream>>>(q);
      st = cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
      // from here on B is the K-major copy in the workspace
      dd.b = hi_b;
      dd.b_stride[0] = d->n * lay.k_pad;
      dd.b_stride[1] = 1;
      dd.b_stride[2] = lay.k_pad;
    }
    if (st != CMPX_OK) return st;
    pre.lo_a = lo_a;
    pre.lo_b = lo_b;
    pre.k_pad = lay.k_pad;
    pre.special = special;
  } else if (b_mn) {
    return CMPX_ERR_WORKSPACE;
  }
  if (d->k <= C::MAX_K) return launch_x3_once(d, ctx, bias, 0, pre);
  const int64_t chunks = (d->k + C::MAX_K - 1) / C::MAX_K;
  const int64_t kc = ((d->k + chunks - 1) / chunks + C::BK - 1) / C::BK * C::BK;
  for (int64_t k0 = 0; k0 < d->k; k0 += kc) {
    cmpx_bmm_desc c = *d;
    c.a = static_cast<const float*>(d->a) + k0;
    c.b = static_cast<const float*>(d->b) + k0;
    c.k = std::min<int64_t>(kc, d->k - k0);
    X3Pre pc = pre;
    if (pre.lo_a) {
      pc.lo_a = pre.lo_a + k0;
      pc.lo_b = pre.lo_b + k0;
    }
    const int st = launch_x3_once(&c, ctx, k0 == 0 ? bias : nullptr, k0 == 0 ? 0 : 1, pc);
    if (st != CMPX_OK) return st;
  }
  return CMPX_OK;
}

}  // namespace

size_t bmm_x3_workspace_bytes(const cmpx_bmm_desc* d) {
  int st = CMPX_OK;
  bmm_x3_plan(d, &st);
  if (d->batch == 0) return 0;
  if (st == CMPX_OK) return x3_ws_layout(d).bytes;
  if (st == CMPX_ERR_MISALIGNED && x3_b_mn_ok(d)) return x3_ws_layout(d, true).bytes;
  return 0;
}

int launch_bmm_x3(const cmpx_bmm_desc* d, const LaunchCtx& ctx, void* ws, size_t ws_bytes) {
  int st = CMPX_OK;
  bmm_x3_plan(d, &st);
  const bool b_mn = st == CMPX_ERR_MISALIGNED && x3_b_mn_ok(d) && x3_ws_layout(d, true).bytes > 0 && ws &&
                    ws_bytes >= x3_ws_layout(d, true).bytes;
  if (st != CMPX_OK && !b_mn) return st;
  if (d->m == 0 || d->n == 0 || d->batch == 0) return CMPX_OK;
  return launch_x3(d, ctx, nullptr, ws, ws_bytes, b_mn);
}

const char* linear_x3_plan(const cmpx_linear_desc* d, int* status) {
  *status = CMPX_OK;
  if (d->m < 0 || d->n < 1 || d->k < 1 || d->x_row_stride < d->k || d->w_row_stride < d->k ||
      d->y_row_stride < d->n) {
    *status = CMPX_ERR_INVALID_ARGUMENT;
    return "none";
  }
  if (d->bias && (reinterpret_cast<uintptr_t>(d->bias) & 3u) != 0) {
    *status = CMPX_ERR_MISALIGNED;
    return "none";
  }
  const cmpx_bmm_desc b = linear_as_bmm(d);
  return bmm_x3_plan(&b, status);
}

size_t linear_x3_workspace_bytes(const cmpx_linear_desc* d) {
  int st = CMPX_OK;
  linear_x3_plan(d, &st);
  if (st != CMPX_OK || d->m == 0) return 0;
  const cmpx_bmm_desc b = linear_as_bmm(d);
  return x3_ws_layout(&b).bytes;
}

int launch_linear_x3(const cmpx_linear_desc* d, const LaunchCtx& ctx, void* ws, size_t ws_bytes) {
  int st = CMPX_OK;
  linear_x3_plan(d, &st);
  if (st != CMPX_OK) return st;
  if (d->m == 0) return CMPX_OK;
  const cmpx_bmm_desc b = linear_as_bmm(d);
  return launch_x3(&b, ctx, static_cast<const float*>(d->bias), ws, ws_bytes);
}

}  // namespace cmpx
