// bmm_sm100.cu -- batched matmul C[b] = A[b] @ B[b] for fp16 / bf16 on B200 (sm_100a).
//
// Replaces the reference's bmm path (custom_bmm_forward, src/main.cpp:363-441), which converts
// bf16 operands to fp32 copies, makes them contiguous, and launches one FMUL/FADD GEMM per batch
// item from a host loop (gemm_fp32_ga100_kernel, src/cuda/fp32_matmul.cu:31-184; fp16 uses
// gemm_fp16_sm75 with half2 accumulation, src/cuda/fp16_matmul.cu:143-367).  Here:
//
//   * one persistent launch: a CTA per SM walks the 128 x BN output tiles of every batch item
//     (flattened, n fastest);
//   * operands are read in place through rank-3 TMA maps, row-major OR column-major (a transposed
//     view such as K^T from an einsum plan is a K-major B operand: no copy);
//   * warp 0 streams 128x64 A and 64xBN B tiles through a ring of 128-byte-swizzled stages that
//     runs across tile boundaries; warp 1 issues tcgen05.mma (M=128, N=BN, K=16 steps) into one of
//     two fp32 TMEM accumulators, so tile i+1's MMAs run while tile i is drained; warps 2-9 drain
//     TMEM -> fp32 -> 16-bit -> swizzled shared staging -> TMA stores (two warps per TMEM lane
//     quarter, each taking every other 64-column chunk);
//   * fp32 accumulation over all of K (the reference's fp16 path accumulates in half).
//   For the attention-score shape (K = 64: one k-block per tile, 64 KB of output per tile) the
//   kernel is an HBM write stream; the double accumulator keeps the stores going back to back.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cmath>
#include <mutex>
#include <string>

#include "cmpx_internal.h"
#include "cmpx_ptx.cuh"
#include "rowstats.cuh"

namespace cmpx {

template <int BN>
struct BmmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;       // 16 KB
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN == 64 ? 6 : 4;
  static constexpr int CHUNKS = BN / 64;            // 64-column (128-byte) chunks of a C tile
  static constexpr int SLOT_BYTES = 32 * 128;       // one warp's 32 rows of one chunk
  // Staging of the C tile for the TMA stores.  BN <= 128: a slot per (quarter, chunk), two buffers
  // alternating by tile.  BN = 256 (4 x 48 KB of stages leave 32 KB): one slot per epilogue warp,
  // reused chunk after chunk once the previous chunk's store has read it (ONE_SLOT).
  static constexpr bool ONE_SLOT = BN == 256;
  static constexpr int STAGING_BYTES = ONE_SLOT ? 8 * SLOT_BYTES : 4 * CHUNKS * SLOT_BYTES;
  static constexpr int NBUF = ONE_SLOT ? 1 : 2;
  static constexpr int OFF_STAGING = STAGES * STAGE_BYTES;
  static constexpr int OFF_BAR = OFF_STAGING + NBUF * STAGING_BYTES;
  static constexpr int B_FULL = 0, B_EMPTY = STAGES;                 // [STAGES] each
  static constexpr int B_ACCF = 2 * STAGES, B_ACCE = 2 * STAGES + 2;  // [2] each
  static constexpr int B_DRAIN = 2 * STAGES + 4;
  // row statistics (STATS): staging slots of [buffer][epilogue warp] written / read by the stats warp
  static constexpr int B_SFULL = 2 * STAGES + 5, B_SFREE = B_SFULL + 16;  // [2][8] each
  static constexpr int NBAR = B_SFREE + 16;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 2 * BN;          // two accumulators (128 / 256 / 512 columns)
  static constexpr int THREADS = 320;               // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
  static constexpr int STATS_THREADS = 576;         // + warps 10-17: row statistics of the staged tile
  static constexpr int EPI_WARPS = 8;
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

struct BmmParams {
  int m, n, k;
  int n_kblocks;
  int tiles_m, tiles_n, n_tiles;
  unsigned long long timeout_ns;
  unsigned int* dev_flags;
  const uint16_t* bias;  // [n], same 16-bit type as C, added to every row in fp32 (linear); or null
  // STATS: per row and 64-column run of C, (max, sum) of the stored values (rowstats.cuh), as
  // float2 [batch][ceil(n / 64)][m] (a run's rows contiguous: one 256-byte store per warp)
  float2* stats;
  int stats_runs;
};

// Adds bias[col0 .. col0+31] (16-bit, converted to fp32) to the 32 fp32 accumulator columns of one
// row; columns at or past n get nothing (their outputs are clipped by the store).  Every lane of
// the warp reads the same 64 bytes: one broadcast request per 16 bytes.
template <bool BF16>
__device__ __forceinline__ void add_bias32(uint32_t (&acc)[32], const uint16_t* bias, int col0, int n) {
  if (col0 + 32 <= n) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(bias + col0) + v);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = BF16 ? __uint_as_float(w[e] << 16) : __half2float(__ushort_as_half(w[e] & 0xffffu));
        const float hi = BF16 ? __uint_as_float(w[e] & 0xffff0000u) : __half2float(__ushort_as_half(w[e] >> 16));
        acc[v * 8 + 2 * e] = __float_as_uint(__uint_as_float(acc[v * 8 + 2 * e]) + lo);
        acc[v * 8 + 2 * e + 1] = __float_as_uint(__uint_as_float(acc[v * 8 + 2 * e + 1]) + hi);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (col0 + j < n) {
        const uint16_t h = bias[col0 + j];
        const float f = BF16 ? __uint_as_float(static_cast<uint32_t>(h) << 16) : __half2float(__ushort_as_half(h));
        acc[j] = __float_as_uint(__uint_as_float(acc[j]) + f);
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN, bool BF16, bool STATS = false>
__global__ void __launch_bounds__(STATS ? BmmCfg<BN>::STATS_THREADS : BmmCfg<BN>::THREADS, 1)
    bmm_sm100_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_c, const BmmParams p) {
  using C = BmmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  auto bar = [&](int i) -> uint32_t { return base + C::OFF_BAR + 8u * i; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  // Tile t of a batch item's tiles in bands of kBand m tiles: inside a band m runs fastest, then n.
  // The CTAs busy at one moment hold consecutive tiles -- kBand row tiles of A and ~G / kBand
  // column tiles of B -- so both stay in L2 while they are reused (n fastest over whole rows would
  // stream all of B through L2 once per ~G / tiles_n rows of tiles).
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
    n0 = (w / rows) * BN;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar(C::B_FULL + s), 1);
      mbar_init(bar(C::B_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(C::B_ACCF + b), 1);
      mbar_init(bar(C::B_ACCE + b), C::EPI_WARPS);
    }
    mbar_init(bar(C::B_DRAIN), 1);
    if (STATS) {
      for (int i = 0; i < 16; ++i) {
        mbar_init(bar(C::B_SFULL + i), 1);
        mbar_init(bar(C::B_SFREE + i), 1);
      }
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_c);
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const WaitCtl ctl{abort_flag, p.dev_flags, p.timeout_ns};

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;  // k-blocks issued so far, over all of this CTA's tiles (ring position)
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.n_tiles; t += gridDim.x) {
        int z, m0, n0;
        decode(t, z, m0, n0);
        for (int kb = 0; kb < p.n_kblocks; ++kb, ++it) {
          const int st = it % C::STAGES;
          const uint32_t rnd = static_cast<uint32_t>(it / C::STAGES);
          if (!(ok = mbar_wait(bar(C::B_EMPTY + st), (rnd & 1u) ^ 1u, ctl))) break;
          const uint32_t sa = base + st * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
          mbar_arrive_expect_tx(bar(C::B_FULL + st), C::STAGE_BYTES);
          if (!A_MN) {
            tma_load_3d(sa, &tm_a, bar(C::B_FULL + st), kb * C::BK, m0, z);
          } else {
            tma_load_3d(sa, &tm_a, bar(C::B_FULL + st), m0, kb * C::BK, z);
            tma_load_3d(sa + 8192, &tm_a, bar(C::B_FULL + st), m0 + 64, kb * C::BK, z);
          }
          if (!B_MN) {
            tma_load_3d(sb, &tm_b, bar(C::B_FULL + st), kb * C::BK, n0, z);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_3d(sb + c * 8192, &tm_b, bar(C::B_FULL + st), n0 + 64 * c, kb * C::BK, z);
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
    // ------------------------------------------------------------------ MMA issuer
    // Warp-uniform control flow, one elected lane issues (the *_w helpers).  Accumulator b of
    // tile i alternates so tile i+1's MMAs overlap tile i's epilogue.
    constexpr uint32_t kIdesc = idesc_f16(128, BN, BF16 ? 1 : 0, A_MN ? 1 : 0, B_MN ? 1 : 0);
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x, i = 0; ok && t < p.n_tiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      if (!(ok = mbar_wait_all(bar(C::B_ACCE + b), (static_cast<uint32_t>(i >> 1) & 1u) ^ 1u, ctl))) break;
      tc_fence_after_sync();
      const uint32_t d_tmem = tmem + b * BN;
      for (int kb = 0; kb < p.n_kblocks; ++kb, ++it) {
        const int st = it % C::STAGES;
        if (!(ok = mbar_wait_all(bar(C::B_FULL + st), static_cast<uint32_t>(it / C::STAGES) & 1u, ctl))) break;
        tc_fence_after_sync();
        const uint32_t sa = base + st * C::STAGE_BYTES;
        const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t da = A_MN ? smem_desc_sw128(sa + k * 2048, 8192, 1024)
                                   : smem_desc_sw128(sa + k * 32, 16, 1024);
          const uint64_t db = B_MN ? smem_desc_sw128(sb + k * 2048, 8192, 1024)
                                   : smem_desc_sw128(sb + k * 32, 16, 1024);
          umma_ss_w(d_tmem, da, db, kIdesc, (kb > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit_w(bar(C::B_EMPTY + st));
      }
      if (ok) umma_commit_w(bar(C::B_ACCF + b));
    }
  } else if (warp < 2 + C::EPI_WARPS) {
    // ------------------------------------------------------------------ epilogue (warps 2..9)
    // Warp w reads TMEM lane quarter w % 4 (rows quarter*32 ..) and the 64-column chunks
    // c = half, half + 2, ... of each tile; each (quarter, chunk) has its own staging slot, stored
    // with one TMA store (clipped at M and N).  Two staging buffers alternate by tile, so writing
    // tile i's rows only waits for tile i-2's stores to have read theirs.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    bool ok = true;
    bool stored = false;  // (ONE_SLOT) this warp has a store in flight that may still read its slot
    for (int t = blockIdx.x, i = 0; ok && t < p.n_tiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      int z, m0, n0;
      decode(t, z, m0, n0);
      if (!(ok = mbar_wait_all(bar(C::B_ACCF + b), static_cast<uint32_t>(i >> 1) & 1u, ctl))) break;
      tc_fence_after_sync();
      if constexpr (C::ONE_SLOT) {
        const uint32_t slot = base + C::OFF_STAGING + (warp - 2) * C::SLOT_BYTES;
        const int r0 = m0 + quarter * 32;
#pragma unroll 1
        for (int c = half; c < C::CHUNKS; c += 2) {
          uint32_t acc[2][32];
          tmem_ld32(t_lane + b * BN + c * 64, acc[0]);
          tmem_ld32(t_lane + b * BN + c * 64 + 32, acc[1]);
          if (p.bias) {
            add_bias32<BF16>(acc[0], p.bias, n0 + c * 64, p.n);
            add_bias32<BF16>(acc[1], p.bias, n0 + c * 64 + 32, p.n);
          }
          if (c + 2 >= C::CHUNKS) {
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(C::B_ACCE + b));  // accumulator b read
          }
          if (stored) {  // the slot's previous chunk must have been read by its store
            if (lane == 0) bulk_wait_group_read0();
            __syncwarp();
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float lo = __uint_as_float(acc[q >> 2][(q & 3) * 8 + 2 * e]);
              const float hi = __uint_as_float(acc[q >> 2][(q & 3) * 8 + 2 * e + 1]);
              w[e] = BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
            }
            st_shared_v4(slot + lane * 128 + ((q ^ (lane & 7)) << 4), w[0], w[1], w[2], w[3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (r0 < p.m && n0 + 64 * c < p.n) tma_store_3d(&tm_c, slot, n0 + 64 * c, r0, z);
            bulk_commit_group();
          }
          __syncwarp();
          stored = true;
        }
        continue;
      }
      const uint32_t staging = base + C::OFF_STAGING + b * C::STAGING_BYTES;
      if (i > 1) {  // this buffer's slots: tile i-2's stores (one group per tile) must have read them
        if (lane == 0) bulk_wait_group_read1();
        __syncwarp();
        // ... and (STATS) tile i-2's statistics warp
        if (STATS && !(ok = mbar_wait_all(bar(C::B_SFREE + b * 8 + (warp - 2)),
                                          static_cast<uint32_t>((i >> 1) - 1) & 1u, ctl)))
          break;
      }
#pragma unroll 1
      for (int c = half; c < C::CHUNKS; c += 2) {
        const uint32_t slot = staging + (quarter * C::CHUNKS + c) * C::SLOT_BYTES;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t acc[32];
          tmem_ld32(t_lane + b * BN + c * 64 + hh * 32, acc);
          if (p.bias) add_bias32<BF16>(acc, p.bias, n0 + c * 64 + hh * 32, p.n);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float lo = __uint_as_float(acc[q * 8 + 2 * e]);
              const float hi = __uint_as_float(acc[q * 8 + 2 * e + 1]);
              w[e] = BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
            }
            const int chunk = hh * 4 + q;  // 16-byte chunk within the 128-byte row
            st_shared_v4(slot + lane * 128 + ((chunk ^ (lane & 7)) << 4), w[0], w[1], w[2], w[3]);
          }
        }
      }
      if (STATS) {  // the staged rows are complete: the statistics warp may read them
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(C::B_SFULL + b * 8 + (warp - 2)));
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C::B_ACCE + b));  // accumulator b read: tile i+2 may reuse it
      fence_proxy_async_smem();
      __syncwarp();
      const int r0 = m0 + quarter * 32;
      if (lane == 0) {
        if (r0 < p.m) {
          for (int c = half; c < C::CHUNKS; c += 2)
            if (n0 + 64 * c < p.n)
              tma_store_3d(&tm_c, staging + (quarter * C::CHUNKS + c) * C::SLOT_BYTES, n0 + 64 * c, r0, z);
        }
        bulk_commit_group();
      }
      __syncwarp();
    }
    if (lane == 0) bulk_wait_group0();  // every store of this warp complete before exit
  } else if (STATS) {
    // ------------------------------------------------------------------ row statistics (10..17)
    // Warp 10 + e reads the staging slots epilogue warp 2 + e wrote (same rows, same chunks) and
    // writes, per row and 64-column run, (max, sum of exp) of the stored 16-bit values.
    static_assert(!STATS || !C::ONE_SLOT, "row statistics with the two-buffer staging only");
    const int e = warp - 10;
    const int quarter = warp & 3;
    const int half = e >> 2;
    bool ok = true;
    for (int t = blockIdx.x, i = 0; ok && t < p.n_tiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      int z, m0, n0;
      decode(t, z, m0, n0);
      if (!(ok = mbar_wait_all(bar(C::B_SFULL + b * 8 + e), static_cast<uint32_t>(i >> 1) & 1u, ctl))) break;
      const uint32_t staging = base + C::OFF_STAGING + b * C::STAGING_BYTES;
      const int r = m0 + quarter * 32 + lane;
      for (int c = half; c < C::CHUNKS; c += 2) {
        const uint32_t row_addr = staging + (quarter * C::CHUNKS + c) * C::SLOT_BYTES + lane * 128;
        float cm = -INFINITY, cs = 0.f;
        uint32_t w[32];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          ld_shared_v4(row_addr + ((q ^ (lane & 7)) << 4), w[q * 4], w[q * 4 + 1], w[q * 4 + 2], w[q * 4 + 3]);
        rowstats64<BF16>(w, n0 + c * 64, p.n, cm, cs);
        const int run = (n0 >> 6) + c;
        if (r < p.m && run < p.stats_runs)
          p.stats[(static_cast<size_t>(z) * p.stats_runs + run) * p.m + r] = make_float2(cm, cs);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C::B_SFREE + b * 8 + e));
    }
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

inline bool s16(int64_t s) { return s > 0 && ((s * 2) % 16) == 0 && (s * 2) < (1ll << 40); }

// Tile width: 256 for compute-bound shapes (wide N, K >= 512), where the operand traffic through
// shared memory sets the pace -- per 128-row MMA step a 128x256 tile moves 24 KB (TMA writes +
// MMA reads) per 128 clk of tensor work against 16 KB per 64 clk for 128x128, so it can run the
// pipe at ~2/3 instead of ~1/2 of its rate on a ~128 B/clk shared-memory port; 128 or 64 otherwise
// (short K: an output-write stream, where the 128-wide tile's double staging keeps stores going).
int pick_bn(int64_t n, int64_t k) { return (n > 128 && k >= 512) ? 256 : n > 64 ? 128 : 64; }

// Name of one tile-table entry (static storage, built once).
const char* bmm_table_name(bool bf16, int bn, int am, int bm) {
  static const std::array<std::string, 24> names = [] {
    std::array<std::string, 24> out;
    const int bns[3] = {64, 128, 256};
    for (int t = 0; t < 2; ++t)
      for (int i = 0; i < 3; ++i)
        for (int a = 0; a < 2; ++a)
          for (int b = 0; b < 2; ++b)
            out[((t * 3 + i) * 2 + a) * 2 + b] =
                std::string("bmm_sm100<") + (t ? "bf16" : "f16") + ",128x" + std::to_string(bns[i]) +
                "x64,A:" + (a ? "mn" : "k") + "-major,B:" + (b ? "mn" : "k") + "-major," +
                std::to_string(bns[i] == 64 ? 6 : 4) + "st,persistent>";
    return out;
  }();
  const int i = bn == 256 ? 2 : bn == 128 ? 1 : 0;
  return names[(((bf16 ? 1 : 0) * 3 + i) * 2 + am) * 2 + bm].c_str();
}

// Layout of one operand: 0 = K-major (contiguous along K), 1 = MN-major, -1 = unusable.
int a_major(const cmpx_bmm_desc* d) {
  if (d->a_stride[2] == 1 && (d->m == 1 || s16(d->a_stride[1])) ) return 0;
  if (d->a_stride[1] == 1 && (d->k == 1 || s16(d->a_stride[2]))) return 1;
  return -1;
}
int b_major(const cmpx_bmm_desc* d) {
  if (d->b_stride[1] == 1 && (d->n == 1 || s16(d->b_stride[2]))) return 0;  // contiguous along K
  if (d->b_stride[2] == 1 && (d->k == 1 || s16(d->b_stride[1]))) return 1;  // contiguous along N
  return -1;
}

}  // namespace

const char* bmm_sm100_plan(const cmpx_bmm_desc* d, int* status) {
  *status = CMPX_OK;
  if (d->dtype != CMPX_F16 && d->dtype != CMPX_BF16) {
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
  const int am = a_major(d), bmj = b_major(d);
  const bool c_ok = d->c_stride[2] == 1 && (d->m == 1 || s16(d->c_stride[1]));
  const bool batch_ok = d->batch == 1 || (s16(d->a_stride[0]) && s16(d->b_stride[0]) && s16(d->c_stride[0]));
  if (am < 0 || bmj < 0 || !c_ok || !batch_ok) {
    *status = CMPX_ERR_MISALIGNED;
    return "none";
  }
  return bmm_table_name(d->dtype == CMPX_BF16, pick_bn(d->n, d->k), am, bmj);
}

namespace {

template <int BN, bool A_MN, bool B_MN, bool BF16, bool STATS = false>
int launch_bmm_typed(const cmpx_bmm_desc* d, const LaunchCtx& ctx, const void* bias, float2* stats = nullptr) {
  using C = BmmCfg<BN>;
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t M = d->m, N = d->n, K = d->k, Z = d->batch;
  CUtensorMap ta, tb, tc;
  {
    const uint64_t dims[3] = {A_MN ? M : K, A_MN ? K : M, Z};
    const uint64_t st[2] = {static_cast<uint64_t>(A_MN ? d->a_stride[2] : d->a_stride[1]) * 2,
                            static_cast<uint64_t>(d->a_stride[0]) * 2};
    const uint32_t box[3] = {64, A_MN ? 64u : 128u, 1};
    if (!encode_tmap(&ta, dt, 3, d->a, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B)) return CMPX_ERR_LAUNCH;
  }
  {
    const uint64_t dims[3] = {B_MN ? N : K, B_MN ? K : N, Z};
    const uint64_t st[2] = {static_cast<uint64_t>(B_MN ? d->b_stride[1] : d->b_stride[2]) * 2,
                            static_cast<uint64_t>(d->b_stride[0]) * 2};
    const uint32_t box[3] = {64, B_MN ? 64u : static_cast<uint32_t>(BN), 1};
    if (!encode_tmap(&tb, dt, 3, d->b, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B)) return CMPX_ERR_LAUNCH;
  }
  {
    const uint64_t dims[3] = {N, M, Z};
    const uint64_t st[2] = {static_cast<uint64_t>(d->c_stride[1]) * 2,
                            static_cast<uint64_t>(d->c_stride[0]) * 2};
    const uint32_t box[3] = {64, 32, 1};
    if (!encode_tmap(&tc, dt, 3, d->c, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B)) return CMPX_ERR_LAUNCH;
  }
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(
        reinterpret_cast<const void*>(&bmm_sm100_kernel<BN, A_MN, B_MN, BF16, STATS>),
        cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return CMPX_ERR_LAUNCH;
  BmmParams p;
  p.m = static_cast<int>(M);
  p.n = static_cast<int>(N);
  p.k = static_cast<int>(K);
  p.n_kblocks = static_cast<int>((K + C::BK - 1) / C::BK);
  p.tiles_m = static_cast<int>((M + C::BM - 1) / C::BM);
  p.tiles_n = static_cast<int>((N + BN - 1) / BN);
  const int64_t n_tiles = static_cast<int64_t>(p.tiles_m) * p.tiles_n * static_cast<int64_t>(Z);
  if (n_tiles > (1ll << 31) - 1) return CMPX_ERR_UNSUPPORTED_SHAPE;
  p.n_tiles = static_cast<int>(n_tiles);
  p.timeout_ns = ctx.timeout_ns;
  p.dev_flags = ctx.dev_flags;
  p.bias = static_cast<const uint16_t*>(bias);
  p.stats = stats;
  p.stats_runs = static_cast<int>((N + 63) / 64);
  const int grid = static_cast<int>(std::min<int64_t>(n_tiles, std::max(1, ctx.num_sms)));
  bmm_sm100_kernel<BN, A_MN, B_MN, BF16, STATS>
      <<<grid, STATS ? C::STATS_THREADS : C::THREADS, C::SMEM_BYTES, ctx.stream>>>(ta, tb, tc, p);
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

template <int BN, bool BF16>
int launch_bmm_bn(const cmpx_bmm_desc* d, const LaunchCtx& ctx, int am, int bm, const void* bias) {
  if (am == 0 && bm == 0) return launch_bmm_typed<BN, false, false, BF16>(d, ctx, bias);
  if (am == 0 && bm == 1) return launch_bmm_typed<BN, false, true, BF16>(d, ctx, bias);
  if (am == 1 && bm == 0) return launch_bmm_typed<BN, true, false, BF16>(d, ctx, bias);
  return launch_bmm_typed<BN, true, true, BF16>(d, ctx, bias);
}

template <bool BF16>
int launch_bmm_dt(const cmpx_bmm_desc* d, const LaunchCtx& ctx, int am, int bm, const void* bias) {
  const int bn = pick_bn(d->n, d->k);
  if (bn == 256) return launch_bmm_bn<256, BF16>(d, ctx, am, bm, bias);
  if (bn == 128) return launch_bmm_bn<128, BF16>(d, ctx, am, bm, bias);
  return launch_bmm_bn<64, BF16>(d, ctx, am, bm, bias);
}

}  // namespace

// The product with its row statistics (rowstats.cuh): the 128-column tile, both operands K-major
// (the attention-score product Q K^T of a head dim <= 128 is this case), stats float2
// [batch][ceil(n / 64)][m].
const char* bmm_rowstats_plan(const cmpx_bmm_desc* d, const void* stats, int* status) {
  bmm_sm100_plan(d, status);
  if (*status != CMPX_OK) return "none";
  if (a_major(d) != 0 || b_major(d) != 0) {
    *status = CMPX_ERR_MISALIGNED;
    return "none";
  }
  if (!stats || (reinterpret_cast<uintptr_t>(stats) & 7u) != 0 ||
      d->batch * ((d->n + 63) / 64) * d->m > (1ll << 40)) {
    *status = CMPX_ERR_INVALID_ARGUMENT;
    return "none";
  }
  return d->dtype == CMPX_BF16 ? "bmm_sm100<bf16,128x128x64,A:k-major,B:k-major,4st,persistent,rowstats>"
                               : "bmm_sm100<f16,128x128x64,A:k-major,B:k-major,4st,persistent,rowstats>";
}

int launch_bmm_rowstats(const cmpx_bmm_desc* d, float* stats, const LaunchCtx& ctx) {
  int st = CMPX_OK;
  bmm_rowstats_plan(d, stats, &st);
  if (st != CMPX_OK) return st;
  if (d->m == 0 || d->n == 0 || d->batch == 0) return CMPX_OK;
  float2* s2 = reinterpret_cast<float2*>(stats);
  return d->dtype == CMPX_BF16 ? launch_bmm_typed<128, false, false, true, true>(d, ctx, nullptr, s2)
                               : launch_bmm_typed<128, false, false, false, true>(d, ctx, nullptr, s2);
}

// The GEMM a linear layer is: x [m, k] (rows ld_x apart) times W^T, W [n, k] (rows ld_w apart) --
// a K-major B operand read in place -- into y [m, n].
cmpx_bmm_desc linear_as_bmm(const cmpx_linear_desc* d) {
  cmpx_bmm_desc b{};
  b.a = d->x;
  b.b = d->w;
  b.c = d->y;
  b.batch = 1;
  b.m = d->m;
  b.n = d->n;
  b.k = d->k;
  b.a_stride[0] = d->m * d->x_row_stride;
  b.a_stride[1] = d->x_row_stride;
  b.a_stride[2] = 1;
  b.b_stride[0] = d->n * d->w_row_stride;
  b.b_stride[1] = 1;                // along K
  b.b_stride[2] = d->w_row_stride;  // along N
  b.c_stride[0] = d->m * d->y_row_stride;
  b.c_stride[1] = d->y_row_stride;
  b.c_stride[2] = 1;
  b.dtype = d->dtype;
  return b;
}

int launch_bmm_sm100(const cmpx_bmm_desc* d, const LaunchCtx& ctx) {
  int st = CMPX_OK;
  bmm_sm100_plan(d, &st);
  if (st != CMPX_OK) return st;
  if (d->m == 0 || d->n == 0 || d->batch == 0) return CMPX_OK;
  const int am = a_major(d), bm = b_major(d);
  return d->dtype == CMPX_BF16 ? launch_bmm_dt<true>(d, ctx, am, bm, nullptr)
                               : launch_bmm_dt<false>(d, ctx, am, bm, nullptr);
}

const char* linear_sm100_plan(const cmpx_linear_desc* d, int* status) {
  *status = CMPX_OK;
  if (d->m < 0 || d->n < 1 || d->k < 1 || d->x_row_stride < d->k || d->w_row_stride < d->k ||
      d->y_row_stride < d->n) {
    *status = CMPX_ERR_INVALID_ARGUMENT;
    return "none";
  }
  if (d->bias && (reinterpret_cast<uintptr_t>(d->bias) & 15u) != 0) {
    *status = CMPX_ERR_MISALIGNED;
    return "none";
  }
  const cmpx_bmm_desc b = linear_as_bmm(d);
  return bmm_sm100_plan(&b, status);
}

int launch_linear_sm100(const cmpx_linear_desc* d, const LaunchCtx& ctx) {
  int st = CMPX_OK;
  linear_sm100_plan(d, &st);
  if (st != CMPX_OK) return st;
  if (d->m == 0) return CMPX_OK;
  const cmpx_bmm_desc b = linear_as_bmm(d);
  const int am = a_major(&b), bm = b_major(&b);
  return d->dtype == CMPX_BF16 ? launch_bmm_dt<true>(&b, ctx, am, bm, d->bias)
                               : launch_bmm_dt<false>(&b, ctx, am, bm, d->bias);
}

}  // namespace cmpx
