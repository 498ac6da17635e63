// softmax_product_sm100.cu -- softmax over the last dimension of a 16-bit batched product,
// Y = softmax(A B) with A [batch, m, k] and B [batch, k, n] both K-major, computed from A, B and the
// product's row statistics (B200 sm_100a).
//
// The einsum-attention chain (cmpext3/einsum_ops.py:69-121 in the reference: scores einsum ->
// softmax -> values einsum, with the softmax left to stock, cmpext3/__init__.py:130-138) writes the
// [batch, m, n] score tensor S = A B and then reads it back for the softmax.  Here the scores
// product (bmm_sm100.cu with its row-statistics warps) also writes, per row and 64-column run, the
// run's max and sum of exp over the stored scores (rowstats.cuh), and this kernel never reads S: it
// recomputes each 128 x 128 chunk of it on the tensor cores, with the same instruction shape and
// the same K order as the bmm kernel (128-row tiles, K=16 steps in order, fp32 accumulation), rounds
// it to the 16-bit type exactly as that kernel's epilogue does -- so the values it takes the
// softmax of are the values of S, bit for bit -- and writes p = 2^(s log2e - max log2e - log2 sum)
// in one pass, one exponential per element.
//
//   * a CTA owns a 128-row block of one batch item at a time (persistent, items strided over the
//     grid, consecutive CTAs on the same batch item so B is shared in L2);
//   * warp 0: TMA of the A block (once per item) and of B in 128-column chunks through a ring;
//   * warp 1: S chunks (tcgen05, M = N = 128, K = 16 steps) into four TMEM buffers of 128 columns,
//     one per softmax warpgroup; chunk i of the whole sequence goes to warpgroup i % 4;
//   * warps 2-17 (four warpgroups, thread = row): each warpgroup folds every fourth run of the
//     row's statistics, the four partials are combined through shared memory, then each writes
//     its chunks of p, rounded to the 16-bit type, through per-warp staging boxes and TMA stores
//     (clipped at m, n).
//
// Every wait is bounded (cmpx_ptx.cuh); a CTA that gives up drains its copies and MMAs, frees
// TMEM, raises the device status word and returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "cmpx_internal.h"
#include "cmpx_ptx.cuh"
#include "rowstats.cuh"

namespace cmpx {

template <int KD>
struct SpCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr int NWG = 4;                     // softmax warpgroups
  static constexpr int NBUF = 4 / NWG;              // TMEM chunk buffers (128 columns) per warpgroup
  static constexpr int KCH = KD / 64;               // 64-element (128-byte) chunks of k
  static constexpr int CH_BYTES = 128 * 128;        // one chunk of 128 rows
  static constexpr int T_BYTES = KCH * CH_BYTES;    // an A block or a B chunk
  static constexpr int NB = KD == 64 ? 4 : 3;       // B ring stages
  static constexpr int NSTG = KD == 64 ? 2 : 1;     // staging boxes per softmax warp
  static constexpr int STG_BYTES = 32 * 128;        // one box: 32 rows x 64 16-bit columns
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + T_BYTES;
  static constexpr int OFF_STG = OFF_B + NB * T_BYTES;                    // [4 NWG warps][NSTG]
  static constexpr int OFF_STATS = OFF_STG + 4 * NWG * NSTG * STG_BYTES;  // [2 items][NWG][128] float2
  static constexpr int OFF_BAR = OFF_STATS + 2 * NWG * 128 * 8;
  static constexpr int B_AFULL = 0, B_AEMPTY = 1;
  static constexpr int B_BFULL = 2, B_BEMPTY = B_BFULL + NB;  // [NB] each
  static constexpr int B_SFULL = B_BEMPTY + NB;               // [4] warpgroup * NBUF + slot
  static constexpr int B_SFREE = B_SFULL + 4;                 // [4] count 128
  static constexpr int B_STATS = B_SFREE + 4;                 // count NWG * 128: every warpgroup's partial written
  static constexpr int B_DRAIN = B_STATS + 1;
  static constexpr int NBAR = B_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int THREADS = 64 + NWG * 128;
  static_assert(SMEM_BYTES <= 232448, "shared memory");
  static_assert(NWG * NBUF * 128 == TMEM_COLS, "TMEM buffers");
};

struct SpParams {
  int m, n, k;
  int tiles_m, n_items, nc;  // 128-row blocks per batch item, items, 128-column chunks per row
  int runs;                  // 64-column runs of the row statistics: ceil(n / 64)
  const float2* stats;       // [batch][runs][m]
  unsigned long long timeout_ns;
  unsigned int* dev_flags;
};

template <int KD, bool BF16>
__global__ void __launch_bounds__(64 + 4 * 128, 1)
    softmax_product_sm100_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                                 const __grid_constant__ CUtensorMap tm_y, const SpParams p) {
  using C = SpCfg<KD>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto bar = [&](int i) -> uint32_t { return base + C::OFF_BAR + 8u * i; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  float2* stats = reinterpret_cast<float2*>(smem + C::OFF_STATS);
  const int n_chunks = p.nc;

  if (threadIdx.x == 0) {
    mbar_init(bar(C::B_AFULL), 1);
    mbar_init(bar(C::B_AEMPTY), 1);
    for (int s = 0; s < C::NB; ++s) {
      mbar_init(bar(C::B_BFULL + s), 1);
      mbar_init(bar(C::B_BEMPTY + s), 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(bar(C::B_SFULL + i), 1);
      mbar_init(bar(C::B_SFREE + i), 128);
    }
    mbar_init(bar(C::B_STATS), C::NWG * 128);
    mbar_init(bar(C::B_DRAIN), 1);
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
    tma_prefetch_desc(&tm_y);
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const WaitCtl ctl{abort_flag, p.dev_flags, p.timeout_ns};

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0, items = 0;
      bool ok = true;
      for (int w = blockIdx.x, k = 0; ok && w < p.n_items; w += gridDim.x, ++k) {
        const int z = w / p.tiles_m, m0 = (w - z * p.tiles_m) * C::BM;
        // the A block is free once every product of the previous item is done
        if (k > 0 && !(ok = mbar_wait(bar(C::B_AEMPTY), static_cast<uint32_t>(k - 1) & 1u, ctl))) break;
        mbar_arrive_expect_tx(bar(C::B_AFULL), C::T_BYTES);
        for (int c = 0; c < C::KCH; ++c)
          tma_load_3d(base + C::OFF_A + c * C::CH_BYTES, &tm_a, bar(C::B_AFULL), c * 64, m0, z);
        ++items;
        for (int g = 0; g < n_chunks; ++g, ++it) {
          const int st = it % C::NB;
          if (!(ok = mbar_wait(bar(C::B_BEMPTY + st), (static_cast<uint32_t>(it / C::NB) & 1u) ^ 1u, ctl))) break;
          mbar_arrive_expect_tx(bar(C::B_BFULL + st), C::T_BYTES);
          for (int c = 0; c < C::KCH; ++c)
            tma_load_3d(base + C::OFF_B + st * C::T_BYTES + c * C::CH_BYTES, &tm_b, bar(C::B_BFULL + st), c * 64,
                        g * C::BN, z);
        }
      }
      if (*abort_flag) {  // let the copies in flight land before the CTA gives its memory back
        if (items > 0) mbar_wait_drain(bar(C::B_AFULL), static_cast<uint32_t>(items - 1) & 1u, p.timeout_ns);
        for (int i = max(0, it - C::NB); i < it; ++i)
          mbar_wait_drain(bar(C::B_BFULL + i % C::NB), static_cast<uint32_t>(i / C::NB) & 1u, p.timeout_ns);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (warp-uniform)
    // The same products as the bmm kernel's 128-row tiles: K=16 steps in k order, fp32 in TMEM.
    constexpr uint32_t kIdesc = idesc_f16(128, 128, BF16 ? 1 : 0, 0, 0);
    int it = 0;  // chunk counter over all items: chunk it goes to warpgroup it % NWG
    bool ok = true;
    for (int w = blockIdx.x, k = 0; ok && w < p.n_items; w += gridDim.x, ++k) {
      if (!(ok = mbar_wait_all(bar(C::B_AFULL), static_cast<uint32_t>(k) & 1u, ctl))) break;
      for (int g = 0; g < n_chunks; ++g, ++it) {
        const int wg = it % C::NWG, uw = it / C::NWG, buf = wg * C::NBUF + uw % C::NBUF;
        // the buffer's previous chunk must have been read by its warpgroup
        if (uw >= C::NBUF &&
            !(ok = mbar_wait_all(bar(C::B_SFREE + buf), static_cast<uint32_t>(uw / C::NBUF - 1) & 1u, ctl)))
          break;
        const int st = it % C::NB;
        if (!(ok = mbar_wait_all(bar(C::B_BFULL + st), static_cast<uint32_t>(it / C::NB) & 1u, ctl))) break;
        tc_fence_after_sync();
        const uint32_t sa = base + C::OFF_A, sb = base + C::OFF_B + st * C::T_BYTES;
#pragma unroll
        for (int s = 0; s < KD / 16; ++s) {
          const uint32_t off = (s >> 2) * C::CH_BYTES + (s & 3) * 32;
          umma_ss_w(tmem + buf * 128, smem_desc_sw128(sa + off, 16, 1024), smem_desc_sw128(sb + off, 16, 1024),
                    kIdesc, s > 0 ? 1u : 0u);
        }
        umma_commit_w(bar(C::B_SFULL + buf));
        umma_commit_w(bar(C::B_BEMPTY + st));
      }
      if (ok) umma_commit_w(bar(C::B_AEMPTY));  // every product reading this item's A block
    }
  } else {
    // ------------------------------------------------------------------ softmax / stores (2..17)
    const int sw = warp - 2;         // softmax warp
    const int wg = sw >> 2;          // warpgroup: chunk it of the whole sequence when it % NWG == wg
    const int quarter = warp & 3;    // TMEM lane quarter of this warp
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t stg0 = base + C::OFF_STG + sw * C::NSTG * C::STG_BYTES;
    int used = 0, boxes = 0;
    int rot = 0;  // (k * n_chunks) % NWG: the warpgroup of the item's chunk 0
    bool ok = true;
    for (int w = blockIdx.x, k = 0; ok && w < p.n_items; w += gridDim.x, ++k) {
      const int z = w / p.tiles_m, m0 = (w - z * p.tiles_m) * C::BM;
      const int row0 = m0 + quarter * 32;  // first row of this warp's stores
      // This warpgroup's share of the row's statistics: runs wg, wg + NWG, ...
      float pm = -INFINITY, ps = 0.f;
      if (m0 + row < p.m) {
        const float2* sp = p.stats + static_cast<size_t>(z) * p.runs * p.m + (m0 + row);
        int j = wg;
        for (; j + 3 * C::NWG < p.runs; j += 4 * C::NWG) {
          float2 v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) v[u] = __ldg(sp + static_cast<size_t>(j + u * C::NWG) * p.m);
#pragma unroll
          for (int u = 0; u < 4; ++u) rowstats_merge(pm, ps, v[u].x, v[u].y);
        }
        for (; j < p.runs; j += C::NWG) {
          const float2 v = __ldg(sp + static_cast<size_t>(j) * p.m);
          rowstats_merge(pm, ps, v.x, v.y);
        }
      }
      // Combine the four partials through shared memory.  Every warpgroup arrives once per item
      // and waits (so that none can arrive for the next item while this item's phase is still
      // open); the buffers alternate by item.
      stats[((k & 1) * C::NWG + wg) * 128 + row] = make_float2(pm, ps);
      mbar_arrive(bar(C::B_STATS));
      if (!(ok = mbar_wait_all(bar(C::B_STATS), static_cast<uint32_t>(k) & 1u, ctl))) break;
      uint64_t l2e2, off2;  // p = 2^(v * log2e + off)
      {
        float m_all = -INFINITY, l = 0.f;
#pragma unroll
        for (int j = 0; j < C::NWG; ++j) {
          const float2 v = stats[((k & 1) * C::NWG + j) * 128 + row];
          rowstats_merge(m_all, l, v.x, v.y);
        }
        // off = -max log2e - log2 sum; a row of -inf only gives -inf * log2e - (-inf) = NaN, as
        // torch's softmax does
        const float off = -m_all * kRowLog2e - __log2f(l);
        l2e2 = f2_pack(kRowLog2e, kRowLog2e);
        off2 = f2_pack(off, off);
      }
      const int g0 = ((wg - rot) % C::NWG + C::NWG) % C::NWG;  // this warpgroup's first chunk of the item
      rot = (rot + n_chunks) % C::NWG;
      for (int g = g0; ok && g < n_chunks; g += C::NWG) {
        const int n0 = g * C::BN;
        const int buf = wg * C::NBUF + used % C::NBUF;
        if (!(ok = mbar_wait_all(bar(C::B_SFULL + buf), static_cast<uint32_t>(used / C::NBUF) & 1u, ctl))) break;
        tc_fence_after_sync();
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // 32 columns at a time
          uint32_t r[32];
          tmem_ld32(lane_base + buf * 128 + q * 32, r);
          if (q == 3) {
            tc_fence_before_sync();
            mbar_arrive(bar(C::B_SFREE + buf));  // the chunk is in registers: the buffer may be reused
          }
          // round to the 16-bit type (what the bmm epilogue stores), then p; columns >= n are
          // clipped by the store
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const uint32_t s16 = pack16<BF16>(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
            pk[e] = pack16x2<BF16>(ex2x2(f2_fma(unpack16x2<BF16>(s16), l2e2, off2)));
          }
          // 32 16-bit columns into the half of the staging box they belong to (128-byte
          // swizzle: row lane at lane * 128, 16-byte unit u at (u ^ (lane & 7)) * 16)
          const uint32_t box = stg0 + (boxes % C::NSTG) * C::STG_BYTES;
          if ((q & 1) == 0 && boxes >= C::NSTG) {  // the box's previous store must have read it
            if (lane == 0) {
              if (C::NSTG == 2)
                bulk_wait_group_read1();
              else
                bulk_wait_group_read0();
            }
            __syncwarp();
          }
          const uint32_t row_addr = box + lane * 128;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int unit = (q & 1) * 4 + u;
            st_shared_v4(row_addr + ((unit ^ (lane & 7)) << 4), pk[4 * u], pk[4 * u + 1], pk[4 * u + 2],
                         pk[4 * u + 3]);
          }
          if (q & 1) {  // the box is complete: store 32 rows x 64 columns (clipped at m, n)
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              const int c0 = n0 + (q >> 1) * 64;
              if (row0 < p.m && c0 < p.n) tma_store_3d(&tm_y, box, c0, row0, z);
              bulk_commit_group();
            }
            __syncwarp();
            ++boxes;
          }
        }
        ++used;
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

inline bool s16h(int64_t s) { return s > 0 && ((s * 2) % 16) == 0 && (s * 2) < (1ll << 40); }

}  // namespace

const char* softmax_product_plan(const cmpx_bmm_desc* d, const void* stats, const void* y, int* status) {
  *status = CMPX_OK;
  if (!d || d->batch < 0 || d->m < 0 || d->n < 0 || d->k < 0) {
    *status = CMPX_ERR_INVALID_ARGUMENT;
    return "none";
  }
  if (d->dtype != CMPX_F16 && d->dtype != CMPX_BF16) {
    *status = CMPX_ERR_UNSUPPORTED_DTYPE;
    return "none";
  }
  if (d->k < 1 || d->k > 128 || d->n < 1 || d->m > (int64_t)128 * 65535 || d->n > (1 << 30) ||
      d->batch > 65535) {
    *status = CMPX_ERR_UNSUPPORTED_SHAPE;
    return "none";
  }
  if (!d->a || !d->b || !y || !stats || (reinterpret_cast<uintptr_t>(stats) & 7u) != 0) {
    *status = CMPX_ERR_INVALID_ARGUMENT;
    return "none";
  }
  // A and B K-major (k contiguous, rows 16-byte aligned), Y rows contiguous and 16-byte aligned:
  // every stride that is stepped a multiple of 8 elements, pointers 16-byte aligned.
  const void* ptrs[3] = {d->a, d->b, y};
  for (const void* ptr : ptrs)
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) {
      *status = CMPX_ERR_MISALIGNED;
      return "none";
    }
  const bool a_ok = d->a_stride[2] == 1 && (d->m == 1 || s16h(d->a_stride[1]));
  const bool b_ok = d->b_stride[1] == 1 && (d->n == 1 || s16h(d->b_stride[2]));
  const bool y_ok = d->c_stride[2] == 1 && (d->m == 1 || s16h(d->c_stride[1]));
  const bool batch_ok = d->batch <= 1 || (s16h(d->a_stride[0]) && s16h(d->b_stride[0]) && s16h(d->c_stride[0]));
  if (!a_ok || !b_ok || !y_ok || !batch_ok) {
    *status = CMPX_ERR_MISALIGNED;
    return "none";
  }
  static const char* const names[2][2] = {
      {"softmax_product_sm100<f16,128x128,k64,rowstats>", "softmax_product_sm100<f16,128x128,k128,rowstats>"},
      {"softmax_product_sm100<bf16,128x128,k64,rowstats>", "softmax_product_sm100<bf16,128x128,k128,rowstats>"}};
  return names[d->dtype == CMPX_BF16 ? 1 : 0][d->k > 64 ? 1 : 0];
}

namespace {

template <int KD, bool BF16>
int launch_sp_typed(const cmpx_bmm_desc* d, const float* stats, void* y, const LaunchCtx& ctx) {
  using C = SpCfg<KD>;
  const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t M = d->m, N = d->n, K = d->k, Z = d->batch;
  CUtensorMap ta, tb, ty;
  {
    const uint64_t dims[3] = {K, M, Z};
    const uint64_t st[2] = {static_cast<uint64_t>(d->a_stride[1]) * 2, static_cast<uint64_t>(d->a_stride[0]) * 2};
    const uint32_t box[3] = {64, 128, 1};
    if (!encode_tmap(&ta, dt, 3, d->a, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B)) return CMPX_ERR_LAUNCH;
  }
  {
    const uint64_t dims[3] = {K, N, Z};
    const uint64_t st[2] = {static_cast<uint64_t>(d->b_stride[2]) * 2, static_cast<uint64_t>(d->b_stride[0]) * 2};
    const uint32_t box[3] = {64, 128, 1};
    if (!encode_tmap(&tb, dt, 3, d->b, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B)) return CMPX_ERR_LAUNCH;
  }
  {
    const uint64_t dims[3] = {N, M, Z};
    const uint64_t st[2] = {static_cast<uint64_t>(d->c_stride[1]) * 2, static_cast<uint64_t>(d->c_stride[0]) * 2};
    const uint32_t box[3] = {64, 32, 1};
    if (!encode_tmap(&ty, dt, 3, y, dims, st, box, CU_TENSOR_MAP_SWIZZLE_128B)) return CMPX_ERR_LAUNCH;
  }
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(reinterpret_cast<const void*>(&softmax_product_sm100_kernel<KD, BF16>),
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  });
  if (attr_err[dev & 63] != cudaSuccess) return CMPX_ERR_LAUNCH;
  SpParams p;
  p.m = static_cast<int>(M);
  p.n = static_cast<int>(N);
  p.k = static_cast<int>(K);
  p.tiles_m = static_cast<int>((M + C::BM - 1) / C::BM);
  const int64_t items = static_cast<int64_t>(p.tiles_m) * static_cast<int64_t>(Z);
  if (items > (1ll << 31) - 1) return CMPX_ERR_UNSUPPORTED_SHAPE;
  p.n_items = static_cast<int>(items);
  p.nc = static_cast<int>((N + C::BN - 1) / C::BN);
  p.runs = static_cast<int>((N + 63) / 64);
  p.stats = reinterpret_cast<const float2*>(stats);
  p.timeout_ns = ctx.timeout_ns;
  p.dev_flags = ctx.dev_flags;
  const int grid = static_cast<int>(std::min<int64_t>(items, std::max(1, ctx.num_sms)));
  softmax_product_sm100_kernel<KD, BF16><<<grid, C::THREADS, C::SMEM_BYTES, ctx.stream>>>(ta, tb, ty, p);
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

}  // namespace

int launch_softmax_product(const cmpx_bmm_desc* d, const float* stats, void* y, const LaunchCtx& ctx) {
  const bool bf = d->dtype == CMPX_BF16;
  if (d->k <= 64)
    return bf ? launch_sp_typed<64, true>(d, stats, y, ctx) : launch_sp_typed<64, false>(d, stats, y, ctx);
  return bf ? launch_sp_typed<128, true>(d, stats, y, ctx) : launch_sp_typed<128, false>(d, stats, y, ctx);
}

}  // namespace cmpx
