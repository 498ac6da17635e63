// attn_tf32x3_sm100.cu -- fp32 scaled-dot-product attention on the tensor cores (B200 sm_100a).
//
// The fp32 contract (1e-4 relative to stock fp32 SDPA) is out of reach of one TF32 product
// (10-bit mantissa: ~1e-3 per element), so every product here is split the 3xTF32 way: with
// x = x_hi + x_lo, x_hi the value truncated to TF32 (exactly representable) and x_lo = x - x_hi
// (exact in fp32), a b ~= a_hi b_hi + a_hi b_lo + a_lo b_hi, dropping only a_lo b_lo (~2^-22
// relative).  It replaces the reference's fp32 attention (attention_fp32_strict_kernel,
// src/cuda/fp32_attention.cu:35-198: one thread per query row on the CUDA cores) for every head dim
// of that kernel (D <= 128; SD1.5's fp32 attention has D = 40).
//
//   * a CTA owns a 128-row Q tile of one (batch, head) at a time (persistent, items strided over
//     the grid); keys stream in 64-key tiles (D <= 64) or 32-key tiles (D <= 128);
//   * K hi / lo and V^T hi / lo: made once per call by x3_kv_split_kernel into the workspace when
//     every (batch, head) has two or more Q tiles to share them, and then loaded by TMA as they
//     are; otherwise the converter warps make them per stage from raw K / V tiles;
//   * warp 0: TMA of Q (once per item, into a staging tile) and of the K / V operand tiles (fp32,
//     128-byte swizzle, OOB zero-filled) into a ring of stages;
//   * warps 2-5 ("converter", thread = row for Q): Q split into hi / lo and written to TMEM (the
//     QK products read A from TMEM); without the split operands also V transposed into V^T hi / lo
//     (the K-major B operand of P V) and K split in place into hi and lo;
//   * warps 1 and 10: tcgen05.mma kind::tf32 -- warp 1 issues S = Qh Kh^T + Qh Kl^T + Ql Kh^T into
//     one of two TMEM S buffers, warp 10 issues O += Ph Vh + Ph Vl + Pl Vh with P read from TMEM.
//     Two issuers on two SMSPs, each waiting only for its own inputs: one warp that polled the
//     inputs of both products and issued whichever was ready measured 348 us on C1 against 318
//     (its MMA issue, a few instructions per MMA on an SMSP shared with a softmax warp, left the
//     tensor pipe idle about half of each tile);
//   * warps 6-9 (thread = row): exact tile max, running max moved only when a tile's max exceeds
//     it by more than 2^64 (fp32 keeps p = 2^(x - m) exact far beyond that; O, l and P share m,
//     so the result is the same), p in fp32, split into Ph (written over the tile's own S buffer)
//     and Pl (one of two buffers); the epilogue writes O / l.  Tile j's S buffer is reused by tile
//     j+2 only after PV(j) is done, so storing P never waits for a PV;
//   * tail split (non-causal): when the last wave holds at most half a wave of Q tiles, those are
//     cut into key ranges whose (O, m, l) rows are parked in the workspace and merged by the CTA
//     of each tile's last range to finish.
//
// TMEM columns (D <= 64): S0 / Ph0 [0,64), S1 / Ph1 [64,128), Pl0 [128,192), Pl1 [192,256),
// O [256,320), Qh [320,384), Ql [384,448) (D <= 128: 32-column S / P buffers, 128-column O, Qh, Ql).
// Every wait is bounded (cmpx_ptx.cuh); a CTA that gives up drains its copies and MMAs, frees
// TMEM, raises the device status word and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "cmpx_internal.h"
#include "cmpx_ptx.cuh"

namespace cmpx {

// DP_ = padded head dim (64 or 128).  D = 128 halves the key tile to 32 keys so that Q hi / lo, O
// and the S / P buffers still fit TMEM's 512 columns, and runs a 2-stage ring (Q staging doubles).
template <int DP_>
struct X3Cfg {
  static constexpr int BM = 128, DP = DP_;          // query rows, padded head dim
  static constexpr int BN = DP == 64 ? 64 : 32;     // keys per tile
  static constexpr int NQC = DP / 32;               // 32-column (128-byte) chunks of the head dim
  static constexpr int QCH = BM * 128;              // one chunk of a Q tile
  static constexpr int Q_BYTES = NQC * QCH;         // staging tile: 32 KB (D 64) / 64 KB (D 128)
  static constexpr int KCH = BN * 128;              // one head-dim chunk of a K / V tile (BN rows)
  static constexpr int T_BYTES = NQC * KCH;         // 16 KB: a K, V, V^T hi or V^T lo tile
  static constexpr int VCH = DP * 128;              // one 32-key chunk of V^T (DP rows)
  static constexpr int NS = DP == 64 ? 3 : 2;       // K/V ring stages
  // stage slots: K (hi in place) | raw V, then K lo | V^T hi | V^T lo
  static constexpr int ST_K = 0, ST_B = T_BYTES, ST_VTH = 2 * T_BYTES, ST_VTL = 3 * T_BYTES;
  static constexpr int STAGE_BYTES = 4 * T_BYTES;   // 64 KB
  static constexpr int OFF_Q = 0, OFF_ST = Q_BYTES;
  static constexpr int OFF_BAR = OFF_ST + NS * STAGE_BYTES;
  static constexpr int B_QFULL = 0;                 // Q staging tile landed
  static constexpr int B_QFREE = 1;                 // converter has read it (count 128)
  static constexpr int B_QEMPTY = 2;                // last S product of the item done: TMEM Q free
  static constexpr int B_QCONV = 3;                 // Q hi / lo in TMEM (count 128)
  static constexpr int B_FULL = 4;                  // [NS]
  static constexpr int B_CONV = B_FULL + NS;        // [NS] count 128
  static constexpr int B_EMPTY = B_CONV + NS;       // [NS]
  static constexpr int B_SFULL = B_EMPTY + NS;      // [2] S buffer b holds its tile's scores
  static constexpr int B_PREADY = B_SFULL + 2;      // [2] P of buffer b written (count 128)
  static constexpr int B_PVD = B_PREADY + 2;        // [2] P V of buffer b's tile done
  static constexpr int B_OFREE = B_PVD + 2;         // count 128
  static constexpr int B_VREAD = B_OFREE + 1;      // converter threads have read a stage's raw V (128)
  static constexpr int B_EPI = B_VREAD + 1;         // tail split: the CTA's partial rows written (count 128)
  static constexpr int B_EPI2 = B_EPI + 1;          // tail split: the range's arrival counted
  static constexpr int B_DRAIN = B_EPI2 + 1;        // [2] the two MMA issuers' drains on abort
  static constexpr int NBAR = B_DRAIN + 2;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static_assert(SMEM_BYTES <= 232448, "shared memory");
  static constexpr int TM_S0 = 0, TM_S1 = BN, TM_PL0 = 2 * BN, TM_PL1 = 3 * BN, TM_O = 4 * BN,
                       TM_QH = 4 * BN + DP, TM_QL = 4 * BN + 2 * DP;
  static constexpr int TMEM_COLS = 512;
  static_assert(TM_QL + DP <= TMEM_COLS, "TMEM columns");
  static constexpr int THREADS = 352;
  static constexpr int W_TMA = 0, W_MMA = 1, W_PV = 10;
};

struct X3Params {
  int heads, len_q, len_k, head_dim;
  int n_qt, n_items;
  // Tail split (non-causal): work items 0 .. n_whole-1 are whole (128-row tile, head) items; each
  // of the last n_items - n_whole items is cut into `split` key ranges, one work item each
  // (n_work in all), whose partial (O, m, l) rows go to part and are merged by the CTA of the
  // item's last range to arrive (cnt: one 8-bit arrival counter per tail item, four to a word, in
  // the workspace's first 256 bytes, left at 0).
  int n_whole, split, n_work;
  unsigned int* cnt;
  float* part;
  // Split operands (pre = 1): K hi / lo and V^T hi / lo made once per call by x3_kv_split_kernel
  // (in the workspace) and loaded by TMA as they are, so the converter warps only split Q.
  int pre;
  int heads_kv;
  int qk_steps;   // ceil(head_dim / 8): K=8 steps of Q K^T
  int causal, neg_scale;
  int group;      // query heads per key/value head (grouped-query attention)
  float scale_log2;
  float* o;
  long long os_b, os_h, os_s;
  // Mask (MK = 1: one byte per element, nonzero = the key takes part; MK = 2: fp32 values added to
  // the scores as value / scale): element (b, h, i, j) at mask[b*mk_b + h*mk_h + i*mk_q + j]
  // (strides in elements, 0 = broadcast); rows start on 16-byte boundaries.
  const void* mask;
  long long mk_b, mk_h, mk_q;
  float mask_inv_scale;
  unsigned long long timeout_ns;
  unsigned int* dev_flags;
};

__device__ __forceinline__ uint32_t tf32_trunc(uint32_t bits) { return bits & 0xFFFFE000u; }

__device__ __forceinline__ void split_v4(uint32_t addr_in, uint32_t addr_hi, uint32_t addr_lo) {
  uint32_t a, b, c, d;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr_in));
  const uint32_t ha = tf32_trunc(a), hb = tf32_trunc(b), hc = tf32_trunc(c), hd = tf32_trunc(d);
  st_shared_v4(addr_hi, ha, hb, hc, hd);
  st_shared_v4(addr_lo, __float_as_uint(__uint_as_float(a) - __uint_as_float(ha)),
               __float_as_uint(__uint_as_float(b) - __uint_as_float(hb)),
               __float_as_uint(__uint_as_float(c) - __uint_as_float(hc)),
               __float_as_uint(__uint_as_float(d) - __uint_as_float(hd)));
}

// S = Qh Kh^T + Qh Kl^T + Ql Kh^T over the first `steps` K=8 steps of the head dim (Q hi / lo from
// TMEM, K hi / lo in shared memory, KCH bytes per 32-column chunk).  The step count is dispatched
// once to a straight-line sequence of exactly that many MMAs per part: measured on B200, a runtime
// guard around each MMA raised the issue cost from ~30-40 to ~70-90 clk per MMA.  Q4: each whole
// 32-column chunk goes as one four-MMA statement under one election (D = 128: measured 1046 ->
// 974 us on [2,8,4096,128]; with D <= 64 it measured 1-3 % slower, so those keep one per MMA).
template <int S, int KCH, bool Q4>
__device__ __forceinline__ void x3_issue_qk(int steps, uint32_t s_tmem, uint32_t qh, uint32_t ql, uint64_t dkh,
                                            uint64_t dkl, uint32_t idesc) {
  if (steps == S) {
#pragma unroll
    for (int part = 0; part < 3; ++part) {
      const uint32_t qa = part == 2 ? ql : qh;
      const uint64_t kb = part == 1 ? dkl : dkh;
      constexpr int S4 = Q4 ? (S & ~3) : 0;  // steps issued four at a time
#pragma unroll
      for (int s = 0; s < S4; s += 4)
        umma_ts_tf32_x4_w(s_tmem, qa + s * 8, kb + static_cast<uint64_t>(((s >> 2) * KCH) >> 4), idesc,
                          (part > 0 || s > 0) ? 1u : 0u);
#pragma unroll
      for (int s = S4; s < S; ++s) {
        const uint64_t koff = static_cast<uint64_t>(((s >> 2) * KCH + (s & 3) * 32) >> 4);
        umma_ts_tf32_w(s_tmem, qa + s * 8, kb + koff, idesc, (part > 0 || s > 0) ? 1u : 0u);
      }
    }
  } else if constexpr (S > 1) {
    x3_issue_qk<S - 1, KCH, Q4>(steps, s_tmem, qh, ql, dkh, dkl, idesc);
  }
}

// O (+)= Ph Vh + Ph Vl + Pl Vh over a tile's BN keys (BN / 8 K-steps of 8; V^T in 32-key chunks of
// VCH bytes), P hi / lo from TMEM.  Q4 as for x3_issue_qk.
template <int BN, int VCH, bool Q4>
__device__ __forceinline__ void x3_issue_pv(uint32_t o_tmem, uint32_t ph, uint32_t pl, uint64_t dvh, uint64_t dvl,
                                            uint32_t idesc, uint32_t acc0) {
#pragma unroll
  for (int part = 0; part < 3; ++part) {
    const uint32_t pa = part == 2 ? pl : ph;
    const uint64_t vb = part == 1 ? dvl : dvh;
#pragma unroll
    for (int s = 0; s < BN / 8; s += Q4 ? 4 : 1) {
      const uint64_t voff = static_cast<uint64_t>(((s >> 2) * VCH + (s & 3) * 32) >> 4);
      const uint32_t acc = (part > 0 || s > 0) ? 1u : acc0;
      if constexpr (Q4)
        umma_ts_tf32_x4_w(o_tmem, pa + s * 8, vb + voff, idesc, acc);
      else
        umma_ts_tf32_w(o_tmem, pa + s * 8, vb + voff, idesc, acc);
    }
  }
}

// MK: no mask (0), a boolean mask (1), an additive fp32 mask (2) -- separate instantiations.
template <int DP, int MK>
__global__ void __launch_bounds__(352, 1)
    attn_tf32x3_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                             const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v,
                             const __grid_constant__ CUtensorMap tm_kh, const __grid_constant__ CUtensorMap tm_kl,
                             const __grid_constant__ CUtensorMap tm_vh, const __grid_constant__ CUtensorMap tm_vl,
                             const X3Params p) {
  using C = X3Cfg<DP>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto bar = [&](int i) -> uint32_t { return base + C::OFF_BAR + 8u * i; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const uint32_t sQ = base + C::OFF_Q;
  auto stage = [&](int load) -> uint32_t { return base + C::OFF_ST + (load % C::NS) * C::STAGE_BYTES; };

  // Work item w -> (b, h, q0, first key tile j0, number of key tiles); causal items heaviest-first
  // within a head.  A tail work item takes key tiles [j0, j0 + n_kv) of its (row tile, head).
  auto geometry = [&](int w, int& b, int& h, int& q0, int& j0, int& n_kv) {
    int item = w, part = 0;
    if (w >= p.n_whole) {
      const int u = w - p.n_whole;
      item = p.n_whole + u / p.split;
      part = u - (u / p.split) * p.split;
    }
    const int bh = item / p.n_qt;
    const int qt = item - bh * p.n_qt;
    b = bh / p.heads;
    h = bh - b * p.heads;
    q0 = (p.causal ? p.n_qt - 1 - qt : qt) * C::BM;
    const int kv_len = p.causal ? min(p.len_k, q0 + C::BM) : p.len_k;
    const int tiles = (kv_len + C::BN - 1) / C::BN;
    j0 = w >= p.n_whole ? part * tiles / p.split : 0;
    n_kv = w >= p.n_whole ? (part + 1) * tiles / p.split - j0 : tiles;
  };

  if (threadIdx.x == 0) {
    mbar_init(bar(C::B_QFULL), 1);
    mbar_init(bar(C::B_QFREE), 128);
    mbar_init(bar(C::B_QEMPTY), 1);
    mbar_init(bar(C::B_QCONV), 128);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(bar(C::B_FULL + s), 1);
      mbar_init(bar(C::B_CONV + s), 128);
      mbar_init(bar(C::B_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(C::B_SFULL + b), 1);
      mbar_init(bar(C::B_PREADY + b), 128);
      mbar_init(bar(C::B_PVD + b), 1);
    }
    mbar_init(bar(C::B_OFREE), 128);
    mbar_init(bar(C::B_VREAD), 128);
    mbar_init(bar(C::B_EPI), 128);
    mbar_init(bar(C::B_EPI2), 1);
    mbar_init(bar(C::B_DRAIN), 1);
    mbar_init(bar(C::B_DRAIN + 1), 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == C::W_MMA) {
    tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == C::W_TMA && lane == 0) {
    tma_prefetch_desc(&tm_q);
    if (p.pre) {
      tma_prefetch_desc(&tm_kh);
      tma_prefetch_desc(&tm_kl);
      tma_prefetch_desc(&tm_vh);
      tma_prefetch_desc(&tm_vl);
    } else {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const WaitCtl ctl{abort_flag, p.dev_flags, p.timeout_ns};

  if (warp == C::W_TMA) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int load = 0;
      bool ok = true;
      for (int k = 0, w = blockIdx.x; ok && w < p.n_work; ++k, w += gridDim.x) {
        int b, h, q0, j0, n_kv;
        geometry(w, b, h, q0, j0, n_kv);
        // the staging tile is free once the converter has read the previous item's Q
        if (k > 0 && !(ok = mbar_wait(bar(C::B_QFREE), static_cast<uint32_t>(k - 1) & 1u, ctl))) break;
        mbar_arrive_expect_tx(bar(C::B_QFULL), C::Q_BYTES);
        for (int c = 0; c < C::NQC; ++c) tma_load_4d(sQ + c * C::QCH, &tm_q, bar(C::B_QFULL), c * 32, q0, h, b);
        for (int j = 0; ok && j < n_kv; ++j, ++load) {
          const int st = load % C::NS;
          if (!(ok = mbar_wait(bar(C::B_EMPTY + st), (static_cast<uint32_t>(load / C::NS) & 1u) ^ 1u, ctl))) break;
          const uint32_t sb = stage(load);
          if (p.pre) {  // the four split operand tiles, as the MMAs read them
            const int bhkv = b * p.heads_kv + h / p.group, key0 = (j0 + j) * C::BN;
            mbar_arrive_expect_tx(bar(C::B_FULL + st), 4 * C::T_BYTES);
            for (int c = 0; c < C::NQC; ++c) {
              tma_load_3d(sb + C::ST_K + c * C::KCH, &tm_kh, bar(C::B_FULL + st), c * 32, key0, bhkv);
              tma_load_3d(sb + C::ST_B + c * C::KCH, &tm_kl, bar(C::B_FULL + st), c * 32, key0, bhkv);
            }
            for (int u = 0; u < C::BN / 32; ++u) {
              tma_load_3d(sb + C::ST_VTH + u * C::VCH, &tm_vh, bar(C::B_FULL + st), key0 + u * 32, 0, bhkv);
              tma_load_3d(sb + C::ST_VTL + u * C::VCH, &tm_vl, bar(C::B_FULL + st), key0 + u * 32, 0, bhkv);
            }
          } else {
            mbar_arrive_expect_tx(bar(C::B_FULL + st), 2 * C::T_BYTES);
            for (int c = 0; c < C::NQC; ++c) {
              tma_load_4d(sb + C::ST_K + c * C::KCH, &tm_k, bar(C::B_FULL + st), c * 32, (j0 + j) * C::BN,
                          h / p.group, b);
              tma_load_4d(sb + C::ST_B + c * C::KCH, &tm_v, bar(C::B_FULL + st), c * 32, (j0 + j) * C::BN,
                          h / p.group, b);
            }
          }
        }
      }
      if (*abort_flag) {
        for (int i = max(0, load - C::NS); i < load; ++i)
          mbar_wait_drain(bar(C::B_FULL + i % C::NS), static_cast<uint32_t>(i / C::NS) & 1u, p.timeout_ns);
      }
    }
  } else if (warp == C::W_MMA) {
    // ------------------------------------------------------------------ S issuer (warp-uniform)
    // S_b = Qh Kh^T + Qh Kl^T + Ql Kh^T (Q from TMEM), qk_steps K-steps of 8.  Issue loops are
    // fully unrolled with compile-time offsets added to descriptors built once per product (the
    // start address sits in the low bits: no carry for shared-memory addresses), so each MMA costs
    // the issuing warp about one MMA slot.
    constexpr uint32_t kIdesc = idesc_tf32(128, C::BN, 0, 0);    // S: K-major A (TMEM) and B
    int load_base = 0;  // ring position of the item's first K/V tile
    int g = 0;          // tiles of all earlier items (S buffer and barrier phase bookkeeping)
    bool ok = true;
    for (int k = 0, w = blockIdx.x; ok && w < p.n_work; ++k, w += gridDim.x) {
      int b, h, q0, j0, n_kv;
      geometry(w, b, h, q0, j0, n_kv);
      (void)b; (void)h; (void)q0; (void)j0;
      if (!(ok = mbar_wait_all(bar(C::B_QCONV), static_cast<uint32_t>(k) & 1u, ctl))) break;
      for (int j = 0; j < n_kv; ++j) {
        const int ld = load_base + j, gq = g + j, bs = gq & 1;
        // K/V tile ready; buffer bs (tile gq-2's S, then P) consumed by PV(gq-2)
        if (!(ok = mbar_wait_all(bar((p.pre ? C::B_FULL : C::B_CONV) + ld % C::NS),
                                 static_cast<uint32_t>(ld / C::NS) & 1u, ctl)))
          break;
        if (gq >= 2 && !(ok = mbar_wait_all(bar(C::B_PVD + bs), static_cast<uint32_t>((gq - 2) >> 1) & 1u, ctl)))
          break;
        tc_fence_after_sync();
        const uint32_t sb = stage(ld);
        const uint64_t dkh = smem_desc_sw128(sb + C::ST_K, 16, 1024);
        const uint64_t dkl = smem_desc_sw128(sb + C::ST_B, 16, 1024);
        x3_issue_qk<DP / 8, C::KCH, DP == 128>(p.qk_steps, tmem + (bs ? C::TM_S1 : C::TM_S0), tmem + C::TM_QH,
                                               tmem + C::TM_QL, dkh, dkl, kIdesc);
        umma_commit_w(bar(C::B_SFULL + bs));
        if (j + 1 == n_kv) umma_commit_w(bar(C::B_QEMPTY));  // last product reading Q
      }
      g += n_kv;
      load_base += n_kv;
    }
  } else if (warp == C::W_PV) {
    // ------------------------------------------------------------------ P V issuer (warp-uniform)
    // O (+)= Ph Vh + Ph Vl + Pl Vh over the tile's keys; P of buffer pb (hi over its S, lo in Pl).
    // Separate from the S issuer, on another SMSP: each waits only for its own inputs.
    // O: K-major A (TMEM) and B (V^T); N = the head dim rounded up to 16 (D = 40: 48 of the 64 O
    // columns; the rest are never read for the output)
    const uint32_t kIdescPV = idesc_tf32(128, DP == 64 ? max(16, (p.head_dim + 15) & ~15) : DP, 0, 0);
    int load_base = 0, g = 0;
    bool ok = true;
    for (int k = 0, w = blockIdx.x; ok && w < p.n_work; ++k, w += gridDim.x) {
      int b, h, q0, j0, n_kv;
      geometry(w, b, h, q0, j0, n_kv);
      (void)b; (void)h; (void)q0; (void)j0;
      for (int j = 0; j < n_kv; ++j) {
        const int gp = g + j, pb = gp & 1;
        if (!(ok = mbar_wait_all(bar(C::B_PREADY + pb), static_cast<uint32_t>(gp >> 1) & 1u, ctl))) break;
        // the item's first PV overwrites O: the previous epilogue must have read it
        if (j == 0 && k > 0 && !(ok = mbar_wait_all(bar(C::B_OFREE), static_cast<uint32_t>(k - 1) & 1u, ctl)))
          break;
        tc_fence_after_sync();
        const uint32_t sb = stage(load_base + j);
        const uint64_t dvh = smem_desc_sw128(sb + C::ST_VTH, 16, 1024);
        const uint64_t dvl = smem_desc_sw128(sb + C::ST_VTL, 16, 1024);
        const uint32_t ph = tmem + (pb ? C::TM_S1 : C::TM_S0), pl = tmem + (pb ? C::TM_PL1 : C::TM_PL0);
        x3_issue_pv<C::BN, C::VCH, DP == 128>(tmem + C::TM_O, ph, pl, dvh, dvl, kIdescPV, j > 0 ? 1u : 0u);
        umma_commit_w(bar(C::B_PVD + pb));
        umma_commit_w(bar(C::B_EMPTY + (load_base + j) % C::NS));  // PV(j) is the stage's last reader
      }
      g += n_kv;
      load_base += n_kv;
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------------ converter (warps 2-5)
    const int tid = threadIdx.x - 64;  // 0..127
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // Q row of this thread = TMEM lane it writes
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    int load = 0;
    bool ok = true;
    for (int k = 0, w = blockIdx.x; ok && w < p.n_work; ++k, w += gridDim.x) {
      int b, h, q0, j0, n_kv;
      geometry(w, b, h, q0, j0, n_kv);
      // Q: this thread's row from the staging tile -> hi / lo -> TMEM, one 32-column chunk at a
      // time.  TMEM Q is free once the previous item's last S product is done.
      if (!(ok = mbar_wait_all(bar(C::B_QFULL), static_cast<uint32_t>(k) & 1u, ctl))) break;
      if (k > 0 && !(ok = mbar_wait_all(bar(C::B_QEMPTY), static_cast<uint32_t>(k - 1) & 1u, ctl))) break;
      tc_fence_after_sync();
#pragma unroll
      for (int c = 0; c < C::NQC; ++c) {
        uint32_t q[32];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint32_t addr = sQ + c * C::QCH + row * 128 + ((u ^ (row & 7)) << 4);
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(q[u * 4]), "=r"(q[u * 4 + 1]), "=r"(q[u * 4 + 2]), "=r"(q[u * 4 + 3])
                       : "r"(addr));
        }
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          hi[e] = tf32_trunc(q[e]);
          lo[e] = __float_as_uint(__uint_as_float(q[e]) - __uint_as_float(hi[e]));
        }
        tmem_st32(lane_base + C::TM_QH + c * 32, hi);
        tmem_st32(lane_base + C::TM_QL + c * 32, lo);
      }
      mbar_arrive(bar(C::B_QFREE));  // the staging tile may take the next item's Q
      tmem_st_wait();
      tc_fence_before_sync();
      mbar_arrive(bar(C::B_QCONV));
      if (p.pre) continue;  // the K / V tiles arrive split
      for (int j = 0; ok && j < n_kv; ++j, ++load) {
        const int st = load % C::NS;
        if (!(ok = mbar_wait_all(bar(C::B_FULL + st), static_cast<uint32_t>(load / C::NS) & 1u, ctl))) break;
        const uint32_t sb = stage(load);
        // V [key][d] (slot B) -> V^T [d][key] hi / lo (K-major B operand: rows d, BN keys in 32-key
        // 128-byte chunks of VCH bytes).  Thread -> (d = tid % DP, keys half*32 .. half*32+31):
        // two threads per row d for D = 64 (64 keys), one for D = 128 (32 keys).
        {
          const int d = tid % DP, half = tid / DP;
          const uint32_t vsrc = sb + C::ST_B + (d >> 5) * C::KCH + (d & 3) * 4;
          const int du = (d & 31) >> 2;  // 16-byte unit of column d inside its 128-byte row
          const uint32_t dst_row = half * C::VCH + d * 128;
#pragma unroll
          for (int u = 0; u < 8; ++u) {  // four keys per 16-byte unit of the V^T row
            uint32_t x[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int r = half * 32 + u * 4 + e;  // key
              asm volatile("ld.shared.b32 %0, [%1];" : "=r"(x[e]) : "r"(vsrc + r * 128 + ((du ^ (r & 7)) << 4)));
            }
            const uint32_t off = dst_row + ((u ^ (d & 7)) << 4);
            const uint32_t h0 = tf32_trunc(x[0]), h1 = tf32_trunc(x[1]), h2 = tf32_trunc(x[2]), h3 = tf32_trunc(x[3]);
            st_shared_v4(sb + C::ST_VTH + off, h0, h1, h2, h3);
            st_shared_v4(sb + C::ST_VTL + off, __float_as_uint(__uint_as_float(x[0]) - __uint_as_float(h0)),
                         __float_as_uint(__uint_as_float(x[1]) - __uint_as_float(h1)),
                         __float_as_uint(__uint_as_float(x[2]) - __uint_as_float(h2)),
                         __float_as_uint(__uint_as_float(x[3]) - __uint_as_float(h3)));
          }
        }
        // Every converter thread has read the raw V: slot B may now take K lo (a bounded wait on
        // an mbarrier, one phase per stage conversion, rather than a named barrier).
        mbar_arrive(bar(C::B_VREAD));
        if (!(ok = mbar_wait_all(bar(C::B_VREAD), static_cast<uint32_t>(load) & 1u, ctl))) break;
#pragma unroll 4
        for (int v = tid; v < C::T_BYTES / 16; v += 128)
          split_v4(sb + C::ST_K + v * 16, sb + C::ST_K + v * 16, sb + C::ST_B + v * 16);
        fence_proxy_async_smem();
        mbar_arrive(bar(C::B_CONV + st));
      }
    }
  } else if (warp < C::W_PV) {
    // ------------------------------------------------------------------ softmax / epilogue (6-9)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    const float masked = p.neg_scale ? INFINITY : -INFINITY;
    volatile int* last_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 8);
    int g = 0, nsp = 0;  // nsp: tail ranges this CTA has finished (barrier phases)
    bool ok = true;
    for (int k = 0, w = blockIdx.x; ok && w < p.n_work; ++k, w += gridDim.x) {
      int b, h, q0, j0, n_kv;
      geometry(w, b, h, q0, j0, n_kv);
      const int qrow = q0 + row;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < n_kv; ++j) {
        const int gj = g + j, bs = gj & 1;
        if (!(ok = mbar_wait_all(bar(C::B_SFULL + bs), static_cast<uint32_t>(gj >> 1) & 1u, ctl))) break;
        tc_fence_after_sync();
        uint32_t sr[C::BN];
        if constexpr (C::BN == 64)
          tmem_ld64(lane_base + (bs ? C::TM_S1 : C::TM_S0), sr);
        else
          tmem_ld32(lane_base + (bs ? C::TM_S1 : C::TM_S0), sr);
        float* s = reinterpret_cast<float*>(sr);
        tc_fence_before_sync();
        const int kv0 = (j0 + j) * C::BN;
        if constexpr (MK != 0) {
          if (qrow < p.len_q) {
            const long long roff = b * p.mk_b + h * p.mk_h + static_cast<long long>(qrow) * p.mk_q + kv0;
            const int nvalid = min(C::BN, p.len_k - kv0);  // keys past len_k are masked below
            if constexpr (MK == 1) {
              const uint8_t* mp = static_cast<const uint8_t*>(p.mask) + roff;
              if (nvalid == C::BN) {
#pragma unroll
                for (int v = 0; v < C::BN / 16; ++v) {
                  const uint4 w = __ldg(reinterpret_cast<const uint4*>(mp) + v);
                  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                  for (int e = 0; e < 16; ++e)
                    if (((ws[e >> 2] >> ((e & 3) * 8)) & 0xffu) == 0u) s[v * 16 + e] = masked;
                }
              } else {
#pragma unroll
                for (int c = 0; c < C::BN; ++c)
                  if (c < nvalid && mp[c] == 0) s[c] = masked;
              }
            } else {
              // s += mask / scale, so that s * scale = q.k * scale + mask
              const float* mp = static_cast<const float*>(p.mask) + roff;
              const float is = p.mask_inv_scale;
              if (nvalid == C::BN) {
#pragma unroll
                for (int v = 0; v < C::BN / 4; ++v) {
                  const float4 w = __ldg(reinterpret_cast<const float4*>(mp) + v);
                  s[4 * v] = fmaf(w.x, is, s[4 * v]);
                  s[4 * v + 1] = fmaf(w.y, is, s[4 * v + 1]);
                  s[4 * v + 2] = fmaf(w.z, is, s[4 * v + 2]);
                  s[4 * v + 3] = fmaf(w.w, is, s[4 * v + 3]);
                }
              } else {
#pragma unroll
                for (int c = 0; c < C::BN; ++c)
                  if (c < nvalid) s[c] = fmaf(mp[c], is, s[c]);
              }
            }
          }
        }
        if (kv0 + C::BN > p.len_k || (p.causal && kv0 + C::BN - 1 > q0)) {
          int lim = p.len_k - kv0;
          if (p.causal) lim = min(lim, qrow - kv0 + 1);
#pragma unroll
          for (int c = 0; c < C::BN; ++c)
            if (c >= lim) s[c] = masked;
        }
        float a8[8];
        if (p.neg_scale) {
#pragma unroll
          for (int e = 0; e < 8; ++e) a8[e] = fminf(s[e], s[8 + e]);
#pragma unroll
          for (int c = 16; c < C::BN; c += 16)
#pragma unroll
            for (int e = 0; e < 8; ++e) a8[e] = fmin3(a8[e], s[c + e], s[c + 8 + e]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) a8[e] = fmaxf(s[e], s[8 + e]);
#pragma unroll
          for (int c = 16; c < C::BN; c += 16)
#pragma unroll
            for (int e = 0; e < 8; ++e) a8[e] = fmax3(a8[e], s[c + e], s[c + 8 + e]);
        }
        const float mx = p.neg_scale
                             ? fmin3(fmin3(a8[0], a8[1], a8[2]), fmin3(a8[3], a8[4], a8[5]), fminf(a8[6], a8[7]))
                             : fmax3(fmax3(a8[0], a8[1], a8[2]), fmax3(a8[3], a8[4], a8[5]), fmaxf(a8[6], a8[7]));
        const float m_tile = mx * sl2;
        float alpha = 1.f;
        if (m_run == -INFINITY || m_tile > m_run + 64.f) {
          const float m_new = fmaxf(m_run, m_tile);
          // (a masked row with no key so far keeps m = -inf and its l and O at 0)
          alpha = m_new == -INFINITY ? 1.f : ex2_approx(m_run - m_new);
          m_run = m_new;
        }
        const float nm = (m_run == -INFINITY) ? 0.f : -m_run;
        const uint64_t sl2x2 = f2_pack(sl2, sl2), nmx2 = f2_pack(nm, nm);
        uint64_t la = f2_pack(0.f, 0.f), lb = la;
#pragma unroll
        for (int c = 0; c < C::BN; c += 2) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(s[c], s[c + 1]), sl2x2, nmx2), x0, x1);
          s[c] = ex2_approx(x0);
          s[c + 1] = ex2_approx(x1);
          if (c & 2)
            lb = f2_add(lb, f2_pack(s[c], s[c + 1]));
          else
            la = f2_add(la, f2_pack(s[c], s[c + 1]));
        }
        float l0, l1;
        f2_unpack(f2_add(la, lb), l0, l1);
        l_run = l_run * alpha + (l0 + l1);
        // O moves only in the (rare) rescale: it needs the previous tile's PV done.  Storing P needs
        // no wait: buffer bs was last read by PV(gj-2), which completed before QK(gj) was issued.
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
          const int gprev = gj - 1;
          if (!(ok = mbar_wait_all(bar(C::B_PVD + (gprev & 1)), static_cast<uint32_t>(gprev >> 1) & 1u, ctl))) break;
          tc_fence_after_sync();
#pragma unroll
          for (int hh = 0; hh < C::NQC; ++hh) {
            uint32_t o[32];
            tmem_ld32(lane_base + C::TM_O + hh * 32, o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(lane_base + C::TM_O + hh * 32, o);
          }
        }
#pragma unroll
        for (int hh = 0; hh < C::BN / 32; ++hh) {
          uint32_t ph[32], pl[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const uint32_t bits = __float_as_uint(s[hh * 32 + e]);
            ph[e] = tf32_trunc(bits);
            pl[e] = __float_as_uint(s[hh * 32 + e] - __uint_as_float(ph[e]));
          }
          tmem_st32(lane_base + (bs ? C::TM_S1 : C::TM_S0) + hh * 32, ph);
          tmem_st32(lane_base + (bs ? C::TM_PL1 : C::TM_PL0) + hh * 32, pl);
        }
        tmem_st_wait();
        tc_fence_before_sync();
        mbar_arrive(bar(C::B_PREADY + bs));
      }
      if (!ok) break;
      // Epilogue: O / l, fp32, straight to global memory (this thread's row).
      const int glast = g + n_kv - 1;
      if (!(ok = mbar_wait_all(bar(C::B_PVD + (glast & 1)), static_cast<uint32_t>(glast >> 1) & 1u, ctl))) break;
      tc_fence_after_sync();
      float* dst = p.o + b * p.os_b + h * p.os_h + static_cast<long long>(qrow) * p.os_s;
      if (w >= p.n_whole) {
        // A key range of a tail item: park this row's (O, m, l); the CTA of the item's last range
        // to arrive merges them all.
        const int u = w - p.n_whole, ti = u / p.split;
        float* mine = p.part + (static_cast<size_t>(u) * C::BM + row) * (DP + 4);
#pragma unroll
        for (int hh = 0; hh < C::NQC; ++hh) {
          uint32_t o[32];
          tmem_ld32(lane_base + C::TM_O + hh * 32, o);
          if (hh + 1 == C::NQC) {
            tc_fence_before_sync();
            mbar_arrive(bar(C::B_OFREE));
          }
#pragma unroll
          for (int c = 0; c < 32; c += 4)
            __stcg(reinterpret_cast<float4*>(mine + hh * 32 + c),
                   make_float4(__uint_as_float(o[c]), __uint_as_float(o[c + 1]), __uint_as_float(o[c + 2]),
                               __uint_as_float(o[c + 3])));
        }
        __stcg(reinterpret_cast<float4*>(mine + DP), make_float4(m_run, l_run, 0.f, 0.f));
        __threadfence();  // this row's partial is visible device-wide before the range's arrival is
        mbar_arrive(bar(C::B_EPI));
        if (warp == 6) {  // one thread counts the range once all 128 rows are parked
          if (!(ok = mbar_wait_all(bar(C::B_EPI), static_cast<uint32_t>(nsp) & 1u, ctl))) break;
          if (lane == 0) {
            const unsigned sh = 8u * static_cast<unsigned>(ti & 3);
            unsigned* word = p.cnt + (ti >> 2);
            const unsigned old = atomicAdd(word, 1u << sh);
            const bool last = ((old >> sh) & 0xffu) == static_cast<unsigned>(p.split - 1);
            if (last) atomicSub(word, static_cast<unsigned>(p.split) << sh);  // left at 0
            *last_flag = last ? 1 : 0;
            mbar_arrive(bar(C::B_EPI2));
          }
          __syncwarp();
        }
        if (!(ok = mbar_wait_all(bar(C::B_EPI2), static_cast<uint32_t>(nsp) & 1u, ctl))) break;
        ++nsp;
        if (*last_flag && qrow < p.len_q) {  // every range of the item has parked: merge this row
          __threadfence();
          const float* first = p.part + (static_cast<size_t>(ti) * p.split * C::BM + row) * (DP + 4);
          const size_t step = static_cast<size_t>(C::BM) * (DP + 4);
          float mall = -INFINITY;
          for (int r = 0; r < p.split; ++r) mall = fmaxf(mall, __ldcg(first + r * step + DP));
          float wgt[8], lsum = 0.f;
          for (int r = 0; r < p.split; ++r) {
            const float mr = __ldcg(first + r * step + DP);
            wgt[r] = mr == -INFINITY ? 0.f : ex2_approx(mr - mall);
            lsum += wgt[r] * __ldcg(first + r * step + DP + 1);
          }
          const float inv_l = (MK != 0 && !(lsum > 0.f)) ? 0.f : 1.f / lsum;  // no key: output 0
          for (int c = 0; c < p.head_dim; ++c) {
            float acc = 0.f;
            for (int r = 0; r < p.split; ++r) acc += wgt[r] * __ldcg(first + r * step + c);
            dst[c] = acc * inv_l;
          }
        }
        g += n_kv;
        continue;
      }
      const float inv_l = (MK != 0 && !(l_run > 0.f)) ? 0.f : 1.f / l_run;  // no key: output 0
      const bool vec = (p.head_dim & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
#pragma unroll
      for (int hh = 0; hh < C::NQC; ++hh) {  // O / l, 32 columns at a time
        uint32_t o[32];
        tmem_ld32(lane_base + C::TM_O + hh * 32, o);
        if (hh + 1 == C::NQC) {
          tc_fence_before_sync();
          mbar_arrive(bar(C::B_OFREE));
        }
        if (qrow < p.len_q && hh * 32 < p.head_dim) {
          if (vec) {
#pragma unroll
            for (int c = 0; c < 32; c += 4)
              if (hh * 32 + c < p.head_dim)
                *reinterpret_cast<float4*>(dst + hh * 32 + c) =
                    make_float4(__uint_as_float(o[c]) * inv_l, __uint_as_float(o[c + 1]) * inv_l,
                                __uint_as_float(o[c + 2]) * inv_l, __uint_as_float(o[c + 3]) * inv_l);
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (hh * 32 + c < p.head_dim) dst[hh * 32 + c] = __uint_as_float(o[c]) * inv_l;
          }
        }
      }
      g += n_kv;
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if ((warp == C::W_MMA || warp == C::W_PV) && *abort_flag) {
    // each issuer waits for its own MMAs (a commit tracks the issuing thread's operations)
    const uint32_t drain = bar(C::B_DRAIN + (warp == C::W_PV ? 1 : 0));
    __syncwarp();
    umma_commit_w(drain);
    if (lane == 0) mbar_wait_drain(drain, 0, p.timeout_ns);
    __syncwarp();
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == C::W_MMA) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// K and V of every (batch, kv head) split once per call into the layouts the MMAs read: K hi / lo
// [bh][key][d] and V^T hi / lo [bh][d][key] (fp32, hi = TF32-truncated, lo = the exact remainder),
// padded with zeros to DP columns / rows and to lk_pad keys.  One block per 32 keys of one (b, h):
// K goes straight through (reads and writes contiguous along d), V through a shared-memory tile so
// that V^T's writes are contiguous along the keys.
struct X3SplitParams {
  const float* k;
  const float* v;
  long long ks_b, ks_h, ks_s, vs_b, vs_h, vs_s;
  int heads_kv, len_k, head_dim, dp, lk_pad;
  float* kh;
  float* kl;
  float* vh;
  float* vl;
};

__global__ void __launch_bounds__(256) x3_kv_split_kernel(const X3SplitParams p) {
  __shared__ float tile[32][129];
  const int bh = blockIdx.y, b = bh / p.heads_kv, h = bh - b * p.heads_kv;
  const int key0 = blockIdx.x * 32;
  const float* kin = p.k + b * p.ks_b + h * p.ks_h;
  const float* vin = p.v + b * p.vs_b + h * p.vs_h;
  for (int e = threadIdx.x; e < 32 * p.dp; e += 256) {
    const int r = e / p.dp, d = e - r * p.dp, key = key0 + r;
    const bool in = key < p.len_k && d < p.head_dim;
    const float x = in ? __ldg(kin + static_cast<long long>(key) * p.ks_s + d) : 0.f;
    const float hi = __uint_as_float(tf32_trunc(__float_as_uint(x)));
    const size_t o = (static_cast<size_t>(bh) * p.lk_pad + key) * p.dp + d;
    p.kh[o] = hi;
    p.kl[o] = x - hi;
    tile[r][d] = in ? __ldg(vin + static_cast<long long>(key) * p.vs_s + d) : 0.f;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 32 * p.dp; e += 256) {
    const int d = e >> 5, r = e & 31;
    const float x = tile[r][d];
    const float hi = __uint_as_float(tf32_trunc(__float_as_uint(x)));
    const size_t o = (static_cast<size_t>(bh) * p.dp + d) * p.lk_pad + key0 + r;
    p.vh[o] = hi;
    p.vl[o] = x - hi;
  }
}

// --------------------------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------------------------
namespace {

bool s16_f32(int64_t s) { return s > 0 && ((s * 4) % 16) == 0 && (s * 4) < (1ll << 40); }

bool make_map_f32(CUtensorMap* map, const void* ptr, int64_t D, int64_t L, int64_t H, int64_t B,
                  const int64_t* st, uint32_t box_rows) {
  const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(L),
                            static_cast<uint64_t>(H), static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(st[2]) * 4, static_cast<uint64_t>(st[1]) * 4,
                               static_cast<uint64_t>(st[0]) * 4};
  const uint32_t box[4] = {32, box_rows, 1, 1};
  return encode_tmap(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ptr, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

bool attn_tf32x3_eligible(const cmpx_attn_desc* d) {
  if (d->dtype != CMPX_F32 || d->head_dim < 1 || d->head_dim > 128) return false;
  if (d->mask) {  // rows read with 16-byte loads: base and stepped strides 16-byte aligned
    const int64_t unit = d->mask_kind == CMPX_MASK_BOOL ? 16 : 4;  // elements per 16 bytes
    if ((reinterpret_cast<uintptr_t>(d->mask) & 15u) != 0 || d->mask_stride[3] != 1) return false;
    const int64_t extent[3] = {d->batch, d->heads, d->len_q};
    for (int i = 0; i < 3; ++i)
      if (extent[i] > 1 && d->mask_stride[i] % unit != 0) return false;  // (a single index: never stepped)
  }
  const void* ptrs[3] = {d->q, d->k, d->v};
  for (const void* ptr : ptrs)
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) return false;
  const int64_t* strides[3] = {d->q_stride, d->k_stride, d->v_stride};
  for (const int64_t* s : strides)
    for (int i = 0; i < 3; ++i)
      if (!s16_f32(s[i])) return false;
  if (((d->len_q + 127) / 128) * d->heads * d->batch > (1ll << 30)) return false;
  return true;
}

namespace {

// Tail split of a non-causal launch: with n_items = waves * grid + rem (0 < rem <= grid / 2), the
// rem items of the partial last wave are cut into split = min(grid / rem, 8, key tiles / 4) key
// ranges, so that the last wave holds rem * split <= grid ranges of 1/split of an item each.  A
// launch of fewer items than SMs cuts every item, into ranges of at least 8 key tiles
// ([2,8,128,8192,64]: 16 items on 16 of the 148 SMs before).
// The counters take the workspace's first 256 bytes (zero before and after every call, the same
// bytes the 16-bit kernels' counters use), the partial rows the bytes after them.
struct X3Split {
  int n_whole = 0, split = 1;
  size_t cnt_bytes = 0, bytes = 0;
};

template <int DP>
X3Split x3_split_plan(const cmpx_attn_desc* d, int num_sms) {
  using C = X3Cfg<DP>;
  X3Split sp;
  if (d->causal) return sp;
  const int64_t n_qt = (d->len_q + C::BM - 1) / C::BM;
  const int64_t n_items = n_qt * d->heads * d->batch;
  const int64_t sms = std::max(1, num_sms);
  const int64_t tiles = (d->len_k + C::BN - 1) / C::BN;
  if (n_items < 1) return sp;
  if (n_items < sms) {  // every item cut, into ranges of at least 8 key tiles
    const int64_t split = std::min<int64_t>({sms / n_items, 8, tiles / 8});
    if (split < 2) return sp;
    sp.n_whole = 0;
    sp.split = static_cast<int>(split);
    sp.cnt_bytes = 256;
    sp.bytes = sp.cnt_bytes + static_cast<size_t>(n_items) * split * C::BM * (DP + 4) * 4;
    return sp;
  }
  const int64_t grid = sms;
  const int64_t rem = n_items % grid;
  if (rem == 0 || 2 * rem > grid) return sp;
  // At least 4 key tiles per range: with fewer, the ranges' park-and-merge costs more than the
  // idle tail it fills (SD1.5 fp32 cross-attention [2,8,4096,77,40], 2 key tiles per item: 68.6 us
  // split into single tiles, 35.8 us unsplit).
  const int64_t split = std::min<int64_t>({grid / rem, 8, tiles / 4});
  if (split < 2 || rem > 256) return sp;  // (one 8-bit counter per tail item in the first 256 bytes)
  sp.n_whole = static_cast<int>(n_items - rem);
  sp.split = static_cast<int>(split);
  sp.cnt_bytes = 256;
  sp.bytes = sp.cnt_bytes + static_cast<size_t>(rem) * split * C::BM * (DP + 4) * 4;
  return sp;
}

// Split operands (pre): four fp32 buffers of B * heads_kv * lk_pad * DP, after the split's bytes
// (1024-aligned), worth it when every (b, h) has two or more 128-row items to share them and an
// item reads four or more key tiles: for shorter key sequences the pre-pass launch costs more than
// the per-stage split it saves ([2,8,1024,77,80]: 31.7 us with it, 20.5 us without).
struct X3Pre {
  bool use = false;
  int lk_pad = 0;
  size_t off = 0, each = 0, bytes = 0;  // bytes: the whole workspace with them
};

template <int DP>
X3Pre x3_pre_plan(const cmpx_attn_desc* d, const X3Split& sp) {
  using C = X3Cfg<DP>;
  X3Pre pr;
  if ((d->len_q + C::BM - 1) / C::BM < 2 || (d->len_k + C::BN - 1) / C::BN < 4) return pr;
  pr.use = true;
  pr.lk_pad = static_cast<int>((d->len_k + 63) / 64 * 64);
  pr.off = (std::max<size_t>(256, sp.bytes) + 1023) & ~static_cast<size_t>(1023);
  pr.each = static_cast<size_t>(d->batch) * attn_heads_kv(d) * pr.lk_pad * DP * 4;
  pr.bytes = pr.off + 4 * pr.each;
  return pr;
}

template <int DP>
int launch_tf32x3_typed(const cmpx_attn_desc* d, const LaunchCtx& ctx) {
  using C = X3Cfg<DP>;
  CUtensorMap tq, tk, tv;
  if (!make_map_f32(&tq, d->q, d->head_dim, d->len_q, d->heads, d->batch, d->q_stride, C::BM) ||
      !make_map_f32(&tk, d->k, d->head_dim, d->len_k, attn_heads_kv(d), d->batch, d->k_stride, C::BN) ||
      !make_map_f32(&tv, d->v, d->head_dim, d->len_k, attn_heads_kv(d), d->batch, d->v_stride, C::BN))
    return CMPX_ERR_LAUNCH;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    const void* ptrs[3] = {reinterpret_cast<const void*>(&attn_tf32x3_sm100_kernel<DP, 0>),
                           reinterpret_cast<const void*>(&attn_tf32x3_sm100_kernel<DP, 1>),
                           reinterpret_cast<const void*>(&attn_tf32x3_sm100_kernel<DP, 2>)};
    for (const void* f : ptrs)
      if (attr_err == cudaSuccess)
        attr_err = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return CMPX_ERR_LAUNCH;
  X3Params p;
  p.heads = static_cast<int>(d->heads);
  p.len_q = static_cast<int>(d->len_q);
  p.len_k = static_cast<int>(d->len_k);
  p.head_dim = static_cast<int>(d->head_dim);
  p.n_qt = static_cast<int>((d->len_q + C::BM - 1) / C::BM);
  p.n_items = static_cast<int>(p.n_qt * d->heads * d->batch);
  p.qk_steps = static_cast<int>((d->head_dim + 7) / 8);
  p.causal = d->causal ? 1 : 0;
  p.neg_scale = d->scale < 0 ? 1 : 0;
  p.group = attn_group(d);
  p.scale_log2 = static_cast<float>(d->scale * 1.4426950408889634);
  p.o = static_cast<float*>(d->o);
  p.os_b = d->o_stride[0];
  p.os_h = d->o_stride[1];
  p.os_s = d->o_stride[2];
  p.mask = d->mask;
  p.mk_b = d->mask_stride[0];
  p.mk_h = d->mask_stride[1];
  p.mk_q = d->mask_stride[2];
  p.mask_inv_scale = static_cast<float>(1.0 / d->scale);
  p.timeout_ns = ctx.timeout_ns;
  p.dev_flags = ctx.dev_flags;
  const X3Split sp = x3_split_plan<DP>(d, ctx.num_sms);
  p.n_whole = p.n_items;
  p.split = 1;
  p.n_work = p.n_items;
  p.cnt = nullptr;
  p.part = nullptr;
  if (sp.split > 1 && d->workspace && d->workspace_bytes >= sp.bytes &&
      (reinterpret_cast<uintptr_t>(d->workspace) & 255u) == 0) {
    p.n_whole = sp.n_whole;
    p.split = sp.split;
    p.n_work = sp.n_whole + (p.n_items - sp.n_whole) * sp.split;
    p.cnt = static_cast<unsigned int*>(d->workspace);
    p.part = reinterpret_cast<float*>(static_cast<char*>(d->workspace) + sp.cnt_bytes);
  }
  const int grid = std::min(p.n_work, std::max(1, ctx.num_sms));
  // Split operands, when the workspace holds them: one pre-pass launch, then TMA maps over them.
  const X3Pre pr = x3_pre_plan<DP>(d, sp);
  p.pre = 0;
  p.heads_kv = static_cast<int>(attn_heads_kv(d));
  CUtensorMap tkh = tk, tkl = tk, tvh = tv, tvl = tv;
  if (pr.use && d->workspace && d->workspace_bytes >= pr.bytes &&
      (reinterpret_cast<uintptr_t>(d->workspace) & 255u) == 0) {
    char* base = static_cast<char*>(d->workspace) + pr.off;
    X3SplitParams xp;
    xp.k = static_cast<const float*>(d->k);
    xp.v = static_cast<const float*>(d->v);
    xp.ks_b = d->k_stride[0];
    xp.ks_h = d->k_stride[1];
    xp.ks_s = d->k_stride[2];
    xp.vs_b = d->v_stride[0];
    xp.vs_h = d->v_stride[1];
    xp.vs_s = d->v_stride[2];
    xp.heads_kv = p.heads_kv;
    xp.len_k = p.len_k;
    xp.head_dim = p.head_dim;
    xp.dp = DP;
    xp.lk_pad = pr.lk_pad;
    xp.kh = reinterpret_cast<float*>(base);
    xp.kl = reinterpret_cast<float*>(base + pr.each);
    xp.vh = reinterpret_cast<float*>(base + 2 * pr.each);
    xp.vl = reinterpret_cast<float*>(base + 3 * pr.each);
    const uint64_t bhkv = static_cast<uint64_t>(d->batch) * p.heads_kv;
    const uint64_t kdims[3] = {static_cast<uint64_t>(DP), static_cast<uint64_t>(pr.lk_pad), bhkv};
    const uint64_t kst[2] = {static_cast<uint64_t>(DP) * 4, static_cast<uint64_t>(pr.lk_pad) * DP * 4};
    const uint32_t kbox[3] = {32, static_cast<uint32_t>(C::BN), 1};
    const uint64_t vdims[3] = {static_cast<uint64_t>(pr.lk_pad), static_cast<uint64_t>(DP), bhkv};
    const uint64_t vst[2] = {static_cast<uint64_t>(pr.lk_pad) * 4, static_cast<uint64_t>(DP) * pr.lk_pad * 4};
    const uint32_t vbox[3] = {32, static_cast<uint32_t>(DP), 1};
    const CUtensorMapDataType f32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    if (!encode_tmap(&tkh, f32, 3, xp.kh, kdims, kst, kbox, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&tkl, f32, 3, xp.kl, kdims, kst, kbox, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&tvh, f32, 3, xp.vh, vdims, vst, vbox, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap(&tvl, f32, 3, xp.vl, vdims, vst, vbox, CU_TENSOR_MAP_SWIZZLE_128B))
      return CMPX_ERR_LAUNCH;
    const dim3 sgrid(static_cast<unsigned>(pr.lk_pad / 32), static_cast<unsigned>(bhkv));
    x3_kv_split_kernel<<<sgrid, 256, 0, ctx.stream>>>(xp);
    p.pre = 1;
  }
  if (!d->mask)
    attn_tf32x3_sm100_kernel<DP, 0><<<grid, C::THREADS, C::SMEM_BYTES, ctx.stream>>>(tq, tk, tv, tkh, tkl, tvh, tvl, p);
  else if (d->mask_kind == CMPX_MASK_BOOL)
    attn_tf32x3_sm100_kernel<DP, 1><<<grid, C::THREADS, C::SMEM_BYTES, ctx.stream>>>(tq, tk, tv, tkh, tkl, tvh, tvl, p);
  else
    attn_tf32x3_sm100_kernel<DP, 2><<<grid, C::THREADS, C::SMEM_BYTES, ctx.stream>>>(tq, tk, tv, tkh, tkl, tvh, tvl, p);
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

}  // namespace

size_t attn_tf32x3_workspace_bytes(const cmpx_attn_desc* d, int num_sms) {
  if (!attn_tf32x3_eligible(d)) return 0;
  if (d->head_dim <= 64) {
    const X3Split sp = x3_split_plan<64>(d, num_sms);
    const X3Pre pr = x3_pre_plan<64>(d, sp);
    return pr.use ? pr.bytes : sp.bytes;
  }
  const X3Split sp = x3_split_plan<128>(d, num_sms);
  const X3Pre pr = x3_pre_plan<128>(d, sp);
  return pr.use ? pr.bytes : sp.bytes;
}

bool attn_tf32x3_tail_split(const cmpx_attn_desc* d, int num_sms) {
  if (!attn_tf32x3_eligible(d)) return false;
  return (d->head_dim <= 64 ? x3_split_plan<64>(d, num_sms).split : x3_split_plan<128>(d, num_sms).split) > 1;
}

int launch_attn_tf32x3(const cmpx_attn_desc* d, const LaunchCtx& ctx) {
  return d->head_dim <= 64 ? launch_tf32x3_typed<64>(d, ctx) : launch_tf32x3_typed<128>(d, ctx);
}

}  // namespace cmpx
