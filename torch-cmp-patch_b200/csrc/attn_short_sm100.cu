// attn_short_sm100.cu -- attention forward for short key sequences (fp16 / bf16, B200 sm_100a).
//
// Cross-attention to a text encoder's tokens (SD1.5 / SDXL: Lk = 77) has one key tile: the
// work per query row is tiny and the call is bound by reading Q and writing O.  The reference
// runs these calls through its non-causal fp16 kernel (flash_attn_hfma2_kernel,
// src/cuda/fp16_flash_attention_hfma2.cu:72-243; any Sq / Sk); the general kernel of this library
// (attn_fwd_sm100.cu) handles them correctly too, but its work item (two Q tiles, then the next
// item's Q) exposes a DRAM latency per item.  This kernel streams instead:
//
//   * each CTA takes a contiguous range of 128-row Q tiles (flattened over batch, head, row
//     tiles) and loads K and V of the current (batch, head) once -- again only when the head
//     changes inside its range;
//   * warp 8 keeps a ring of Q tiles in flight (6 stages for D <= 64, 3 for D = 128) with TMA;
//   * warp 9 issues S = Q K^T (tcgen05, fp32 in TMEM) for tile i+1 while tile i's softmax and PV
//     run, and O = P V with P read from TMEM, over only the key steps that hold keys;
//   * warps 0-3 / 4-7 take even / odd tiles: thread = row; one exact softmax pass (row max,
//     exp2, row sum -- no running max is needed with a single key tile), P (16-bit) to TMEM; then
//     the epilogue O / l through a per-warpgroup staging tile and TMA stores (clipped at Lq, D),
//     which overlaps the other warpgroup's softmax and the next QK.
//
// TMEM columns: S [0,128) (shared, the two warpgroups take it in turns), P0 [128,192),
// P1 [192,256), O0, O1.  Every wait is bounded (cmpx_ptx.cuh); on a timeout the CTA drains its
// copies and MMAs, frees TMEM, raises the device status word and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "cmpx_internal.h"
#include "cmpx_ptx.cuh"

namespace cmpx {

template <int DP>
struct ShortCfg {
  static constexpr int BM = 128;                     // query rows per tile
  static constexpr int NCH = DP / 64;                // 64-element (128-byte) chunks of the head dim
  static constexpr int CH_BYTES = 128 * 128;         // one chunk of 128 rows
  static constexpr int TILE_BYTES = NCH * CH_BYTES;  // one Q, K, V or O tile
  static constexpr int NQ = DP <= 64 ? 6 : 3;        // Q ring stages
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE_BYTES;
  static constexpr int OFF_Q = OFF_V + TILE_BYTES;
  static constexpr int OFF_OST = OFF_Q + NQ * TILE_BYTES;  // [2] staging tiles, one per warpgroup
  static constexpr int OFF_BAR = OFF_OST + 2 * TILE_BYTES;
  static constexpr int B_KVFULL = 0;             // K and V of the current head landed
  static constexpr int B_KVEMPTY = 1;            // every MMA reading the previous head's K/V done
  static constexpr int B_QFULL = 2;              // [NQ]
  static constexpr int B_QEMPTY = B_QFULL + NQ;  // [NQ]
  static constexpr int B_SFULL = B_QEMPTY + NQ;  // [2] S holds the tile of warpgroup g
  static constexpr int B_SFREE = B_SFULL + 2;    // S read (count 128; the warpgroups alternate)
  static constexpr int B_PREADY = B_SFREE + 1;   // [2] P_g written (count 128)
  static constexpr int B_PVDONE = B_PREADY + 2;  // [2] O_g = P_g V complete
  static constexpr int B_OFREE = B_PVDONE + 2;   // [2] epilogue has read O_g (count 128)
  static constexpr int B_DRAIN = B_OFREE + 2;
  static constexpr int NBAR = B_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // tmem base, abort word
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // +1024: runtime alignment slack
  static constexpr int TM_S = 0, TM_P0 = 128, TM_P1 = 192, TM_O0 = 256, TM_O1 = 256 + DP;
  static constexpr int TMEM_COLS = 512;
  static constexpr int THREADS = 320;
  static constexpr int W_TMA = 8, W_MMA = 9;
};

struct ShortParams {
  int heads;
  int len_q;
  int len_k;
  int n_qt;       // ceil(len_q / 128)
  int n_tiles;    // n_qt * heads * batch
  int pv_steps;   // ceil(len_k / 16): K=16 steps of P V that hold keys
  int neg_scale;  // scale < 0: masked scores are +inf so that masked * scale = -inf
  int group;      // query heads per key/value head (grouped-query attention)
  float scale_log2;
  unsigned long long timeout_ns;
  unsigned int* dev_flags;
};

// Position of a 128-row Q tile in the flattened (batch, head, row tile) order, stepped forward
// without integer division (one division per role at start).
struct TileCursor {
  int qt, h, b;  // row tile, head, batch
  __device__ void init(int t, const ShortParams& p) {
    const int bh = t / p.n_qt;
    qt = t - bh * p.n_qt;
    b = bh / p.heads;
    h = bh - b * p.heads;
  }
  __device__ void step(int k, const ShortParams& p) {
    qt += k;
    while (qt >= p.n_qt) {
      qt -= p.n_qt;
      if (++h == p.heads) {
        h = 0;
        ++b;
      }
    }
  }
  __device__ bool last_of_head(const ShortParams& p) const { return qt + 1 == p.n_qt; }
};

template <int DP, bool BF16>
__global__ void __launch_bounds__(320, 1)
    fmha_short_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v,
                            const __grid_constant__ CUtensorMap tm_o, const ShortParams p) {
  using C = ShortCfg<DP>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto bar = [&](int i) -> uint32_t { return base + C::OFF_BAR + 8u * i; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  // This CTA's tiles: [t_begin, t_end) of the flattened (batch, head, row tile) order.
  const int t_begin = static_cast<int>(static_cast<long long>(blockIdx.x) * p.n_tiles / gridDim.x);
  const int t_end = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * p.n_tiles / gridDim.x);
  const int n = t_end - t_begin;

  if (threadIdx.x == 0) {
    mbar_init(bar(C::B_KVFULL), 1);
    mbar_init(bar(C::B_KVEMPTY), 1);
    for (int s = 0; s < C::NQ; ++s) {
      mbar_init(bar(C::B_QFULL + s), 1);
      mbar_init(bar(C::B_QEMPTY + s), 1);
    }
    mbar_init(bar(C::B_SFREE), 128);
    for (int g = 0; g < 2; ++g) {
      mbar_init(bar(C::B_SFULL + g), 1);
      mbar_init(bar(C::B_PREADY + g), 128);
      mbar_init(bar(C::B_PVDONE + g), 1);
      mbar_init(bar(C::B_OFREE + g), 128);
    }
    mbar_init(bar(C::B_DRAIN), 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == C::W_MMA) {
    tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == C::W_TMA && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_o);
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_holder;
  const WaitCtl ctl{abort_flag, p.dev_flags, p.timeout_ns};

  if (warp == C::W_TMA) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int kv_round = 0, issued = 0;
      bool ok = true;
      TileCursor cur;
      cur.init(t_begin, p);
      for (int i = 0; ok && i < n; ++i, cur.step(1, p)) {
        const int b = cur.b, h = cur.h;
        if (i == 0 || cur.qt == 0) {  // first tile, or the first tile of a new head
          // K/V of a new head: wait until every MMA reading the previous head's K/V is done.
          if (kv_round > 0 &&
              !(ok = mbar_wait(bar(C::B_KVEMPTY), static_cast<uint32_t>(kv_round - 1) & 1u, ctl)))
            break;
          mbar_arrive_expect_tx(bar(C::B_KVFULL), 2 * C::TILE_BYTES);
          for (int c = 0; c < C::NCH; ++c) {
            tma_load_4d(base + C::OFF_K + c * C::CH_BYTES, &tm_k, bar(C::B_KVFULL), c * 64, 0, h / p.group, b);
            tma_load_4d(base + C::OFF_V + c * C::CH_BYTES, &tm_v, bar(C::B_KVFULL), c * 64, 0, h / p.group, b);
          }
          ++kv_round;
        }
        const int st = i % C::NQ;
        const uint32_t rnd = static_cast<uint32_t>(i / C::NQ);
        if (!(ok = mbar_wait(bar(C::B_QEMPTY + st), (rnd & 1u) ^ 1u, ctl))) break;
        mbar_arrive_expect_tx(bar(C::B_QFULL + st), C::TILE_BYTES);
        for (int c = 0; c < C::NCH; ++c)
          tma_load_4d(base + C::OFF_Q + st * C::TILE_BYTES + c * C::CH_BYTES, &tm_q,
                      bar(C::B_QFULL + st), c * 64, cur.qt * C::BM, h, b);
        issued = i + 1;
      }
      if (*abort_flag) {
        // Let every copy still in flight land before shared memory goes away.
        for (int i = max(0, issued - C::NQ); i < issued; ++i)
          mbar_wait_drain(bar(C::B_QFULL + i % C::NQ), static_cast<uint32_t>(i / C::NQ) & 1u,
                          p.timeout_ns);
        if (kv_round > 0)
          mbar_wait_drain(bar(C::B_KVFULL), static_cast<uint32_t>(kv_round - 1) & 1u, p.timeout_ns);
      }
    }
  } else if (warp == C::W_MMA) {
    // ------------------------------------------------------------------ MMA issuer
    // Warp-uniform control flow; one elected lane issues the MMAs and commits (the *_w helpers).
    constexpr uint32_t kIdescQK = idesc_f16(128, 128, BF16 ? 1 : 0, 0, 0);
    constexpr uint32_t kIdescPV = idesc_f16(128, DP, BF16 ? 1 : 0, 0, 1);
    auto issue_qk = [&](int st) {
      const uint32_t q_addr = base + C::OFF_Q + st * C::TILE_BYTES;
      const uint32_t k_addr = base + C::OFF_K;
#pragma unroll
      for (int k = 0; k < DP / 16; ++k) {
        const uint32_t off = (k >> 2) * C::CH_BYTES + (k & 3) * 32;
        umma_ss_w(tmem + C::TM_S, smem_desc_sw128(q_addr + off, 16, 1024),
                  smem_desc_sw128(k_addr + off, 16, 1024), kIdescQK, k > 0 ? 1u : 0u);
      }
    };
    auto issue_pv = [&](int g) {
      const uint32_t p_tmem = tmem + (g ? C::TM_P1 : C::TM_P0);
      const uint32_t d_tmem = tmem + (g ? C::TM_O1 : C::TM_O0);
      const uint32_t v_addr = base + C::OFF_V;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k < p.pv_steps)
          umma_ts_w(d_tmem, p_tmem + k * 8, smem_desc_sw128(v_addr + k * 2048, C::CH_BYTES, 1024),
                    kIdescPV, k > 0 ? 1u : 0u);
      }
    };
    // QK of tile i (the S buffer must have been read by tile i-1's softmax).
    auto start_qk = [&](int i, uint32_t& n_sfree) -> bool {
      if (i > 0 && !mbar_wait_all(bar(C::B_SFREE), (n_sfree++) & 1u, ctl)) return false;
      const int st = i % C::NQ;
      if (!mbar_wait_all(bar(C::B_QFULL + st), static_cast<uint32_t>(i / C::NQ) & 1u, ctl)) return false;
      tc_fence_after_sync();
      issue_qk(st);
      umma_commit_w(bar(C::B_SFULL + (i & 1)));
      umma_commit_w(bar(C::B_QEMPTY + st));
      return true;
    };
    bool ok = n > 0;
    int kv_round = 0;
    uint32_t n_sfree = 0;
    if (ok) {
      ok = mbar_wait_all(bar(C::B_KVFULL), 0u, ctl);
      kv_round = 1;
      ok = ok && start_qk(0, n_sfree);
    }
    TileCursor cur;
    cur.init(t_begin, p);
    for (int i = 0; ok && i < n; ++i, cur.step(1, p)) {
      const int g = i & 1;
      const bool next = i + 1 < n;
      const bool same_head = next && !cur.last_of_head(p);
      if (same_head && !(ok = start_qk(i + 1, n_sfree))) break;
      if (!(ok = mbar_wait_all(bar(C::B_PREADY + g), static_cast<uint32_t>(i >> 1) & 1u, ctl))) break;
      // O_g is overwritten: the epilogue of tile i-2 must have read it.
      if (i >= 2 &&
          !(ok = mbar_wait_all(bar(C::B_OFREE + g), static_cast<uint32_t>((i - 2) >> 1) & 1u, ctl)))
        break;
      tc_fence_after_sync();
      issue_pv(g);
      umma_commit_w(bar(C::B_PVDONE + g));
      if (next && !same_head) {
        // Tile i+1 belongs to another head: release K/V once every MMA so far is done, then
        // wait for the new head's K/V.
        umma_commit_w(bar(C::B_KVEMPTY));
        if (!(ok = mbar_wait_all(bar(C::B_KVFULL), static_cast<uint32_t>(kv_round) & 1u, ctl))) break;
        ++kv_round;
        if (!(ok = start_qk(i + 1, n_sfree))) break;
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    const int g = warp >> 2;            // warpgroup: tiles i with i % 2 == g
    const int wq = warp & 3;            // TMEM lane quarter of this warp
    const int row = wq * 32 + lane;     // row inside the tile
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    const uint32_t s_tm = lane_base + C::TM_S;
    const uint32_t p_tm = lane_base + (g ? C::TM_P1 : C::TM_P0);
    const uint32_t o_tm = lane_base + (g ? C::TM_O1 : C::TM_O0);
    const float sl2 = p.scale_log2;
    const float masked = p.neg_scale ? INFINITY : -INFINITY;  // masked * sl2 == -inf
    const int p_chunks = (p.pv_steps + 1) >> 1;  // 32-key chunks of P that the PV reads
    const uint32_t stage = base + C::OFF_OST + g * C::TILE_BYTES;
    bool ok = true;
    TileCursor cur;
    cur.init(t_begin + g, p);
    for (int i = g; ok && i < n; i += 2, cur.step(2, p)) {
      const uint32_t par = static_cast<uint32_t>(i >> 1) & 1u;
      if (!(ok = mbar_wait_all(bar(C::B_SFULL + g), par, ctl))) break;
      tc_fence_after_sync();
      uint32_t sr[128];
      tmem_ld128(s_tm, sr);
      float* s = reinterpret_cast<float*>(sr);
      tc_fence_before_sync();
      mbar_arrive(bar(C::B_SFREE));  // S is in registers: the next tile's QK may overwrite it
      // Only the first p_chunks 32-key chunks are used; mask keys >= Lk inside the partial one.
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q < p_chunks && (q + 1) * 32 > p.len_k) {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (q * 32 + c >= p.len_k) s[q * 32 + c] = masked;
        }
      }
      // Exact row max (min for a negative scale) over the used chunks, 8 chains of 3-input max.
      float a[8];
      if (p.neg_scale) {
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = fmin3(s[2 * e], s[2 * e + 1], s[16 + 2 * e]);
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = fminf(a[e], s[16 + 2 * e + 1]);
#pragma unroll
        for (int q = 1; q < 4; ++q)
          if (q < p_chunks) {
#pragma unroll
            for (int c = 0; c < 32; c += 16)
#pragma unroll
              for (int e = 0; e < 8; ++e) a[e] = fmin3(a[e], s[q * 32 + c + 2 * e], s[q * 32 + c + 2 * e + 1]);
          }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = fmax3(s[2 * e], s[2 * e + 1], s[16 + 2 * e]);
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = fmaxf(a[e], s[16 + 2 * e + 1]);
#pragma unroll
        for (int q = 1; q < 4; ++q)
          if (q < p_chunks) {
#pragma unroll
            for (int c = 0; c < 32; c += 16)
#pragma unroll
              for (int e = 0; e < 8; ++e) a[e] = fmax3(a[e], s[q * 32 + c + 2 * e], s[q * 32 + c + 2 * e + 1]);
          }
      }
      const float mx = p.neg_scale ? fmin3(fmin3(a[0], a[1], a[2]), fmin3(a[3], a[4], a[5]), fminf(a[6], a[7]))
                                   : fmax3(fmax3(a[0], a[1], a[2]), fmax3(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
      const float m = mx * sl2;
      // p = 2^(s*sl2 - m), 16-bit pairs to TMEM, chunk by chunk (only the chunks the PV reads).
      const uint64_t sl2x2 = f2_pack(sl2, sl2), nmx2 = f2_pack(-m, -m);
      uint64_t la = f2_pack(0.f, 0.f), lb = la;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q < p_chunks) {
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int cc = q * 16 + c;
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(s[2 * cc], s[2 * cc + 1]), sl2x2, nmx2), x0, x1);
            const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
            if (c & 1)
              lb = f2_add(lb, f2_pack(p0, p1));
            else
              la = f2_add(la, f2_pack(p0, p1));
            pk[c] = BF16 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
          }
          tmem_st16(p_tm + q * 16, pk);
        }
      }
      float l0, l1;
      f2_unpack(f2_add(la, lb), l0, l1);
      const float inv_l = 1.f / (l0 + l1);
      tmem_st_wait();
      tc_fence_before_sync();
      mbar_arrive(bar(C::B_PREADY + g));

      // Epilogue: O / l, 16-bit, through this warpgroup's staging tile, TMA stores per warp.
      if (!(ok = mbar_wait_all(bar(C::B_PVDONE + g), par, ctl))) break;
      tc_fence_after_sync();
      if (i >= 2) {  // this warp's staging rows: the store of tile i-2 must have read them
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
      }
#pragma unroll 1
      for (int c = 0; c < C::NCH; ++c) {
        const uint32_t row_addr = stage + c * C::CH_BYTES + row * 128;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t o[32];
          tmem_ld32(o_tm + c * 64 + hh * 32, o);
          if (c == C::NCH - 1 && hh == 1) {
            tc_fence_before_sync();
            mbar_arrive(bar(C::B_OFREE + g));  // O_g is read: tile i+2's PV may overwrite it
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t wv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float lo = __uint_as_float(o[q * 8 + 2 * e]) * inv_l;
              const float hi = __uint_as_float(o[q * 8 + 2 * e + 1]) * inv_l;
              wv[e] = BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
            }
            const int chunk = hh * 4 + q;  // 16-byte chunk within the 128-byte row
            st_shared_v4(row_addr + ((chunk ^ (row & 7)) << 4), wv[0], wv[1], wv[2], wv[3]);
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int row0 = cur.qt * C::BM + wq * 32;
        if (row0 < p.len_q) {
          for (int c = 0; c < C::NCH; ++c)
            tma_store_4d(&tm_o, stage + c * C::CH_BYTES + wq * 32 * 128, c * 64, row0, cur.h, cur.b);
        }
        bulk_commit_group();
      }
      __syncwarp();
    }
    if (lane == 0) bulk_wait_group0();  // every store of this warp complete before exit
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == C::W_MMA) {
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
bool fmha_short_eligible(const cmpx_attn_desc* d) {
  return (d->dtype == CMPX_F16 || d->dtype == CMPX_BF16) && !d->causal && d->len_k >= 1 &&
         d->len_k <= 128 && d->len_q > 0 && d->head_dim <= 128 && !d->mask;
}

const char* fmha_short_name(const cmpx_attn_desc* d) {
  const bool bf = d->dtype == CMPX_BF16;
  if (d->head_dim <= 64)
    return bf ? "fmha_sm100_short<bf16,D64,128q,kv<=128,6st,streamed>"
              : "fmha_sm100_short<f16,D64,128q,kv<=128,6st,streamed>";
  return bf ? "fmha_sm100_short<bf16,D128,128q,kv<=128,3st,streamed>"
            : "fmha_sm100_short<f16,D128,128q,kv<=128,3st,streamed>";
}

namespace {

template <int DP, bool BF16>
int launch_short_typed(const cmpx_attn_desc* d, const LaunchCtx& ctx) {
  using C = ShortCfg<DP>;
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv, to;
  if (!make_bhsd_map(&tq, dt, d->q, d->head_dim, d->len_q, d->heads, d->batch, d->q_stride, 128) ||
      !make_bhsd_map(&tk, dt, d->k, d->head_dim, d->len_k, attn_heads_kv(d), d->batch, d->k_stride, 128) ||
      !make_bhsd_map(&tv, dt, d->v, d->head_dim, d->len_k, attn_heads_kv(d), d->batch, d->v_stride, 128) ||
      !make_bhsd_map(&to, dt, d->o, d->head_dim, d->len_q, d->heads, d->batch, d->o_stride, 32))
    return CMPX_ERR_LAUNCH;

  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(reinterpret_cast<const void*>(&fmha_short_sm100_kernel<DP, BF16>),
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return CMPX_ERR_LAUNCH;

  ShortParams p;
  p.heads = static_cast<int>(d->heads);
  p.len_q = static_cast<int>(d->len_q);
  p.len_k = static_cast<int>(d->len_k);
  p.n_qt = static_cast<int>((d->len_q + C::BM - 1) / C::BM);
  p.n_tiles = static_cast<int>(p.n_qt * d->heads * d->batch);
  p.pv_steps = static_cast<int>((d->len_k + 15) / 16);
  p.neg_scale = d->scale < 0 ? 1 : 0;
  p.group = attn_group(d);
  p.scale_log2 = static_cast<float>(d->scale * 1.4426950408889634);
  p.timeout_ns = ctx.timeout_ns;
  p.dev_flags = ctx.dev_flags;
  const int grid = std::min(p.n_tiles, std::max(1, ctx.num_sms));
  fmha_short_sm100_kernel<DP, BF16><<<grid, C::THREADS, C::SMEM_BYTES, ctx.stream>>>(tq, tk, tv, to, p);
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

}  // namespace

int launch_fmha_short(const cmpx_attn_desc* d, const LaunchCtx& ctx) {
  const bool bf = d->dtype == CMPX_BF16;
  if (d->head_dim <= 64) return bf ? launch_short_typed<64, true>(d, ctx) : launch_short_typed<64, false>(d, ctx);
  return bf ? launch_short_typed<128, true>(d, ctx) : launch_short_typed<128, false>(d, ctx);
}

}  // namespace cmpx
