// attn_short_sm100.cu -- attention forward for short key sequences (fp16 / bf16, B200 sm_100a).
//
// Cross-attention to a text encoder's tokens (SD1.5 / SDXL: Lk = 77) has one key tile: the
// work per query row is tiny and the call is bound by reading Q and writing O.  The reference
// runs these calls through its non-causal fp16 kernel (flash_attn_hfma2_kernel,
// src/cuda/fp16_flash_attention_hfma2.cu:72-243, launched for any Sq / Sk at :269-286); the general
// kernel of this library (attn_fwd_sm100.cu) handles them correctly too, but a whole SM then works
// on one pair of Q tiles at a time.  At C2-cross sizes every SM owns only 4-5 Q tiles, so the
// kernel's duration is the latency chain of those few tiles (load Q, S = Q K^T, softmax, O = P V,
// store O), and the design goal here is to run as many of them side by side as the SM holds:
//
//   * each CTA takes a contiguous range of 128-row Q tiles (flattened over batch, head, row
//     tiles) and loads K and V of each (batch, head) it meets once, into one of two K/V buffers
//     (D <= 64), so a range that crosses a head boundary finds the next head's K/V already loaded;
//   * TMEM is cut into NSLOT tile slots, one per softmax warpgroup: S (fp32, SN columns, SN = Lk
//     rounded up to 64 / 96 / 128), with P (16-bit pairs) written over S, then O (DP columns).
//     D = 64 with Lk <= 64 / 96 / 128 gives 4 / 3 / 2 tiles in flight; D = 128 gives 2;
//   * the producer warp keeps a ring of Q tiles in flight (8 stages for D <= 64, 4 for D = 128);
//     it sets up the barriers those loads need, issues its first loads, and only then sets up the
//     other barriers, all before the CTA-wide barrier, so the first loads leave as early as possible
//     and overlap the TMEM allocation and the other warps' start;
//   * the MMA warp issues S = Q K^T of each tile into its slot, as soon as the Q tile has landed and
//     the slot's previous tile is retired (its O = P V, which reads P from the S columns, is done),
//     and retires tiles in order: once the last tile of a head is retired, that head's K/V buffer
//     goes back to the producer;
//   * softmax warpgroup g takes tiles i with i % NSLOT == g, thread = row: one exact pass (row max
//     and the exponentials only over the 16-key groups that hold keys; no running max is needed
//     with a single key tile); then the warpgroup meets at an mbarrier and one of its threads
//     issues O = P V itself (over only the K=16 key steps that hold keys), so no other warp has to
//     notice that P is ready; then the epilogue O / l, which stages the 16-bit O tile in the same Q
//     stage and stores it with TMA (clipped at Lq and D).  The stage goes back to the producer one
//     tile later, once the store has surely read it, so the wait for that read is off the path.
//     Meanwhile the MMA warp already computes the slot's next S.
//
// Every wait is bounded (cmpx_ptx.cuh); on a timeout the CTA drains its copies and MMAs, frees
// TMEM, raises the device status word and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "cmpx_internal.h"
#include "cmpx_ptx.cuh"

namespace cmpx {

template <int DP, int SN>
struct ShortCfg {
  static constexpr int BM = 128;                     // query rows per tile
  static constexpr int NCH = DP / 64;                // 64-element (128-byte) chunks of the head dim
  static constexpr int CH_BYTES = 128 * 128;         // one chunk of 128 rows
  static constexpr int TILE_BYTES = NCH * CH_BYTES;  // one Q, K, V or O tile
  static constexpr int SLOT_COLS = SN + DP;          // TMEM columns of one tile: S (and P), then O
  static constexpr int NSLOT = 512 / SLOT_COLS < 4 ? 512 / SLOT_COLS : 4;
  static constexpr int NKV = DP <= 64 ? 2 : 1;       // K/V buffers
  static constexpr int KV_BYTES = NKV * 2 * TILE_BYTES;
  static constexpr int NQ = DP <= 64 ? 8 : 4;        // Q ring stages (each also stages its tile's O)
  static constexpr int OFF_KV = 0;                   // [NKV] x {K, V}
  static constexpr int OFF_Q = OFF_KV + KV_BYTES;
  static constexpr int OFF_BAR = OFF_Q + NQ * TILE_BYTES;
  static constexpr int B_KVFULL = 0;                   // [NKV] K and V of a head landed
  static constexpr int B_KVEMPTY = B_KVFULL + NKV;     // [NKV] every MMA reading that head's K/V done
  static constexpr int B_QFULL = B_KVEMPTY + NKV;      // [NQ] Q tile landed
  static constexpr int B_QEMPTY = B_QFULL + NQ;        // [NQ] O stored from the stage (count 4)
  static constexpr int B_SFULL = B_QEMPTY + NQ;        // [NSLOT] S = Q K^T complete
  static constexpr int B_PREADY = B_SFULL + NSLOT;     // [NSLOT] P written (count 128)
  static constexpr int B_PVDONE = B_PREADY + NSLOT;    // [NSLOT] O = P V complete
  static constexpr int B_DRAIN = B_PVDONE + NSLOT;     // [1 + NSLOT] clean-up after an abort
  static constexpr int NBAR = B_DRAIN + 1 + NSLOT;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // tmem base, abort word
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // +1024: runtime alignment slack
  static constexpr int TMEM_COLS = 512;
  static constexpr int W_TMA = 4 * NSLOT, W_MMA = 4 * NSLOT + 1;
  static constexpr int THREADS = 128 * NSLOT + 64;
  static_assert(NSLOT >= 2 && NSLOT * SLOT_COLS <= TMEM_COLS, "TMEM slots");
  static_assert(SLOT_COLS % 32 == 0, "slot bases on 32-column boundaries");
  static_assert(SMEM_BYTES <= 232448 && NQ >= NSLOT + 1, "shared memory");
};

struct ShortParams {
  int heads;
  int len_q;
  int len_k;
  int n_qt;       // ceil(len_q / 128)
  int n_tiles;    // n_qt * heads * batch
  int pv_steps;   // ceil(len_k / 16): K=16 steps of P V that hold keys (= 16-key groups of P)
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
  int hidx;      // heads entered since the cursor was initialised (K/V buffer = hidx % NKV)
  __device__ void init(int t, const ShortParams& p) {
    const int bh = t / p.n_qt;
    qt = t - bh * p.n_qt;
    b = bh / p.heads;
    h = bh - b * p.heads;
    hidx = 0;
  }
  __device__ void step(int k, const ShortParams& p) {
    qt += k;
    while (qt >= p.n_qt) {
      qt -= p.n_qt;
      ++hidx;
      if (++h == p.heads) {
        h = 0;
        ++b;
      }
    }
  }
  __device__ bool last_of_head(const ShortParams& p) const { return qt + 1 == p.n_qt; }
};

// A row's scores: SN fp32 columns of TMEM starting at taddr, loaded with as few waits as possible.
template <int SN>
__device__ __forceinline__ void load_scores(uint32_t taddr, uint32_t (&s)[SN]) {
  static_assert(SN == 64 || SN == 96 || SN == 128, "score widths");
  if constexpr (SN == 128) {
    tmem_ld128(taddr, s);
  } else {
    tmem_ld64(taddr, *reinterpret_cast<uint32_t(*)[64]>(&s[0]));
    if constexpr (SN == 96) tmem_ld32(taddr + 64, *reinterpret_cast<uint32_t(*)[32]>(&s[64]));
  }
}

// Row maximum (NEG: minimum) over the first `groups` 16-key groups of s: 8 chains of 3-input max.
template <int SN, bool NEG>
__device__ __forceinline__ float group_max(const uint32_t (&s)[SN], int groups) {
  auto f = [](uint32_t v) { return __uint_as_float(v); };
  float a[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) a[e] = NEG ? fminf(f(s[2 * e]), f(s[2 * e + 1])) : fmaxf(f(s[2 * e]), f(s[2 * e + 1]));
#pragma unroll
  for (int gg = 1; gg < SN / 16; ++gg)
    if (gg < groups) {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        a[e] = NEG ? fmin3(a[e], f(s[16 * gg + 2 * e]), f(s[16 * gg + 2 * e + 1]))
                   : fmax3(a[e], f(s[16 * gg + 2 * e]), f(s[16 * gg + 2 * e + 1]));
    }
  return NEG ? fmin3(fmin3(a[0], a[1], a[2]), fmin3(a[3], a[4], a[5]), fminf(a[6], a[7]))
             : fmax3(fmax3(a[0], a[1], a[2]), fmax3(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
}

// O = P V over the first `groups` K=16 key steps: P from TMEM (16-bit pairs, 8 columns per step), V
// MN-major in shared memory.  The step count is dispatched once to a straight-line sequence of
// exactly that many MMAs: measured on B200, a runtime guard around each MMA raised the issue cost
// from ~28 to ~90 clk per 128x64x16 MMA.
template <int G, int DP, bool BF16>
__device__ __forceinline__ void issue_pv(int groups, uint32_t o_tmem, uint32_t p_tmem, uint32_t v_addr) {
  constexpr uint32_t kIdescPV = idesc_f16(128, DP, BF16 ? 1 : 0, 0, 1);  // P K-major, V MN-major
  if (groups == G) {
#pragma unroll
    for (int k = 0; k < G; ++k)
      umma_ts_w(o_tmem, p_tmem + k * 8, smem_desc_sw128(v_addr + k * 2048, 128 * 128, 1024),
                kIdescPV, k > 0 ? 1u : 0u);
  } else if constexpr (G > 1) {
    issue_pv<G - 1, DP, BF16>(groups, o_tmem, p_tmem, v_addr);
  }
}

template <int DP, int SN, bool BF16>
__global__ void __launch_bounds__(ShortCfg<DP, SN>::THREADS, 1)
    fmha_short_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v,
                            const __grid_constant__ CUtensorMap tm_o, const ShortParams p) {
  using C = ShortCfg<DP, SN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto bar = [&](int i) -> uint32_t { return base + C::OFF_BAR + 8u * i; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const WaitCtl ctl{abort_flag, p.dev_flags, p.timeout_ns};

  // This CTA's tiles: [t_begin, t_end) of the flattened (batch, head, row tile) order.
  const int t_begin = static_cast<int>(static_cast<long long>(blockIdx.x) * p.n_tiles / gridDim.x);
  const int t_end = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * p.n_tiles / gridDim.x);
  const int n = t_end - t_begin;

  // ---- producer state (lane 0 of the TMA warp) ----
  int pi = 0;         // next tile to load
  int phead = -1;     // index (within this CTA's range) of the last head whose K/V was loaded
  int pq_issued = 0;  // Q tiles loaded so far
  bool pok = true;
  TileCursor pcur;
  // Loads tiles from pi on.  With prologue set it stops before the first wait (a Q stage or a K/V
  // buffer still in use), so that it can run before the CTA-wide barrier.
  auto produce = [&](bool prologue) {
    for (; pok && pi < n; ++pi, pcur.step(1, p)) {
      const bool new_head = pi == 0 || pcur.qt == 0;
      if (prologue && (pi >= C::NQ || (new_head && phead + 1 >= C::NKV))) return;
      if (new_head) {
        const int hx = phead + 1, kb = hx % C::NKV;
        // The buffer's previous head (hx - NKV) must be released by every MMA reading it.
        if (hx >= C::NKV &&
            !(pok = mbar_wait(bar(C::B_KVEMPTY + kb), static_cast<uint32_t>(hx / C::NKV - 1) & 1u, ctl)))
          return;
        phead = hx;
        const uint32_t kv = base + C::OFF_KV + kb * 2 * C::TILE_BYTES;
        mbar_arrive_expect_tx(bar(C::B_KVFULL + kb), 2 * C::TILE_BYTES);
        for (int c = 0; c < C::NCH; ++c) {
          tma_load_4d(kv + c * C::CH_BYTES, &tm_k, bar(C::B_KVFULL + kb), c * 64, 0, pcur.h / p.group, pcur.b);
          tma_load_4d(kv + C::TILE_BYTES + c * C::CH_BYTES, &tm_v, bar(C::B_KVFULL + kb), c * 64, 0,
                      pcur.h / p.group, pcur.b);
        }
      }
      const int st = pi % C::NQ;
      const int rnd = pi / C::NQ;
      // The stage's previous tile (pi - NQ) must have stored its O from it.
      if (rnd > 0 && !(pok = mbar_wait(bar(C::B_QEMPTY + st), static_cast<uint32_t>(rnd - 1) & 1u, ctl)))
        return;
      mbar_arrive_expect_tx(bar(C::B_QFULL + st), C::TILE_BYTES);
      for (int c = 0; c < C::NCH; ++c)
        tma_load_4d(base + C::OFF_Q + st * C::TILE_BYTES + c * C::CH_BYTES, &tm_q, bar(C::B_QFULL + st),
                    c * 64, pcur.qt * C::BM, pcur.h, pcur.b);
      pq_issued = pi + 1;
    }
  };

  if (warp == C::W_TMA && lane == 0) {
    // The barriers the first loads complete on, then the loads, then every other barrier.
    for (int i = 0; i < C::NKV; ++i) mbar_init(bar(C::B_KVFULL + i), 1);
    for (int s = 0; s < C::NQ; ++s) mbar_init(bar(C::B_QFULL + s), 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    fence_proxy_async_smem();  // the initialised barriers are visible to this thread's copies
    pcur.init(t_begin, p);
    produce(true);
    for (int i = 0; i < C::NKV; ++i) mbar_init(bar(C::B_KVEMPTY + i), 1);
    for (int s = 0; s < C::NQ; ++s) mbar_init(bar(C::B_QEMPTY + s), 4);  // one per storing warp
    for (int g = 0; g < C::NSLOT; ++g) {
      mbar_init(bar(C::B_SFULL + g), 1);
      mbar_init(bar(C::B_PREADY + g), 128);
      mbar_init(bar(C::B_PVDONE + g), 1);
    }
    for (int g = 0; g <= C::NSLOT; ++g) mbar_init(bar(C::B_DRAIN + g), 1);
    fence_mbarrier_init();
    tma_prefetch_desc(&tm_o);
  }
  if (warp == C::W_MMA) {
    tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_holder;

  if (warp == C::W_TMA) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      produce(false);
      if (*abort_flag) {
        // Let every copy still in flight land before shared memory goes away: the last load
        // issued into each Q stage and each K/V buffer.
        for (int i = max(0, pq_issued - C::NQ); i < pq_issued; ++i)
          mbar_wait_drain(bar(C::B_QFULL + i % C::NQ), static_cast<uint32_t>(i / C::NQ) & 1u, p.timeout_ns);
        for (int hx = max(0, phead - C::NKV + 1); hx <= phead; ++hx)
          mbar_wait_drain(bar(C::B_KVFULL + hx % C::NKV), static_cast<uint32_t>(hx / C::NKV) & 1u,
                          p.timeout_ns);
      }
    }
  } else if (warp == C::W_MMA) {
    // ------------------------------------------------------------------ QK issuer / retirer
    // Warp-uniform control flow; one elected lane issues the MMAs and commits (the *_w helpers).
    // The warp polls for the next tile it can retire (its P V done) and for the inputs of the next
    // Q K^T, and acts on whichever is ready first.
    constexpr uint32_t kIdescQK = idesc_f16(128, SN, BF16 ? 1 : 0, 0, 0);
    auto ready = [&](uint32_t b, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_test_wait(b, parity));
    };
    TileCursor cq, cr;  // tiles of the next QK and of the next retirement
    cq.init(t_begin, p);
    cr.init(t_begin, p);
    int j = 0, ir = 0;  // next QK, next tile to retire
    int released = 0;   // heads whose K/V buffer has been handed back
    bool ok = true;
    uint64_t t_idle = global_timer_ns();
    while (ok && ir < n) {
      bool progress = false;
      // Retire the oldest tile whose P V is complete; after the last tile of a head (tiles retire
      // in order, and each tile's QK completed before its P V was issued) no MMA reads that head's
      // K/V any more.
      if (ir < j && ready(bar(C::B_PVDONE + ir % C::NSLOT), static_cast<uint32_t>(ir / C::NSLOT) & 1u)) {
        if (ir + 1 == n || cr.last_of_head(p)) {
          if (lane == 0) mbar_arrive(bar(C::B_KVEMPTY + cr.hidx % C::NKV));
          ++released;
        }
        ++ir;
        cr.step(1, p);
        progress = true;
      }
      // S = Q K^T of the next tile, into its slot.  The slot's previous tile must be retired (its
      // softmax has read S and its P V is done), its head's K/V buffer must hold that head (a
      // buffer is reloaded only after the head before it was released), and the Q tile must have
      // landed.
      if (j < n && j < ir + C::NSLOT && cq.hidx < released + C::NKV &&
          ready(bar(C::B_KVFULL + cq.hidx % C::NKV), static_cast<uint32_t>(cq.hidx / C::NKV) & 1u) &&
          ready(bar(C::B_QFULL + j % C::NQ), static_cast<uint32_t>(j / C::NQ) & 1u)) {
        const int slot = j % C::NSLOT;
        tc_fence_after_sync();
        const uint32_t q_addr = base + C::OFF_Q + (j % C::NQ) * C::TILE_BYTES;
        const uint32_t k_addr = base + C::OFF_KV + (cq.hidx % C::NKV) * 2 * C::TILE_BYTES;
#pragma unroll
        for (int k = 0; k < DP / 16; ++k) {
          const uint32_t off = (k >> 2) * C::CH_BYTES + (k & 3) * 32;
          umma_ss_w(tmem + slot * C::SLOT_COLS, smem_desc_sw128(q_addr + off, 16, 1024),
                    smem_desc_sw128(k_addr + off, 16, 1024), kIdescQK, k > 0 ? 1u : 0u);
        }
        umma_commit_w(bar(C::B_SFULL + slot));
        ++j;
        cq.step(1, p);
        progress = true;
      }
      if (progress) {
        t_idle = global_timer_ns();
      } else {
        if (*abort_flag) {
          ok = false;
          break;
        }
        if (global_timer_ns() - t_idle > p.timeout_ns) {
          if (lane == 0) {
            *abort_flag = 1;
            atomicOr(p.dev_flags, 1u /* CMPX_DEVFLAG_WAIT_TIMEOUT */);
          }
          ok = false;
          break;
        }
        __nanosleep(32);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax / P V / epilogue
    const int g = warp >> 2;         // warpgroup = TMEM slot: tiles i with i % NSLOT == g
    const int wq = warp & 3;         // TMEM lane quarter of this warp
    const int row = wq * 32 + lane;  // row inside the tile
    const uint32_t s_tm = tmem + (static_cast<uint32_t>(wq * 32) << 16) + g * C::SLOT_COLS;  // S, P
    const uint32_t o_tm = s_tm + SN;
    const float sl2 = p.scale_log2;
    const float masked = p.neg_scale ? INFINITY : -INFINITY;  // masked * sl2 == -inf
    const int groups = p.pv_steps;  // 16-key groups of P that the PV reads
    bool ok = true;
    int pending_stage = -1;  // Q stage whose O store may still be reading it
    TileCursor cur;
    cur.init(t_begin, p);
    cur.step(g, p);
    for (int i = g; ok && i < n; i += C::NSLOT, cur.step(C::NSLOT, p)) {
      const uint32_t par = static_cast<uint32_t>(i / C::NSLOT) & 1u;
      if (!(ok = mbar_wait_all(bar(C::B_SFULL + g), par, ctl))) break;
      tc_fence_after_sync();
      uint32_t s[SN];
      load_scores<SN>(s_tm, s);
      // Keys >= Lk inside the last group that holds keys are masked (written as a range test over
      // the groups from the last used one on: an equality test lets the compiler fold the loop into
      // one runtime-indexed access, which moves the whole row to local memory).
#pragma unroll
      for (int gg = 0; gg < SN / 16; ++gg) {
        if (gg + 1 >= groups) {
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (gg * 16 + c >= p.len_k) s[gg * 16 + c] = __float_as_uint(masked);
        }
      }
      // Exact row max (min for a negative scale), then p = 2^(s*sl2 - m) group by group: 16-bit
      // pairs written over the group's S columns, the row sum in fp32.
      const float mx = p.neg_scale ? group_max<SN, true>(s, groups) : group_max<SN, false>(s, groups);
      const uint64_t sl2x2 = f2_pack(sl2, sl2), nmx2 = f2_pack(-mx * sl2, -mx * sl2);
      uint64_t la = f2_pack(0.f, 0.f), lb = la;
#pragma unroll
      for (int gg = 0; gg < SN / 16; ++gg) {
        if (gg < groups) {
          uint32_t pk[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int k = gg * 16 + 2 * c;
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(s[k]), __uint_as_float(s[k + 1])), sl2x2, nmx2), x0, x1);
            const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
            if (c & 1)
              lb = f2_add(lb, f2_pack(p0, p1));
            else
              la = f2_add(la, f2_pack(p0, p1));
            pk[c] = BF16 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
          }
          tmem_st8(s_tm + gg * 8, pk);
        }
      }
      float l0, l1;
      f2_unpack(f2_add(la, lb), l0, l1);
      const float inv_l = 1.f / (l0 + l1);
      // Every row's P is written (and this warpgroup's loads of the slot's previous O are done):
      // one thread of the warpgroup issues O = P V.  (An mbarrier rather than a named barrier, so
      // that the wait stays bounded if the launch is aborted.)
      tmem_st_wait();
      tc_fence_before_sync();
      mbar_arrive(bar(C::B_PREADY + g));
      if (wq == 0) {
        if (!(ok = mbar_wait_all(bar(C::B_PREADY + g), par, ctl))) break;
        tc_fence_after_sync();
        const uint32_t p_tmem = tmem + g * C::SLOT_COLS;
        const uint32_t v_addr = base + C::OFF_KV + (cur.hidx % C::NKV) * 2 * C::TILE_BYTES + C::TILE_BYTES;
        issue_pv<SN / 16, DP, BF16>(groups, p_tmem + SN, p_tmem, v_addr);
        umma_commit_w(bar(C::B_PVDONE + g));
      }

      // Epilogue: O / l, 16-bit, staged in the tile's own Q stage (its Q was read by the QK, which
      // completed before S was handed over), TMA stores per warp, then the stage goes back to the
      // producer.
      // The previous tile's O store has long read its stage by now: hand that stage back.
      if (lane == 0 && pending_stage >= 0) {
        bulk_wait_group_read0();
        mbar_arrive(bar(C::B_QEMPTY + pending_stage));
      }
      pending_stage = -1;
      if (!(ok = mbar_wait_all(bar(C::B_PVDONE + g), par, ctl))) break;
      tc_fence_after_sync();
      const int st = i % C::NQ;
      const uint32_t stage = base + C::OFF_Q + st * C::TILE_BYTES;
#pragma unroll 1
      for (int c = 0; c < C::NCH; ++c) {
        const uint32_t row_addr = stage + c * C::CH_BYTES + row * 128;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t o[32];
          tmem_ld32(o_tm + c * 64 + hh * 32, o);
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
      tc_fence_before_sync();  // O is read: the slot's next P V (after the next P-ready) may write it
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
      pending_stage = st;  // handed back once the store has read it (next tile, or below)
      __syncwarp();
    }
    if (lane == 0) {
      if (pending_stage >= 0) {
        bulk_wait_group_read0();
        mbar_arrive(bar(C::B_QEMPTY + pending_stage));
      }
      bulk_wait_group0();  // every store of this warp complete before exit
    }
    if (wq == 0 && *abort_flag) {
      // Let this warpgroup's P V (if one is in flight) finish before TMEM is given back.
      __syncwarp();
      umma_commit_w(bar(C::B_DRAIN + 1 + g));  // same election as the P V MMAs
      if (lane == 0) mbar_wait_drain(bar(C::B_DRAIN + 1 + g), 0, p.timeout_ns);
      __syncwarp();
    }
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

namespace {

// S columns of a tile slot: the key count rounded up to 64 / 96 / 128 (D <= 64); 128 for D = 128.
int short_sn(const cmpx_attn_desc* d) {
  if (d->head_dim > 64) return 128;
  return d->len_k <= 64 ? 64 : d->len_k <= 96 ? 96 : 128;
}

template <int DP, int SN, bool BF16>
int launch_short_typed(const cmpx_attn_desc* d, const LaunchCtx& ctx) {
  using C = ShortCfg<DP, SN>;
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv, to;
  if (!make_bhsd_map(&tq, dt, d->q, d->head_dim, d->len_q, d->heads, d->batch, d->q_stride, 128) ||
      !make_bhsd_map(&tk, dt, d->k, d->head_dim, d->len_k, attn_heads_kv(d), d->batch, d->k_stride, 128) ||
      !make_bhsd_map(&tv, dt, d->v, d->head_dim, d->len_k, attn_heads_kv(d), d->batch, d->v_stride, 128) ||
      !make_bhsd_map(&to, dt, d->o, d->head_dim, d->len_q, d->heads, d->batch, d->o_stride, 32))
    return CMPX_ERR_LAUNCH;

  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(
        reinterpret_cast<const void*>(&fmha_short_sm100_kernel<DP, SN, BF16>),
        cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  });
  if (attr_err[dev & 63] != cudaSuccess) return CMPX_ERR_LAUNCH;

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
  fmha_short_sm100_kernel<DP, SN, BF16><<<grid, C::THREADS, C::SMEM_BYTES, ctx.stream>>>(tq, tk, tv, to, p);
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

}  // namespace

const char* fmha_short_name(const cmpx_attn_desc* d) {
  static const char* const names[2][4] = {
      {"fmha_sm100_short<f16,D64,S64,4slot,8st,streamed>", "fmha_sm100_short<f16,D64,S96,3slot,8st,streamed>",
       "fmha_sm100_short<f16,D64,S128,2slot,8st,streamed>", "fmha_sm100_short<f16,D128,S128,2slot,4st,streamed>"},
      {"fmha_sm100_short<bf16,D64,S64,4slot,8st,streamed>", "fmha_sm100_short<bf16,D64,S96,3slot,8st,streamed>",
       "fmha_sm100_short<bf16,D64,S128,2slot,8st,streamed>",
       "fmha_sm100_short<bf16,D128,S128,2slot,4st,streamed>"}};
  const int sn = short_sn(d);
  const int e = d->head_dim > 64 ? 3 : sn == 64 ? 0 : sn == 96 ? 1 : 2;
  return names[d->dtype == CMPX_BF16 ? 1 : 0][e];
}

int launch_fmha_short(const cmpx_attn_desc* d, const LaunchCtx& ctx) {
  const bool bf = d->dtype == CMPX_BF16;
  if (d->head_dim > 64) return bf ? launch_short_typed<128, 128, true>(d, ctx) : launch_short_typed<128, 128, false>(d, ctx);
  switch (short_sn(d)) {
    case 64:
      return bf ? launch_short_typed<64, 64, true>(d, ctx) : launch_short_typed<64, 64, false>(d, ctx);
    case 96:
      return bf ? launch_short_typed<64, 96, true>(d, ctx) : launch_short_typed<64, 96, false>(d, ctx);
    default:
      return bf ? launch_short_typed<64, 128, true>(d, ctx) : launch_short_typed<64, 128, false>(d, ctx);
  }
}

}  // namespace cmpx
