// attn_tf32x3_sm100.cu -- fp32 scaled-dot-product attention on the tensor cores (B200 sm_100a).
//
// The fp32 contract (1e-4 relative to stock fp32 SDPA) is out of reach of one TF32 product
// (10-bit mantissa: ~1e-3 per element), so every product here is split the 3xTF32 way: with
// x = x_hi + x_lo, x_hi the value truncated to TF32 (exactly representable) and x_lo = x - x_hi
// (exact in fp32), a b ~= a_hi b_hi + a_hi b_lo + a_lo b_hi, dropping only a_lo b_lo (~2^-22
// relative).  It replaces the reference's fp32 attention (attention_fp32_strict_kernel,
// src/cuda/fp32_attention.cu:35-198: one thread per query row on the CUDA cores) for head dims
// <= 64 (SD1.5's fp32 attention has D = 40); larger head dims keep the CUDA-core kernel of
// attn_fwd_f32.cu.
//
//   * a CTA owns a 128-row Q tile of one (batch, head) at a time (persistent, items strided over
//     the grid); keys stream in 64-key tiles;
//   * warp 0: TMA of Q (once per item) and K, V tiles (fp32, 128-byte swizzle, OOB zero-filled)
//     into a 2-stage ring;
//   * warps 2-5 ("converter"): Q and K split in place into hi (truncated) and lo parts; V
//     transposed into V^T hi / lo (the K-major B operand of P V);
//   * warp 1: tcgen05.mma kind::tf32 -- S = Qh Kh^T + Qh Kl^T + Ql Kh^T into one of two TMEM S
//     buffers, the next tile's S issued before this tile's P V; O += Ph Vh + Ph Vl + Pl Vh with
//     P read from TMEM;
//   * warps 6-9 (thread = row): exact tile max, running max moved only when a tile's max exceeds
//     it by more than 2^64 (fp32 keeps p = 2^(x - m) exact far beyond that; O, l and P share m,
//     so the result is the same), p in fp32, split into Ph / Pl in TMEM; the epilogue writes O / l.
//
// TMEM columns: S0 [0,64), S1 [64,128), Ph [128,192), Pl [192,256), O [256,320).
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

struct X3Cfg {
  static constexpr int BM = 128, BN = 64, DP = 64;  // query rows, keys per tile, padded head dim
  static constexpr int QCH = BM * 128;              // one 32-column (128-byte) chunk of a Q tile
  static constexpr int Q_BYTES = 2 * QCH;           // 32 KB
  static constexpr int KCH = BN * 128;              // one chunk of a K / V / V^T tile (64 rows)
  static constexpr int T_BYTES = 2 * KCH;           // 16 KB
  static constexpr int NS = 2;                      // K/V ring stages
  static constexpr int ST_K = 0, ST_KL = T_BYTES, ST_V = 2 * T_BYTES, ST_VTH = 3 * T_BYTES,
                       ST_VTL = 4 * T_BYTES;
  static constexpr int STAGE_BYTES = 5 * T_BYTES;   // 80 KB
  static constexpr int OFF_Q = 0, OFF_QL = Q_BYTES, OFF_ST = 2 * Q_BYTES;
  static constexpr int OFF_BAR = OFF_ST + NS * STAGE_BYTES;
  static constexpr int B_QFULL = 0, B_QCONV = 1, B_QEMPTY = 2;
  static constexpr int B_FULL = 3;                  // [NS]
  static constexpr int B_CONV = B_FULL + NS;        // [NS] count 128
  static constexpr int B_EMPTY = B_CONV + NS;       // [NS]
  static constexpr int B_SFULL = B_EMPTY + NS;      // [2]
  static constexpr int B_SFREE = B_SFULL + 2;       // [2] count 128
  static constexpr int B_PREADY = B_SFREE + 2;      // count 128
  static constexpr int B_PVDONE = B_PREADY + 1;
  static constexpr int B_OFREE = B_PVDONE + 1;      // count 128
  static constexpr int B_DRAIN = B_OFREE + 1;
  static constexpr int NBAR = B_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TM_S0 = 0, TM_S1 = 64, TM_PH = 128, TM_PL = 192, TM_O = 256;
  static constexpr int TMEM_COLS = 512;
  static constexpr int THREADS = 320;
  static constexpr int W_TMA = 0, W_MMA = 1;
};

struct X3Params {
  int heads, len_q, len_k, head_dim;
  int n_qt, n_items;
  int qk_steps;   // ceil(head_dim / 8): K=8 steps of Q K^T
  int causal, neg_scale;
  float scale_log2;
  float* o;
  long long os_b, os_h, os_s;
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

__global__ void __launch_bounds__(320, 1)
    attn_tf32x3_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                             const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v, const X3Params p) {
  using C = X3Cfg;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto bar = [&](int i) -> uint32_t { return base + C::OFF_BAR + 8u * i; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  const uint32_t sQ = base + C::OFF_Q, sQL = base + C::OFF_QL;
  auto stage = [&](int load) -> uint32_t { return base + C::OFF_ST + (load % C::NS) * C::STAGE_BYTES; };

  // Item w -> (b, h, q0, number of 64-key tiles); causal items heaviest-first within a head.
  auto geometry = [&](int w, int& b, int& h, int& q0, int& n_kv) {
    const int bh = w / p.n_qt;
    const int qt = w - bh * p.n_qt;
    b = bh / p.heads;
    h = bh - b * p.heads;
    q0 = (p.causal ? p.n_qt - 1 - qt : qt) * C::BM;
    const int kv_len = p.causal ? min(p.len_k, q0 + C::BM) : p.len_k;
    n_kv = (kv_len + C::BN - 1) / C::BN;
  };

  if (threadIdx.x == 0) {
    mbar_init(bar(C::B_QFULL), 1);
    mbar_init(bar(C::B_QCONV), 128);
    mbar_init(bar(C::B_QEMPTY), 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(bar(C::B_FULL + s), 1);
      mbar_init(bar(C::B_CONV + s), 128);
      mbar_init(bar(C::B_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(C::B_SFULL + b), 1);
      mbar_init(bar(C::B_SFREE + b), 128);
    }
    mbar_init(bar(C::B_PREADY), 128);
    mbar_init(bar(C::B_PVDONE), 1);
    mbar_init(bar(C::B_OFREE), 128);
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
      for (int k = 0, w = blockIdx.x; ok && w < p.n_items; ++k, w += gridDim.x) {
        int b, h, q0, n_kv;
        geometry(w, b, h, q0, n_kv);
        if (k > 0 && !(ok = mbar_wait(bar(C::B_QEMPTY), static_cast<uint32_t>(k - 1) & 1u, ctl))) break;
        mbar_arrive_expect_tx(bar(C::B_QFULL), C::Q_BYTES);
        for (int c = 0; c < 2; ++c) tma_load_4d(sQ + c * C::QCH, &tm_q, bar(C::B_QFULL), c * 32, q0, h, b);
        for (int j = 0; ok && j < n_kv; ++j, ++load) {
          const int st = load % C::NS;
          if (!(ok = mbar_wait(bar(C::B_EMPTY + st), (static_cast<uint32_t>(load / C::NS) & 1u) ^ 1u, ctl))) break;
          const uint32_t sb = stage(load);
          mbar_arrive_expect_tx(bar(C::B_FULL + st), 2 * C::T_BYTES);
          for (int c = 0; c < 2; ++c) {
            tma_load_4d(sb + C::ST_K + c * C::KCH, &tm_k, bar(C::B_FULL + st), c * 32, j * C::BN, h, b);
            tma_load_4d(sb + C::ST_V + c * C::KCH, &tm_v, bar(C::B_FULL + st), c * 32, j * C::BN, h, b);
          }
        }
      }
      if (*abort_flag) {
        for (int i = max(0, load - C::NS); i < load; ++i)
          mbar_wait_drain(bar(C::B_FULL + i % C::NS), static_cast<uint32_t>(i / C::NS) & 1u, p.timeout_ns);
      }
    }
  } else if (warp == C::W_MMA) {
    // ------------------------------------------------------------------ MMA issuer (warp-uniform)
    constexpr uint32_t kIdesc = idesc_tf32(128, 64, 0, 0);
    int load_base = 0;  // ring position of the item's first K/V tile
    int g = 0;          // tiles of all earlier items (S buffer and barrier phase bookkeeping)
    bool ok = true;
    // One S product: S_b = Qh Kh^T + Qh Kl^T + Ql Kh^T.
    auto issue_qk = [&](uint32_t sb, uint32_t s_tmem) {
      const uint32_t kh = sb + C::ST_K, kl = sb + C::ST_KL;
#pragma unroll 1
      for (int part = 0; part < 3; ++part) {
        const uint32_t qa = part == 2 ? sQL : sQ;
        const uint32_t kb = part == 1 ? kl : kh;
        for (int s = 0; s < p.qk_steps; ++s) {
          const uint32_t qoff = (s >> 2) * C::QCH + (s & 3) * 32;
          const uint32_t koff = (s >> 2) * C::KCH + (s & 3) * 32;
          umma_ss_tf32_w(s_tmem, smem_desc_sw128(qa + qoff, 16, 1024), smem_desc_sw128(kb + koff, 16, 1024),
                         kIdesc, (part > 0 || s > 0) ? 1u : 0u);
        }
      }
    };
    // O (+)= Ph Vh + Ph Vl + Pl Vh over the tile's 64 keys (8 K-steps of 8).
    auto issue_pv = [&](uint32_t sb, bool acc) {
      const uint32_t vh = sb + C::ST_VTH, vl = sb + C::ST_VTL;
#pragma unroll 1
      for (int part = 0; part < 3; ++part) {
        const uint32_t pa = tmem + (part == 2 ? C::TM_PL : C::TM_PH);
        const uint32_t vb = part == 1 ? vl : vh;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t voff = (s >> 2) * C::KCH + (s & 3) * 32;
          umma_ts_tf32_w(tmem + C::TM_O, pa + s * 8, smem_desc_sw128(vb + voff, 16, 1024), kIdesc,
                         (acc || part > 0 || s > 0) ? 1u : 0u);
        }
      }
    };
    for (int k = 0, w = blockIdx.x; ok && w < p.n_items; ++k, w += gridDim.x) {
      int b, h, q0, n_kv;
      geometry(w, b, h, q0, n_kv);
      (void)b; (void)h; (void)q0;
      if (!(ok = mbar_wait_all(bar(C::B_QCONV), static_cast<uint32_t>(k) & 1u, ctl))) break;
      auto do_pv = [&](int jj) -> bool {
        const int gj = g + jj;
        if (!mbar_wait_all(bar(C::B_PREADY), static_cast<uint32_t>(gj) & 1u, ctl)) return false;
        // The item's first PV overwrites O: the previous item's epilogue must have read it.
        if (jj == 0 && k > 0 && !mbar_wait_all(bar(C::B_OFREE), static_cast<uint32_t>(k - 1) & 1u, ctl))
          return false;
        tc_fence_after_sync();
        issue_pv(stage(load_base + jj), jj > 0);
        umma_commit_w(bar(C::B_PVDONE));
        umma_commit_w(bar(C::B_EMPTY + (load_base + jj) % C::NS));
        return true;
      };
      for (int j = 0; ok && j < n_kv; ++j) {
        const int gj = g + j, ld = load_base + j, bs = gj & 1;
        if (!(ok = mbar_wait_all(bar(C::B_CONV + ld % C::NS), static_cast<uint32_t>(ld / C::NS) & 1u, ctl))) break;
        // S buffer bs is free once the softmax of its previous tile (gj - 2) has read it.
        if (!(ok = mbar_wait_all(bar(C::B_SFREE + bs), (static_cast<uint32_t>(gj >> 1) & 1u) ^ 1u, ctl))) break;
        tc_fence_after_sync();
        issue_qk(stage(ld), tmem + (bs ? C::TM_S1 : C::TM_S0));
        umma_commit_w(bar(C::B_SFULL + bs));
        if (j + 1 == n_kv) umma_commit_w(bar(C::B_QEMPTY));  // last product reading Q
        if (j > 0 && !(ok = do_pv(j - 1))) break;
      }
      if (ok) ok = do_pv(n_kv - 1);
      g += n_kv;
      load_base += n_kv;
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------------ converter (warps 2-5)
    const int tid = threadIdx.x - 64;  // 0..127
    int load = 0;
    bool ok = true;
    for (int k = 0, w = blockIdx.x; ok && w < p.n_items; ++k, w += gridDim.x) {
      int b, h, q0, n_kv;
      geometry(w, b, h, q0, n_kv);
      if (!(ok = mbar_wait_all(bar(C::B_QFULL), static_cast<uint32_t>(k) & 1u, ctl))) break;
      // Q (32 KB) -> hi in place, lo alongside (same swizzled layout: the split is elementwise).
#pragma unroll 4
      for (int v = tid; v < C::Q_BYTES / 16; v += 128) split_v4(sQ + v * 16, sQ + v * 16, sQL + v * 16);
      fence_proxy_async_smem();
      mbar_arrive(bar(C::B_QCONV));
      for (int j = 0; ok && j < n_kv; ++j, ++load) {
        const int st = load % C::NS;
        if (!(ok = mbar_wait_all(bar(C::B_FULL + st), static_cast<uint32_t>(load / C::NS) & 1u, ctl))) break;
        const uint32_t sb = stage(load);
        // K -> hi in place, lo alongside.
#pragma unroll 4
        for (int v = tid; v < C::T_BYTES / 16; v += 128)
          split_v4(sb + C::ST_K + v * 16, sb + C::ST_K + v * 16, sb + C::ST_KL + v * 16);
        // V [key][d] -> V^T [d][key] hi / lo (K-major B operand: rows d, 64 keys in two 128-byte
        // chunks).  Thread -> (d = tid % 64, keys half*32 .. half*32+31).
        {
          const int d = tid & 63, half = tid >> 6;
          const uint32_t vsrc = sb + C::ST_V + (d >> 5) * C::KCH + (d & 3) * 4;
          const int du = (d & 31) >> 2;  // 16-byte unit of column d inside its 128-byte row
          const uint32_t dst_row = half * C::KCH + d * 128;
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
        fence_proxy_async_smem();
        mbar_arrive(bar(C::B_CONV + st));
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue (6-9)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    const float masked = p.neg_scale ? INFINITY : -INFINITY;
    int g = 0;
    bool ok = true;
    for (int k = 0, w = blockIdx.x; ok && w < p.n_items; ++k, w += gridDim.x) {
      int b, h, q0, n_kv;
      geometry(w, b, h, q0, n_kv);
      const int qrow = q0 + row;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < n_kv; ++j) {
        const int gj = g + j, bs = gj & 1;
        if (!(ok = mbar_wait_all(bar(C::B_SFULL + bs), static_cast<uint32_t>(gj >> 1) & 1u, ctl))) break;
        tc_fence_after_sync();
        uint32_t sr[64];
        tmem_ld64(lane_base + (bs ? C::TM_S1 : C::TM_S0), sr);
        float* s = reinterpret_cast<float*>(sr);
        tc_fence_before_sync();
        mbar_arrive(bar(C::B_SFREE + bs));
        const int kv0 = j * C::BN;
        if (kv0 + C::BN > p.len_k || (p.causal && kv0 + C::BN - 1 > q0)) {
          int lim = p.len_k - kv0;
          if (p.causal) lim = min(lim, qrow - kv0 + 1);
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= lim) s[c] = masked;
        }
        float mx = s[0];
        if (p.neg_scale) {
#pragma unroll
          for (int c = 1; c < 64; ++c) mx = fminf(mx, s[c]);
        } else {
#pragma unroll
          for (int c = 1; c < 64; ++c) mx = fmaxf(mx, s[c]);
        }
        const float m_tile = mx * sl2;
        float alpha = 1.f;
        if (m_run == -INFINITY || m_tile > m_run + 64.f) {
          const float m_new = fmaxf(m_run, m_tile);
          alpha = ex2_approx(m_run - m_new);
          m_run = m_new;
        }
        const float nm = (m_run == -INFINITY) ? 0.f : -m_run;
        float l0 = 0.f, l1 = 0.f;
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          s[c] = ex2_approx(fmaf(s[c], sl2, nm));
          s[c + 1] = ex2_approx(fmaf(s[c + 1], sl2, nm));
          l0 += s[c];
          l1 += s[c + 1];
        }
        l_run = l_run * alpha + (l0 + l1);
        // P buffers and O are free once the previous tile's PV is done (none before the first).
        if (j > 0) {
          if (!(ok = mbar_wait_all(bar(C::B_PVDONE), static_cast<uint32_t>(gj - 1) & 1u, ctl))) break;
          tc_fence_after_sync();
          if (__any_sync(0xffffffffu, alpha != 1.f)) {
            uint32_t o[64];
            tmem_ld64(lane_base + C::TM_O, o);
#pragma unroll
            for (int e = 0; e < 64; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              uint32_t part[32];
#pragma unroll
              for (int e = 0; e < 32; ++e) part[e] = o[hh * 32 + e];
              tmem_st32(lane_base + C::TM_O + hh * 32, part);
            }
          }
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t ph[32], pl[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const uint32_t bits = __float_as_uint(s[hh * 32 + e]);
            ph[e] = tf32_trunc(bits);
            pl[e] = __float_as_uint(s[hh * 32 + e] - __uint_as_float(ph[e]));
          }
          tmem_st32(lane_base + C::TM_PH + hh * 32, ph);
          tmem_st32(lane_base + C::TM_PL + hh * 32, pl);
        }
        tmem_st_wait();
        tc_fence_before_sync();
        mbar_arrive(bar(C::B_PREADY));
      }
      if (!ok) break;
      // Epilogue: O / l, fp32, straight to global memory (this thread's row).
      if (!(ok = mbar_wait_all(bar(C::B_PVDONE), static_cast<uint32_t>(g + n_kv - 1) & 1u, ctl))) break;
      tc_fence_after_sync();
      uint32_t o[64];
      tmem_ld64(lane_base + C::TM_O, o);
      tc_fence_before_sync();
      mbar_arrive(bar(C::B_OFREE));
      if (qrow < p.len_q) {
        const float inv_l = 1.f / l_run;
        float* dst = p.o + b * p.os_b + h * p.os_h + static_cast<long long>(qrow) * p.os_s;
        if ((p.head_dim & 3) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
#pragma unroll
          for (int c = 0; c < 64; c += 4)
            if (c < p.head_dim)
              *reinterpret_cast<float4*>(dst + c) =
                  make_float4(__uint_as_float(o[c]) * inv_l, __uint_as_float(o[c + 1]) * inv_l,
                              __uint_as_float(o[c + 2]) * inv_l, __uint_as_float(o[c + 3]) * inv_l);
        } else {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c < p.head_dim) dst[c] = __uint_as_float(o[c]) * inv_l;
        }
      }
      g += n_kv;
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == C::W_MMA) {
    if (*abort_flag) {
      __syncwarp();
      umma_commit_w(bar(C::B_DRAIN));
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
  if (d->dtype != CMPX_F32 || d->head_dim < 1 || d->head_dim > 64) return false;
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

int launch_attn_tf32x3(const cmpx_attn_desc* d, const LaunchCtx& ctx) {
  using C = X3Cfg;
  CUtensorMap tq, tk, tv;
  if (!make_map_f32(&tq, d->q, d->head_dim, d->len_q, d->heads, d->batch, d->q_stride, C::BM) ||
      !make_map_f32(&tk, d->k, d->head_dim, d->len_k, d->heads, d->batch, d->k_stride, C::BN) ||
      !make_map_f32(&tv, d->v, d->head_dim, d->len_k, d->heads, d->batch, d->v_stride, C::BN))
    return CMPX_ERR_LAUNCH;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(reinterpret_cast<const void*>(&attn_tf32x3_sm100_kernel),
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
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
  p.scale_log2 = static_cast<float>(d->scale * 1.4426950408889634);
  p.o = static_cast<float*>(d->o);
  p.os_b = d->o_stride[0];
  p.os_h = d->o_stride[1];
  p.os_s = d->o_stride[2];
  p.timeout_ns = ctx.timeout_ns;
  p.dev_flags = ctx.dev_flags;
  const int grid = std::min(p.n_items, std::max(1, ctx.num_sms));
  attn_tf32x3_sm100_kernel<<<grid, C::THREADS, C::SMEM_BYTES, ctx.stream>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

}  // namespace cmpx
