// attn_fwd_sm100.cu -- scaled-dot-product attention forward for fp16 / bf16 on B200 (sm_100a).
//
// Computes O = softmax(Q K^T * scale [+ top-left causal mask]) V for [B, H, L, D] views with a
// contiguous head dim, D <= 128.  This replaces the reference's two fp16 attention kernels
// (flash_attn_hfma2_kernel, src/cuda/fp16_flash_attention_hfma2.cu:72-243, non-causal; and
// flash_attention_fp16_optimized, src/cuda/fp16_attention.cu:135-319, causal, D=128) with one
// tensor-core kernel.  The algorithm is the same online-softmax forward (running row max m,
// running sum l, O rescaled when m grows, O / l at the end, exp2 domain with the scale folded
// in); the machinery is Blackwell's:
//
//   * one CTA owns two 128-row Q tiles (rows q0 .. q0+255) of one (batch, head);
//   * warp 8 streams K_j and V_j (128 keys x D) through a ring of shared-memory stages with TMA
//     (128-byte swizzle, OOB rows/cols zero-filled), Q once;
//   * warp 9 issues tcgen05.mma: S = Q_t K_j^T into TMEM (fp32; one S buffer the two tiles take
//     in turns), then O_t += P_t V_j with P_t read straight from TMEM (A-from-TMEM form) -- P never
//     touches shared memory;
//   * warps 0-3 / 4-7 are the softmax warpgroups of tile 0 / tile 1: thread i owns row i, reads
//     its 128 scores with tcgen05.ld and releases S at once, applies the mask, updates m and l,
//     writes P (16-bit) into its tile's P buffer with tcgen05.st, and rescales its O row in TMEM
//     when the running max grew by more than 2^8 (otherwise the stale max is kept: exact, since O
//     and l share it);
//   * the QK of one tile runs while the other tile's softmax -- and its own exponentials -- run.
//   * epilogue: O / l, converted, staged in the (now idle) Q buffer in the swizzled layout and
//     written with TMA stores that clip rows >= Lq and cols >= D.
//
// TMEM columns: S [0,128) (shared by the two tiles), P0 [128,192), P1 [192,256), O0, O1.
// Every wait is bounded (see cmpx_ptx.cuh); a CTA that gives up drains its in-flight copies
// and MMAs, frees TMEM, sets the device status word and returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <mutex>
#include <string>
#include <type_traits>

#include "cmpx_internal.h"
#include "cmpx_ptx.cuh"

// Causal launches: work items per CTA in the longest-first tail (0: no such tail).
#ifndef CMPX_FMHA_LPT
#define CMPX_FMHA_LPT 2
#endif

namespace cmpx {

// Most key ranges one item of the tail split is cut into.
constexpr int kMaxSplit = 8;

// Keys per K/V tile of an instantiation: 128; 64 for head dims above 128, where the two O
// accumulators take 2 x 192 TMEM columns and S / P0 / P1 have to fit in the 128 left, and for
// additive masks (MK = 2), whose values in flight would not fit the softmax's registers next to a
// 128-key row of scores.
template <int DP, int MK>
constexpr int fmha_bn() { return (DP > 128 || MK == 2) ? 64 : 128; }

template <int DP, int BN_ = fmha_bn<DP, 0>()>
struct FmhaCfg {
  static constexpr int BM = 128;                    // rows of one Q tile
  static constexpr int BN = BN_;                    // keys per K/V tile
  static constexpr int NCH = DP / 64;               // 128-byte chunks per row
  static constexpr int CH_BYTES = 128 * 128;        // one chunk of a 128-row (Q / O) tile
  static constexpr int KV_CH_BYTES = BN * 128;      // one chunk of a K / V tile
  static constexpr int QTILE_BYTES = NCH * CH_BYTES;
  static constexpr int KV_BYTES = NCH * KV_CH_BYTES;
  static constexpr int NSTAGE = DP > 128 ? 3 : DP == 128 ? 4 : 6;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = 2 * QTILE_BYTES;
  static constexpr int OFF_OST = OFF_KV + NSTAGE * KV_BYTES;   // O staging (one tile) for TMA stores
  static constexpr int OFF_BAR = OFF_OST + QTILE_BYTES;
  // barrier slots
  static constexpr int B_QFULL = 0;                 // Q of the current item landed
  static constexpr int B_QEMPTY = 1;                // last QK of an item done: Q may be reloaded
  static constexpr int B_FULL = 2;
  static constexpr int B_EMPTY = B_FULL + NSTAGE;
  static constexpr int B_SFULL = B_EMPTY + NSTAGE;  // [2] S holds tile t's scores
  static constexpr int B_SFREE = B_SFULL + 2;       // [2] tile t's softmax has read S
  static constexpr int B_PREADY = B_SFREE + 2;      // [2] P_t written
  static constexpr int B_PVDONE = B_PREADY + 2;     // [2] O_t += P_t V complete
  static constexpr int B_OFREE = B_PVDONE + 2;      // [2] epilogue has read O_t
  static constexpr int B_ITFULL = B_OFREE + 2;      // [2] work-item slot written
  static constexpr int B_ITEMPTY = B_ITFULL + 2;    // [2] work-item slot read by every consumer
  static constexpr int B_OST = B_ITEMPTY + 2;       // [2 tile][4 quarter] staging rows free for tile t
  static constexpr int B_DRAIN = B_OST + 8;
  static constexpr int NBAR = B_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // tmem base, abort word, item slots [2]
  static constexpr int SMEM_BYTES = OFF_MISC + 32 + 1024;  // +1024: runtime alignment slack
  // One S buffer shared by the two Q tiles (their QKs alternate), a P buffer per tile, an O
  // accumulator per tile: S [0,BN) P0 [BN,1.5BN) P1 [1.5BN,2BN) O0 [2BN,2BN+DP) O1 [2BN+DP, 2BN+2DP).
  static constexpr int TM_S = 0, TM_P0 = BN, TM_P1 = BN + BN / 2, TM_O0 = 2 * BN, TM_O1 = 2 * BN + DP;
  static_assert(TM_O1 + DP <= 512, "TMEM columns");
  static constexpr int TMEM_COLS = 512;
  // Warp roles: 0-3 softmax/epilogue of tile 0, 4-7 of tile 1 (thread = row), 8 TMA producer
  // (and work fetch), 9 QK issuer (and TMEM owner), 10 PV issuer.
  static constexpr int THREADS = 352;
  static constexpr int W_TMA = 8, W_MMA = 9, W_PV = 10;
  static constexpr int ITEM_CONSUMERS = 2 + 8;  // lane 0 of each MMA warp and of each softmax warp
};

struct FmhaParams {
  int heads;
  int len_q;
  int len_k;
  int n_pairs;        // ceil(len_q / 256)
  int n_items;        // n_pairs * heads * batch
  // Causal launches: items from lpt_first on (the last lpt_heads (b, h) slices) are dealt heaviest
  // row pair first across those slices, not slice by slice (n_items: no such tail).
  int lpt_first;
  int lpt_heads;
  int causal;
  int neg_scale;      // scale < 0: masked scores are +inf so that masked * scale = -inf
  float scale_log2;   // scale * log2(e)
  void* o;            // output [B, H, Lq, D] view
  long long os_b, os_h, os_s;  // its strides (elements)
  int head_dim;
  int group;                   // query heads per key/value head (grouped-query attention)
  unsigned int* work;          // [0] next work item, [1] CTAs finished (both 0 at launch and exit)
  // Tail split (non-causal): work items 0 .. n_whole-1 are whole (row pair, head) items; each item
  // after them is cut into `split` key ranges, one work item each (n_work items in all).  The
  // range's partial O (fp32, not normalised) and its row max / sum go to part_o / part_ml, and
  // fmha_split_merge_kernel merges them.
  int n_whole;
  int split;
  int n_work;
  float* part_ml;              // [n_work - n_whole][2][128] (m, l) pairs
  float* part_o;               // [n_work - n_whole][2][128][DP]
  // Boolean mask packed to bits (MK = 1): key j of query row i of (b, h) is bit j%32
  // of word mask_bits[b*mb_b + h*mb_h + i*mb_q + j/32] (strides in words, 0 = broadcast); rows
  // hold a multiple of 4 words, so each 128-key tile's bits are one aligned 16-byte load.
  const uint32_t* mask_bits;
  long long mb_b, mb_h, mb_q;
  // Additive mask (MK = 2): 16-bit values in the call's type at mask_add[b*ma_b + h*ma_h + i*ma_q + j]
  // (element strides, 0 = broadcast; rows 16-byte aligned), added to the scores as value / scale.
  const uint16_t* mask_add;
  long long ma_b, ma_h, ma_q;
  float mask_inv_scale;
  unsigned long long timeout_ns;
  unsigned int* dev_flags;
};

// Work item -> (b*heads + h, row pair).  Items of one (b, h) slice are consecutive and within a slice
// the heavy (late, causal) row pairs go first, so the CTAs busy at any moment share a few slices' K/V
// in L2.  The last lpt_heads slices are dealt heaviest row pair first across all of them instead
// (longest-processing-time order): dealt slice by slice, the last slice's heaviest pair would start
// shortly before the work runs out and finish long after every other CTA.
__device__ __forceinline__ void item_slice_pair(const FmhaParams& p, int item, int& bh, int& pair) {
  if (item < p.lpt_first) {
    bh = item / p.n_pairs;
    pair = p.n_pairs - 1 - (item - bh * p.n_pairs);
  } else {
    const int t = item - p.lpt_first;
    const int r = t / p.lpt_heads;
    bh = p.lpt_first / p.n_pairs + (t - r * p.lpt_heads);
    pair = p.n_pairs - 1 - r;
  }
}

// Packs a boolean mask (one byte per element, nonzero = the key takes part; element strides sb, sh,
// sq over the packed extents nb x nh x nq, keys contiguous) to bits: one warp per mask row, one
// ballot per 32 keys; words past the last key are 0.
__global__ void __launch_bounds__(256) fmha_pack_mask_kernel(const uint8_t* __restrict__ mask,
                                                             long long sb, long long sh, long long sq,
                                                             int nh, int nq, int len_k, int words,
                                                             long long rows, uint32_t* __restrict__ bits) {
  const long long row = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const long long q = row % nq;
  const long long bh = row / nq;
  const long long src = (bh / nh) * sb + (bh % nh) * sh + q * sq;
#pragma unroll 4
  for (int w = 0; w < words; ++w) {
    const int key = w * 32 + lane;
    const bool on = key < len_k && mask[src + key] != 0;
    const uint32_t word = __ballot_sync(0xffffffffu, on);
    if (lane == 0) bits[row * words + w] = word;
  }
}

// One chunk (16 column pairs = 32 keys) of a row's exponentials: p = 2^(s*sl2 + nmb) packed to
// 16-bit pairs in pk, the row sum accumulated in la/lb.  x = s*sl2 + nmb is formed and the sum
// accumulated two keys at a time with packed f32x2 arithmetic; exponentials on MUFU.
template <bool BF16>
__device__ __forceinline__ void exp_chunk(const float* s, int q, uint64_t sl2x2, uint64_t nmbx2,
                                          uint64_t& la, uint64_t& lb, uint32_t (&pk)[16]) {
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const int cc = q * 16 + c;
    const uint64_t xv = f2_fma(f2_pack(s[2 * cc], s[2 * cc + 1]), sl2x2, nmbx2);
    float x0, x1;
    f2_unpack(xv, x0, x1);
    const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
    if (c & 1)
      lb = f2_add(lb, f2_pack(p0, p1));
    else
      la = f2_add(la, f2_pack(p0, p1));
    pk[c] = BF16 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
  }
}

// One pass over a row's BN scores: the BN/32 chunks' P stored to TMEM (16 columns each at p_tm);
// returns the row sum of p.  before_store() runs after the first chunk is computed and before
// anything is stored: the wait for the P buffer to be free (the previous PV) overlaps the first
// chunk of the exponentials instead of preceding them.
template <int BN, bool BF16, class BeforeStore>
__device__ __forceinline__ float exp_pass(const float* s, float sl2, float nmb, uint32_t p_tm,
                                          BeforeStore&& before_store) {
  uint64_t la = f2_pack(0.f, 0.f), lb = la;
  const uint64_t sl2x2 = f2_pack(sl2, sl2), nmbx2 = f2_pack(nmb, nmb);
  uint32_t pk[16];
  exp_chunk<BF16>(s, 0, sl2x2, nmbx2, la, lb, pk);
  before_store();
#pragma unroll
  for (int q = 0; q < BN / 32; ++q) {
    if (q > 0) exp_chunk<BF16>(s, q, sl2x2, nmbx2, la, lb, pk);
    tmem_st16(p_tm + q * 16, pk);
  }
  float a0, a1;
  f2_unpack(f2_add(la, lb), a0, a1);
  return a0 + a1;
}

// Row maximum / minimum of BN values: 8 independent chains, the first 16 values seed them in pairs,
// the others follow two at a time with the 3-input form.
template <int BN>
__device__ __forceinline__ float row_max(const float* s) {
  float a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = fmaxf(s[2 * i], s[2 * i + 1]);
#pragma unroll
  for (int c = 16; c < BN; c += 16)
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = fmax3(a[i], s[c + 2 * i], s[c + 2 * i + 1]);
  return fmax3(fmax3(a[0], a[1], a[2]), fmax3(a[3], a[4], a[5]), fmaxf(a[6], a[7]));
}
template <int BN>
__device__ __forceinline__ float row_min(const float* s) {
  float a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = fminf(s[2 * i], s[2 * i + 1]);
#pragma unroll
  for (int c = 16; c < BN; c += 16)
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = fmin3(a[i], s[c + 2 * i], s[c + 2 * i + 1]);
  return fmin3(fmin3(a[0], a[1], a[2]), fmin3(a[3], a[4], a[5]), fminf(a[6], a[7]));
}

// Epilogue of one key range of a split item, for the calling warp's 32 rows of tile t (thread =
// row): the row's O (fp32, scaled by 2^-m) and (m, l) go to the range's slot, and O_t is released
// (ofree_bar).  fmha_split_merge_kernel, launched next on the stream, merges the ranges.
// (Not inlined: its registers stay out of the softmax loop's allocation.)
template <int DP>
__device__ __noinline__ void fmha_split_epilogue(float* part_o, float* part_ml, int part, int t,
                                                 int row, float m_run, float l_run, uint32_t o_tm,
                                                 uint32_t ofree_bar) {
  const size_t slot = (static_cast<size_t>(part) * 2 + t) * 128 + row;
  float* po = part_o + slot * DP;
#pragma unroll 1
  for (int c = 0; c < DP / 32; ++c) {
    uint32_t o[32];
    tmem_ld32(o_tm + c * 32, o);
    if (c == DP / 32 - 1) {
      tc_fence_before_sync();
      mbar_arrive(ofree_bar);  // O_t is read: the next item may overwrite it
    }
#pragma unroll
    for (int e = 0; e < 32; e += 4)
      *reinterpret_cast<uint4*>(po + c * 32 + e) = make_uint4(o[e], o[e + 1], o[e + 2], o[e + 3]);
  }
  reinterpret_cast<float2*>(part_ml)[slot] = make_float2(m_run, l_run);
}

// Merge of the split items' key ranges: for each of their rows, O = sum_r 2^(m_r - M) O_r /
// sum_r 2^(m_r - M) l_r with M = max_r m_r -- the online-softmax rescale step applied across
// ranges instead of across key tiles -- written as the 16-bit output row.  A warp takes 2 rows
// (one after the other in the row order of the ranges' slots); lane l takes columns
// [l*CPL, (l+1)*CPL) of every range's row, so every load is one contiguous row.  Spread over
// ~rows/32 CTAs, the merge costs a round trip or two to L2 per warp; done by the last range's own
// CTA it was bound by the loads one SM can keep in flight.
template <int DP, bool BF16>
__global__ void __launch_bounds__(128) fmha_split_merge_kernel(const __grid_constant__ FmhaParams p) {
  constexpr int CPL = DP / 32;  // fp32 columns per lane: 2, 4 or 6
  constexpr int ROWS = 2;       // rows per warp
  const int lane = threadIdx.x & 31;
  const int col = lane * CPL;
  const int split = p.split;
  const int n_rows = (p.n_items - p.n_whole) * 256;
  const int r0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * ROWS;
  float2 ml[ROWS][kMaxSplit];
  float o[ROWS][kMaxSplit][CPL];
#pragma unroll
  for (int i = 0; i < ROWS; ++i) {
    const int gr = min(r0 + i, n_rows - 1);  // (rows past the end repeat the last; not stored)
    const int item = p.n_whole + gr / 256;
    const int tr = gr % 256;
    const size_t slot0 = (static_cast<size_t>(item - p.n_whole) * split * 2 + tr / 128) * 128 + tr % 128;
#pragma unroll
    for (int r = 0; r < kMaxSplit; ++r) {
      const size_t slot = slot0 + static_cast<size_t>(r) * 2 * 128;
      if (r < split) {
        ml[i][r] = __ldcg(reinterpret_cast<const float2*>(p.part_ml) + slot);
        if constexpr (CPL == 4) {
          const float4 x = ld_cg_f4(p.part_o + slot * DP + col);
          o[i][r][0] = x.x;
          o[i][r][1] = x.y;
          o[i][r][2] = x.z;
          o[i][r][3] = x.w;
        } else {
#pragma unroll
          for (int e = 0; e < CPL; e += 2) {
            const float2 x = ld_cg_f2(p.part_o + slot * DP + col + e);
            o[i][r][e] = x.x;
            o[i][r][e + 1] = x.y;
          }
        }
      } else {
        ml[i][r] = make_float2(-INFINITY, 0.f);
#pragma unroll
        for (int e = 0; e < CPL; ++e) o[i][r][e] = 0.f;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < ROWS; ++i) {
    const int gr = r0 + i;
    if (gr >= n_rows) break;
    const int item = p.n_whole + gr / 256;
    int bh, pair;
    item_slice_pair(p, item, bh, pair);
    const int b = bh / p.heads;
    const int h = bh - b * p.heads;
    const int qrow = pair * 256 + gr % 256;
    if (qrow >= p.len_q) continue;
    float mx = -INFINITY;
#pragma unroll
    for (int r = 0; r < kMaxSplit; ++r) mx = fmaxf(mx, ml[i][r].x);
    float a[CPL];
#pragma unroll
    for (int e = 0; e < CPL; ++e) a[e] = 0.f;
    float lsum = 0.f;
    // (ranges in which a masked row has no key: m = -inf, l = 0, O = 0 -- weight 0)
#pragma unroll
    for (int r = 0; r < kMaxSplit; ++r) {
      const float w = (r < split && ml[i][r].x > -INFINITY) ? ex2_approx(ml[i][r].x - mx) : 0.f;
      lsum += w * ml[i][r].y;
#pragma unroll
      for (int e = 0; e < CPL; ++e) a[e] += w * o[i][r][e];
    }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;  // a row with no key at all: output 0
    uint16_t* dst = static_cast<uint16_t*>(p.o) + b * p.os_b + h * p.os_h +
                    static_cast<long long>(qrow) * p.os_s + col;
    // column pairs inside the head dim (a multiple of 8, so a pair is all in or all out)
#pragma unroll
    for (int e = 0; e < CPL; e += 2)
      if (col + e < p.head_dim)
        *reinterpret_cast<uint32_t*>(dst + e) =
            BF16 ? pack_bf16x2(a[e] * inv, a[e + 1] * inv) : pack_f16x2(a[e] * inv, a[e + 1] * inv);
  }
}

// Persistent schedule: CTAs take work items from a counter; item_slice_pair gives each item's (b, h)
// slice and row pair.  SPLIT: the launch has a tail split;
// MK: no mask (0), a boolean mask packed to bits (1), an additive 16-bit mask (2) -- separate
// instantiations, so that plain launches run their code unchanged.
template <int DP, bool BF16, bool SPLIT, int MK>
__global__ void __launch_bounds__(352, 1)
    fmha_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_o,
                          const __grid_constant__ FmhaParams p) {
  using C = FmhaCfg<DP, fmha_bn<DP, MK>()>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_base);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const uint32_t sQ = base + C::OFF_Q;
  const uint32_t sKV = base + C::OFF_KV;
  auto bar = [&](int i) -> uint32_t { return base + C::OFF_BAR + 8u * i; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  volatile int* item_slot = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 8);  // [2]

  if (threadIdx.x == 0) {
    mbar_init(bar(C::B_QFULL), 1);
    mbar_init(bar(C::B_QEMPTY), 1);
    for (int s = 0; s < C::NSTAGE; ++s) {
      mbar_init(bar(C::B_FULL + s), 1);
      mbar_init(bar(C::B_EMPTY + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(C::B_SFULL + t), 1);
      mbar_init(bar(C::B_SFREE + t), 128);
      mbar_init(bar(C::B_PREADY + t), 128);
      mbar_init(bar(C::B_PVDONE + t), 1);
      mbar_init(bar(C::B_OFREE + t), 128);
      mbar_init(bar(C::B_ITFULL + t), 1);
      mbar_init(bar(C::B_ITEMPTY + t), C::ITEM_CONSUMERS);
    }
    for (int i = 0; i < 8; ++i) mbar_init(bar(C::B_OST + i), 1);
    mbar_init(bar(C::B_DRAIN), 2);  // one commit from each MMA warp
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

  // Item k of this CTA: wait for its slot, read it, release the slot (consumers only).
  auto next_item = [&](int k, int& w) -> bool {
    const int slot = k & 1;
    if (!mbar_wait(bar(C::B_ITFULL + slot), static_cast<uint32_t>(k >> 1) & 1u, ctl)) return false;
    w = item_slot[slot];
    mbar_arrive(bar(C::B_ITEMPTY + slot));
    return true;
  };
  // Same for a whole warp: a warp-wide wait, every lane reads the slot, lane 0 releases it.
  auto next_item_warp = [&](int k, int& w) -> bool {
    const int slot = k & 1;
    if (!mbar_wait_all(bar(C::B_ITFULL + slot), static_cast<uint32_t>(k >> 1) & 1u, ctl)) return false;
    w = item_slot[slot];
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(C::B_ITEMPTY + slot));
    return true;
  };
  // Work item w -> (b, h, rows q0 .. q0+255, key tiles [j0, j1) of the item's n_kv); part >= 0 is
  // the index of a split item's key range among all ranges (-1: whole item).
  struct Work {
    int b, h, q0, n_kv, j0, j1, item, part;
  };
  auto work_geometry = [&](int w) -> Work {
    Work g;
    g.item = w;
    g.part = -1;
    if (SPLIT && w >= p.n_whole) {
      g.part = w - p.n_whole;
      g.item = p.n_whole + g.part / p.split;
    }
    int bh, pair;
    item_slice_pair(p, g.item, bh, pair);
    g.b = bh / p.heads;
    g.h = bh - g.b * p.heads;
    g.q0 = pair * 256;
    const int kv_len = p.causal ? min(p.len_k, g.q0 + 256) : p.len_k;
    g.n_kv = (kv_len + C::BN - 1) / C::BN;
    g.j0 = 0;
    g.j1 = g.n_kv;
    if (SPLIT && g.part >= 0) {  // (the host splits only non-causal calls, with n_kv >= 4 * split)
      const int r = g.part - (g.item - p.n_whole) * p.split;
      g.j0 = r * g.n_kv / p.split;
      g.j1 = (r + 1) * g.n_kv / p.split;
    }
    return g;
  };
  // Key tiles tile 0 of an item takes part in: under the causal mask its rows (q0 .. q0+127) see no
  // key past q0 + 127, so QK_0, its softmax and PV_0 skip the item's last key tiles that start
  // past it (one tile of 128 keys, two of 64).
  auto tile0_kv = [&](int q0, int n_kv) -> int {
    return p.causal ? min(n_kv, (min(p.len_k, q0 + C::BM) + C::BN - 1) / C::BN) : n_kv;
  };

  if (warp >= 8) {
    if (warp == C::W_TMA) {
      // ---------------------------------------------------------------- work fetch + TMA producer
      if (lane == 0) {
        int load = 0;  // K/V ring loads issued so far (K_j and V_j of every item, in order)
        bool ok = true;
        bool took_range = false;
        for (int k = 0; ok; ++k) {
          const int slot = k & 1;
          if (!(ok = mbar_wait(bar(C::B_ITEMPTY + slot), (static_cast<uint32_t>(k >> 1) & 1u) ^ 1u, ctl))) break;
          // Whole items come from the shared counter.  The split items' key ranges (never more
          // than CTAs) are dealt one per CTA, range blockIdx.x: drawn from the counter, a CTA
          // whose producer runs ahead -- it takes its next item as soon as it has issued the
          // current one's loads, which for a short range is early -- would take several.
          const int wi = static_cast<int>(atomicAdd(p.work, 1u));
          int w = wi < p.n_whole ? wi : -1;
          if (SPLIT && w < 0 && !took_range && static_cast<int>(blockIdx.x) < p.n_work - p.n_whole) {
            w = p.n_whole + static_cast<int>(blockIdx.x);
            took_range = true;
          }
          item_slot[slot] = w;
          mbar_arrive(bar(C::B_ITFULL + slot));
          if (w < 0) break;
          const Work g = work_geometry(w);
          const int b = g.b, h = g.h, q0 = g.q0;
          if (k > 0 && !(ok = mbar_wait(bar(C::B_QEMPTY), static_cast<uint32_t>(k - 1) & 1u, ctl))) break;
          mbar_arrive_expect_tx(bar(C::B_QFULL), 2 * C::QTILE_BYTES);
          for (int t = 0; t < 2; ++t)
            for (int c = 0; c < C::NCH; ++c)
              tma_load_4d(sQ + t * C::QTILE_BYTES + c * C::CH_BYTES, &tm_q, bar(C::B_QFULL), c * 64,
                          q0 + t * C::BM, h, b);
          for (int j = g.j0; ok && j < g.j1; ++j) {
            for (int which = 0; which < 2; ++which, ++load) {
              const int st = load % C::NSTAGE;
              const uint32_t rnd = static_cast<uint32_t>(load / C::NSTAGE);
              if (!(ok = mbar_wait(bar(C::B_EMPTY + st), (rnd & 1u) ^ 1u, ctl))) break;
              mbar_arrive_expect_tx(bar(C::B_FULL + st), C::KV_BYTES);
              const CUtensorMap* m = which ? &tm_v : &tm_k;
              for (int c = 0; c < C::NCH; ++c)
                tma_load_4d(sKV + st * C::KV_BYTES + c * C::KV_CH_BYTES, m, bar(C::B_FULL + st), c * 64,
                            j * C::BN, h / p.group, b);
            }
          }
        }
        if (*abort_flag) {
          // Let every copy still in flight land before shared memory goes away.
          for (int i = max(0, load - C::NSTAGE); i < load; ++i)
            mbar_wait_drain(bar(C::B_FULL + i % C::NSTAGE), static_cast<uint32_t>(i / C::NSTAGE) & 1u,
                            p.timeout_ns);
        }
      }
    } else {
      // ---------------------------------------------------------------- MMA issuers
      // Two issuing warps feed the one tensor pipe: W_MMA issues the QK products, W_PV the PV
      // products.  The pipe's queue is only a few MMAs deep and every MMA issue costs the issuing
      // thread a good part of an MMA's execution time, so one warp alone lets the pipe drain
      // while it does the bookkeeping (barrier waits, commits) between two products; with two,
      // one warp's MMAs keep the pipe busy while the other waits.  Each warp runs its loop with
      // warp-uniform control flow (waits are warp-wide and return one verdict) and one elected
      // lane issues its MMAs and commits (the *_w helpers).  The two streams touch disjoint TMEM
      // (QK: S;  PV: P_t, O_t); every cross-dependency goes through an mbarrier.
      constexpr uint32_t kIdescQK = idesc_f16(128, C::BN, BF16 ? 1 : 0, 0, 0);
      constexpr uint32_t kIdescPV = idesc_f16(128, DP, BF16 ? 1 : 0, 0, 1);
      auto stage_of = [&](int load) -> uint32_t { return sKV + (load % C::NSTAGE) * C::KV_BYTES; };
      auto full_bar = [&](int load) -> uint32_t { return bar(C::B_FULL + load % C::NSTAGE); };
      auto empty_bar = [&](int load) -> uint32_t { return bar(C::B_EMPTY + load % C::NSTAGE); };
      auto round_par = [&](int load) -> uint32_t { return static_cast<uint32_t>(load / C::NSTAGE) & 1u; };
      int base_load = 0;  // K/V ring loads of the items before this one (K_j = +2j, V_j = +2j+1)
      bool ok = true;
      if (warp == C::W_MMA) {
        // QK_t(j) = Q_t K_j^T into S.  Order per key tile j:  QK_1(j) once tile 0 has read S(j);
        // QK_0(j+1) once tile 1 has read S(j).  Tile 0 stops after n_kv0 key tiles (tile0_kv).
        auto issue_qk = [&](int t, uint32_t k_addr) {
          const uint32_t q_addr = sQ + t * C::QTILE_BYTES;
#pragma unroll
          for (int k = 0; k < DP / 16; ++k) {
            const uint32_t q_off = (k >> 2) * C::CH_BYTES + (k & 3) * 32;
            const uint32_t k_off = (k >> 2) * C::KV_CH_BYTES + (k & 3) * 32;
            umma_ss_w(tmem + C::TM_S, smem_desc_sw128(q_addr + q_off, 16, 1024),
                      smem_desc_sw128(k_addr + k_off, 16, 1024), kIdescQK, k > 0 ? 1u : 0u);
          }
        };
        uint32_t n_sfree0 = 0, n_sfree1 = 0;  // barrier phase counters carried across items
        for (int k = 0; ok; ++k) {
          int w;
          if (!(ok = next_item_warp(k, w))) break;
          if (w < 0) break;
          const Work g = work_geometry(w);
          const int n_kv0 = tile0_kv(g.q0, g.n_kv);  // (split items are non-causal: n_kv0 = n_kv)
          if (!(ok = mbar_wait_all(bar(C::B_QFULL), static_cast<uint32_t>(k) & 1u, ctl))) break;
          // S is free once tile 1's softmax read the previous item's last S.
          if (k > 0 && !(ok = mbar_wait_all(bar(C::B_SFREE + 1), (n_sfree1++) & 1u, ctl))) break;
          if (!(ok = mbar_wait_all(full_bar(base_load), round_par(base_load), ctl))) break;
          tc_fence_after_sync();
          issue_qk(0, stage_of(base_load));
          umma_commit_w(bar(C::B_SFULL + 0));
          for (int j = g.j0; ok && j < g.j1; ++j) {
            const int lk = base_load + 2 * (j - g.j0), lk1 = lk + 2;
            if (j < n_kv0 && !(ok = mbar_wait_all(bar(C::B_SFREE + 0), (n_sfree0++) & 1u, ctl))) break;
            tc_fence_after_sync();
            issue_qk(1, stage_of(lk));
            umma_commit_w(bar(C::B_SFULL + 1));
            umma_commit_w(empty_bar(lk));  // K_j done
            if (j + 1 == g.j1) {
              umma_commit_w(bar(C::B_QEMPTY));  // last QK of the item
              break;
            }
            if (!(ok = mbar_wait_all(bar(C::B_SFREE + 1), (n_sfree1++) & 1u, ctl))) break;
            if (!(ok = mbar_wait_all(full_bar(lk1), round_par(lk1), ctl))) break;
            if (j + 1 < n_kv0) {
              tc_fence_after_sync();
              issue_qk(0, stage_of(lk1));
              umma_commit_w(bar(C::B_SFULL + 0));
            }
          }
          base_load += 2 * (g.j1 - g.j0);
        }
      } else {
        // O_t += P_t V_j, P_t from TMEM (16-bit, two keys per 32-bit column).  Order per key tile
        // j: PV_0(j) once P_0(j) is written, PV_1(j) once P_1(j) is written; the first PV_t of an
        // item overwrites O_t, so it also waits for the previous item's epilogue to have read O_t.
        auto issue_pv = [&](int t, uint32_t v_addr, bool acc) {
          const uint32_t p_tmem = tmem + (t ? C::TM_P1 : C::TM_P0);
          const uint32_t d_tmem = tmem + (t ? C::TM_O1 : C::TM_O0);
#pragma unroll
          for (int k = 0; k < C::BN / 16; ++k) {
            umma_ts_w(d_tmem, p_tmem + k * 8,
                      smem_desc_sw128(v_addr + k * 2048, C::KV_CH_BYTES, 1024), kIdescPV,
                      (acc || k > 0) ? 1u : 0u);
          }
        };
        uint32_t n_pready0 = 0, n_pready1 = 0;
        for (int k = 0; ok; ++k) {
          int w;
          if (!(ok = next_item_warp(k, w))) break;
          if (w < 0) break;
          const Work g = work_geometry(w);
          const int n_kv0 = tile0_kv(g.q0, g.n_kv);
          for (int j = g.j0; ok && j < g.j1; ++j) {
            const int lv = base_load + 2 * (j - g.j0) + 1;
            if (!(ok = mbar_wait_all(full_bar(lv), round_par(lv), ctl))) break;
            if (j < n_kv0) {
              if (!(ok = mbar_wait_all(bar(C::B_PREADY + 0), (n_pready0++) & 1u, ctl))) break;
              if (j == g.j0 && k > 0 &&
                  !(ok = mbar_wait_all(bar(C::B_OFREE + 0), static_cast<uint32_t>(k - 1) & 1u, ctl)))
                break;
              tc_fence_after_sync();
              issue_pv(0, stage_of(lv), j > g.j0);
              umma_commit_w(bar(C::B_PVDONE + 0));
            }
            if (!(ok = mbar_wait_all(bar(C::B_PREADY + 1), (n_pready1++) & 1u, ctl))) break;
            if (j == g.j0 && k > 0 &&
                !(ok = mbar_wait_all(bar(C::B_OFREE + 1), static_cast<uint32_t>(k - 1) & 1u, ctl)))
              break;
            tc_fence_after_sync();
            issue_pv(1, stage_of(lv), j > g.j0);
            umma_commit_w(bar(C::B_PVDONE + 1));
            umma_commit_w(empty_bar(lv));  // V_j done (read by both tiles' PVs)
          }
          base_load += 2 * (g.j1 - g.j0);
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    const int t = warp >> 2;            // Q tile of this warpgroup
    const int wq = warp & 3;            // TMEM lane quarter of this warp
    const int row = wq * 32 + lane;     // row inside the tile
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    const uint32_t s_tm = lane_base + C::TM_S;
    const uint32_t p_tm = lane_base + (t ? C::TM_P1 : C::TM_P0);
    const uint32_t o_tm = lane_base + (t ? C::TM_O1 : C::TM_O0);
    const float sl2 = p.scale_log2;
    const float masked = p.neg_scale ? INFINITY : -INFINITY;  // masked * sl2 == -inf
    uint32_t n_sfull = 0, n_pvdone = 0;  // barrier phase counters carried across items
    bool ok = true;

    for (int k = 0; ok; ++k) {
      int w = -1;
      if (lane == 0) ok = next_item(k, w);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!ok || w < 0) break;
      int q0, j_begin, j_end;  // (the rest of the geometry is recomputed for the epilogue)
      const uint32_t* mrow = nullptr;  // (MK 1) this row's mask words
      const uint16_t* arow = nullptr;  // (MK 2) this row's additive mask values
      {
        const Work g = work_geometry(w);
        q0 = g.q0;
        j_begin = g.j0;
        j_end = t == 0 ? min(g.j1, tile0_kv(q0, g.n_kv)) : g.j1;
        const int r = q0 + t * C::BM + row;
        if constexpr (MK == 1) {
          if (r < p.len_q) mrow = p.mask_bits + g.b * p.mb_b + g.h * p.mb_h + r * p.mb_q;
        } else if constexpr (MK == 2) {
          if (r < p.len_q) arow = p.mask_add + g.b * p.ma_b + g.h * p.ma_h + r * p.ma_q;
        }
      }
      const int qrow = q0 + t * C::BM + row;
      float m_run = -INFINITY;  // running max of s * scale * log2(e)
      float l_run = 0.f;

      for (int j = j_begin; j < j_end; ++j) {
        // (MK 1) this tile's mask bits, (MK 2) its first 32 additive values: loaded before the
        // wait for S so the load overlaps it
        const int kv_first = j * C::BN;
        uint32_t mw[C::BN / 32];
        uint4 acur[4];
        auto load_add = [&](int c, uint4 (&v)[4]) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = kv_first + c * 32 + e * 8;
            v[e] = (arow && key < p.len_k) ? __ldg(reinterpret_cast<const uint4*>(arow + key))
                                           : make_uint4(0u, 0u, 0u, 0u);
          }
        };
        if constexpr (MK == 2) load_add(0, acur);
        if constexpr (MK == 1) {
          if (mrow) {
            if constexpr (C::BN == 128) {
              const uint4 v = __ldg(reinterpret_cast<const uint4*>(mrow) + j);
              mw[0] = v.x; mw[1] = v.y; mw[2] = v.z; mw[3] = v.w;
            } else {
              const uint2 v = __ldg(reinterpret_cast<const uint2*>(mrow) + j);
              mw[0] = v.x; mw[1] = v.y;
            }
          } else {
#pragma unroll
            for (int i = 0; i < C::BN / 32; ++i) mw[i] = ~0u;  // rows past Lq: not stored
          }
        }
        if (!mbar_wait_all(bar(C::B_SFULL + t), (n_sfull++) & 1u, ctl)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        uint32_t sr[C::BN];
        if constexpr (C::BN == 128) {
          tmem_ld128(s_tm, sr);
        } else {
          tmem_ld32(s_tm, *reinterpret_cast<uint32_t(*)[32]>(sr));
          tmem_ld32(s_tm + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
        }
        float* s = reinterpret_cast<float*>(sr);
        if constexpr (MK == 1) {
#pragma unroll
          for (int c = 0; c < C::BN; ++c)
            if (!((mw[c >> 5] >> (c & 31)) & 1u)) s[c] = masked;
        } else if constexpr (MK == 2) {
          // s += mask / scale (so that s * scale = q.k * scale + mask), chunk by chunk with the
          // next chunk's values in flight
#pragma unroll
          for (int c = 0; c < C::BN / 32; ++c) {
            uint4 anext[4];
            if (c + 1 < C::BN / 32) load_add(c + 1, anext);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t wds[4] = {acur[e].x, acur[e].y, acur[e].z, acur[e].w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int idx = c * 32 + e * 8 + 2 * i;
                const float lo = BF16 ? __uint_as_float(wds[i] << 16) : __half2float(__ushort_as_half(wds[i] & 0xffffu));
                const float hi = BF16 ? __uint_as_float(wds[i] & 0xffff0000u) : __half2float(__ushort_as_half(wds[i] >> 16));
                s[idx] = fmaf(lo, p.mask_inv_scale, s[idx]);
                s[idx + 1] = fmaf(hi, p.mask_inv_scale, s[idx + 1]);
              }
            }
            if (c + 1 < C::BN / 32) {
#pragma unroll
              for (int e = 0; e < 4; ++e) acur[e] = anext[e];
            }
          }
        }
        tc_fence_before_sync();
        mbar_arrive(bar(C::B_SFREE + t));  // S is in registers: the other tile's QK may overwrite it

        const int kv0 = j * C::BN;
        if ((kv0 + C::BN > p.len_k) || (p.causal && kv0 + C::BN - 1 > q0 + t * C::BM)) {
          int lim = p.len_k - kv0;
          if (p.causal) lim = min(lim, qrow - kv0 + 1);
#pragma unroll
          for (int c = 0; c < C::BN; ++c)
            if (c >= lim) s[c] = masked;
        }
        // Fast pass against the running max m_run.  Any p above 2^8 (a key more than 8 above
        // m_run in log2 units) forces the tile's row sum above 256, so a row sum <= 256 proves the
        // stale max is usable (exact: O, l and P share it).  Otherwise -- and on a row's first
        // tile, where m_run is still -inf -- the warp takes the slow path: exact tile max, new
        // running max, P recomputed, l and O rescaled.  After a slow pass m_run is the true running
        // max, so later triggers are rare.  (The first key of a work item's range is never masked,
        // so m_run is finite after its first tile.)  P_t and O_t are free once PV_t(j-1) has
        // completed: the fast pass waits for that between computing and storing its first half (no
        // wait on a range's first tile: the previous item's epilogue already waited for its last PV).
        float l_tile = 0.f;
        float alpha = 1.f;
        bool slow = (j == j_begin);
        if (!slow) {
          bool pv_ok = true;
          l_tile = exp_pass<C::BN, BF16>(s, sl2, -m_run, p_tm, [&] {
            pv_ok = mbar_wait_all(bar(C::B_PVDONE + t), (n_pvdone++) & 1u, ctl);
            tc_fence_after_sync();
          });
          if (!pv_ok) {
            ok = false;
            break;
          }
          slow = __any_sync(0xffffffffu, !(l_tile <= 256.f));
          if (slow) tmem_st_wait();  // the redo overwrites the fast pass's P columns
        }
        if (slow) {
          const float m_tile = (p.neg_scale ? row_min<C::BN>(s) : row_max<C::BN>(s)) * sl2;
          if (m_tile > m_run) {  // (always on the first tile: m_run = -inf, m_tile finite)
            alpha = ex2_approx(m_run - m_tile);
            m_run = m_tile;
          }
          // (a masked row with no key left so far keeps m_run = -inf; its p are 0, not NaN)
          const float nm = (MK != 0 && m_run == -INFINITY) ? 0.f : -m_run;
          l_tile = exp_pass<C::BN, BF16>(s, sl2, nm, p_tm, [] {});
          if (j > j_begin && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
            for (int c = 0; c < DP / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(o_tm + c * 32, o);
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
              tmem_st32(o_tm + c * 32, o);
            }
          }
        }
        l_run = l_run * alpha + l_tile;
        tmem_st_wait();
        tc_fence_before_sync();
        mbar_arrive(bar(C::B_PREADY + t));
      }
      if (!ok) break;

      // Epilogue: O_t / l, 16-bit, staged in shared memory (swizzled) and written with TMA stores
      // that clip rows >= Lq and columns >= D.  The staging buffer holds one tile: the two tiles
      // take turns per 32-row quarter (tile 0 of item k waits for tile 1 of item k-1 and vice versa).
      if (!(ok = mbar_wait_all(bar(C::B_PVDONE + t), (n_pvdone++) & 1u, ctl))) break;
      tc_fence_after_sync();
      const Work g = work_geometry(w);
      const int b = g.b, h = g.h;
      // (a masked row with no key left has l = 0 and O = 0: output 0, as torch)
      const float inv_l = (MK != 0 && !(l_run > 0.f)) ? 0.f : 1.f / l_run;
      const uint32_t turn_bar = bar(C::B_OST + t * 4 + wq);
      if (t == 1 || k > 0) {
        const uint32_t par = t == 1 ? static_cast<uint32_t>(k) & 1u : static_cast<uint32_t>(k - 1) & 1u;
        if (!(ok = mbar_wait_all(turn_bar, par, ctl))) break;
      }
      if (SPLIT && g.part >= 0) {
        // A key range of a split item: park this row's partial result for the merge kernel.  The
        // staging turn is taken and handed straight on, unused (the turn order of later items
        // stays as it is).
        if (lane == 0) mbar_arrive(bar(C::B_OST + (1 - t) * 4 + wq));
        __syncwarp();
        fmha_split_epilogue<DP>(p.part_o, p.part_ml, g.part, t, row, m_run, l_run, o_tm,
                                bar(C::B_OFREE + t));
        continue;
      }
      const uint32_t stage = base + C::OFF_OST;
#pragma unroll 1
      for (int c = 0; c < C::NCH; ++c) {
        const uint32_t row_addr = stage + c * C::CH_BYTES + row * 128;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t o[32];
          tmem_ld32(o_tm + c * 64 + hh * 32, o);
          if (c == C::NCH - 1 && hh == 1) {
            tc_fence_before_sync();
            mbar_arrive(bar(C::B_OFREE + t));  // O_t is read: the next item may overwrite it
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
        const int row0 = q0 + t * C::BM + wq * 32;
        if (row0 < p.len_q) {
          for (int c = 0; c < C::NCH; ++c)
            tma_store_4d(&tm_o, stage + c * C::CH_BYTES + wq * 32 * 128, c * 64, row0, h, b);
          bulk_commit_group();
          bulk_wait_group_read0();
        }
        mbar_arrive(bar(C::B_OST + (1 - t) * 4 + wq));  // these staging rows are free again
      }
      __syncwarp();
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (*abort_flag && (warp == C::W_MMA || warp == C::W_PV)) {
    // Each issuing warp commits to DRAIN (same election as its MMAs, so the commit tracks all of
    // them); the TMEM owner waits for both before giving TMEM back.
    umma_commit_w(bar(C::B_DRAIN));
    if (warp == C::W_MMA && lane == 0) mbar_wait_drain(bar(C::B_DRAIN), 0, p.timeout_ns);
    __syncwarp();
  }
  if (warp == C::W_MMA) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  // The last CTA to finish puts the work counters back to zero for the next launch.
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.work + 1, 1u) == gridDim.x - 1) {
      atomicExch(p.work, 0u);
      atomicExch(p.work + 1, 0u);
    }
  }
}

// --------------------------------------------------------------------------------------------
// Host side
// --------------------------------------------------------------------------------------------
namespace {

bool stride_ok(int64_t s, int esize) { return s > 0 && ((s * esize) % 16) == 0 && (s * esize) < (1ll << 40); }

template <int DP, bool BF16, bool SPLIT, int MK>
void* fmha_kernel_ptr() {
  return reinterpret_cast<void*>(&fmha_fwd_sm100_kernel<DP, BF16, SPLIT, MK>);
}

// Tail split of a non-causal launch on num_sms persistent CTAs.  With n items and G CTAs, the
// first n - n % G items run whole (full waves); the n % G items of the last, partial wave would
// leave most CTAs idle while they run, so each is cut into split = G / (n % G) key ranges (at most
// kMaxSplit, and at least 4 key tiles per range; 8 when n < G and every item is cut; no split
// for items of fewer than 16 key tiles).  Workspace: the 256-byte work counters, the
// packed mask if the call has one, then each range's (m, l) per row and its fp32 O rows (scratch:
// written before they are read).
struct FmhaSplit {
  int n_whole = 0, split = 1, n_work = 0;
  size_t ml_off = 0, o_off = 0, bytes = kAttnWorkspaceMin;
};

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// The packed form of a call's boolean mask: extents (1 along a broadcast dimension), words per
// row (a multiple of 4) and word strides (0 along a broadcast dimension).
struct MaskPack {
  long long nb = 0, nh = 0, nq = 0, words = 0, rows = 0;
  long long wb = 0, wh = 0, wq = 0;
  size_t bytes = 0;
};

MaskPack mask_pack_plan(const cmpx_attn_desc* d) {
  MaskPack m;
  if (!d->mask || d->mask_kind != CMPX_MASK_BOOL) return m;
  m.nb = d->mask_stride[0] == 0 ? 1 : d->batch;
  m.nh = d->mask_stride[1] == 0 ? 1 : d->heads;
  m.nq = d->mask_stride[2] == 0 ? 1 : d->len_q;
  m.words = ((d->len_k + 31) / 32 + 3) / 4 * 4;
  m.rows = m.nb * m.nh * m.nq;
  m.wq = m.nq > 1 ? m.words : 0;
  m.wh = m.nh > 1 ? m.nq * m.words : 0;
  m.wb = m.nb > 1 ? m.nh * m.nq * m.words : 0;
  m.bytes = align256(static_cast<size_t>(m.rows * m.words) * sizeof(uint32_t));
  return m;
}

FmhaSplit fmha_split_plan(const cmpx_attn_desc* d, int num_sms) {
  FmhaSplit sp;
  sp.bytes = kAttnWorkspaceMin + mask_pack_plan(d).bytes;
  const int64_t n_items = ((d->len_q + 255) / 256) * d->heads * d->batch;
  sp.n_whole = static_cast<int>(n_items);
  sp.n_work = static_cast<int>(n_items);
  if (d->causal || num_sms <= 1 || n_items <= 0) return sp;
  const int64_t rem = n_items % num_sms;
  if (rem == 0) return sp;
  const bool add_mask = d->mask && d->mask_kind == CMPX_MASK_ADD;
  const int64_t bn = (d->head_dim <= 128 && !add_mask) ? 128 : 64;
  const int64_t n_kv = (d->len_k + bn - 1) / bn;
  // Items of fewer than 16 key tiles are not cut: the ranges' park-and-merge then costs more than
  // the idle tail it fills ([4,40,1024,1024,64] fp16, 8 tiles an item: 91.1 us split, 81.9 us not;
  // [2,10,2048,2048,64], 16 tiles: 54.2 us split, 63.5 us not).  A launch of fewer items than SMs
  // splits every item, and every range then parks and merges its whole 256-row partial: at least 8
  // key tiles a range there, 4 for the tail of a longer launch.
  if (n_kv < 16) return sp;
  const int64_t per_range = n_items < num_sms ? 8 : 4;
  const int64_t split = std::min<int64_t>({num_sms / rem, n_kv / per_range, kMaxSplit});
  if (split < 2) return sp;
  const int dp = d->head_dim <= 64 ? 64 : d->head_dim <= 128 ? 128 : 192;
  sp.split = static_cast<int>(split);
  sp.n_whole = static_cast<int>(n_items - rem);
  sp.n_work = static_cast<int>(sp.n_whole + rem * split);
  const size_t ranges = static_cast<size_t>(rem * split);
  sp.ml_off = kAttnWorkspaceMin + mask_pack_plan(d).bytes;
  sp.o_off = sp.ml_off + align256(ranges * 256 * 2 * sizeof(float));
  sp.bytes = sp.o_off + ranges * 256 * dp * sizeof(float);
  return sp;
}

}  // namespace

// Grouped-query heads with few query rows (decode steps, short prefills): the `group` query heads
// of a key/value head are folded into one head of group * len_q rows, so the two 128-row Q tiles of
// an item hold several heads' rows against one K/V stream -- each K/V tile is read once per
// key/value head instead of once per query head, and there are `group` times fewer mostly empty
// items ([8,32,1,4096,128] bf16 with 8 key/value heads: 256 items of one query row each before).
// Exact (attention treats every query row on its own).  Needs the query and output rows of the
// group to be one stride apart: always for one query row (the head stride then serves as the row
// stride), else when a head's rows follow each other (head stride = len_q * row stride); no mask
// and no causal mask (both are per head and row).
static bool fmha_gqa_fold(const cmpx_attn_desc* d, cmpx_attn_desc* f) {
  if (d->causal || d->mask || d->heads_kv <= 0 || d->heads_kv >= d->heads || d->heads % d->heads_kv != 0 ||
      d->len_q < 1 || d->len_q >= 256)
    return false;
  const int64_t group = d->heads / d->heads_kv;
  const bool one_row = d->len_q == 1;
  if (!one_row && (d->q_stride[1] != d->len_q * d->q_stride[2] || d->o_stride[1] != d->len_q * d->o_stride[2]))
    return false;
  *f = *d;
  f->heads = d->heads_kv;
  f->len_q = d->len_q * group;
  if (one_row) {  // row r of the folded head = query head g * group + r
    f->q_stride[2] = d->q_stride[1];
    f->o_stride[2] = d->o_stride[1];
  }
  f->q_stride[1] = d->q_stride[1] * group;
  f->o_stride[1] = d->o_stride[1] * group;
  f->heads_kv = 0;  // one query head (of group * len_q rows) per key/value head
  return true;
}

size_t fmha_workspace_bytes(const cmpx_attn_desc* d_in, int num_sms) {
  cmpx_attn_desc fd;
  const cmpx_attn_desc* d = fmha_gqa_fold(d_in, &fd) ? &fd : d_in;
  if (fmha_short_eligible(d)) return kAttnWorkspaceMin;
  return fmha_split_plan(d, num_sms).bytes;
}

size_t fmha_workspace_min(const cmpx_attn_desc* d_in) {
  cmpx_attn_desc fd;
  const cmpx_attn_desc* d = fmha_gqa_fold(d_in, &fd) ? &fd : d_in;
  return kAttnWorkspaceMin + (fmha_short_eligible(d) ? 0 : mask_pack_plan(d).bytes);
}

const char* fmha_sm100_plan(const cmpx_attn_desc* d_in, int* status) {
  *status = CMPX_OK;
  cmpx_attn_desc fd;
  const cmpx_attn_desc* d = fmha_gqa_fold(d_in, &fd) ? &fd : d_in;
  if (d->dtype != CMPX_F16 && d->dtype != CMPX_BF16) {
    *status = CMPX_ERR_UNSUPPORTED_DTYPE;
    return "none";
  }
  if (d->head_dim < 8 || d->head_dim > 192 || (d->head_dim % 8) != 0) {
    *status = CMPX_ERR_UNSUPPORTED_SHAPE;
    return "none";
  }
  if (d->len_q > (1ll << 31) - 256 || d->len_k > (1ll << 31) - 256 || d->heads > 65535 || d->batch > 65535) {
    *status = CMPX_ERR_UNSUPPORTED_SHAPE;
    return "none";
  }
  const void* ptrs[4] = {d->q, d->k, d->v, d->o};
  for (const void* ptr : ptrs)
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) {
      *status = CMPX_ERR_MISALIGNED;
      return "none";
    }
  const int64_t* strides[4] = {d->q_stride, d->k_stride, d->v_stride, d->o_stride};
  for (const int64_t* s : strides)
    for (int i = 0; i < 3; ++i)
      if (!stride_ok(s[i], 2)) {
        *status = CMPX_ERR_MISALIGNED;
        return "none";
      }
  if (((d->len_q + 255) / 256) * d->heads * d->batch > (1ll << 30)) {
    *status = CMPX_ERR_UNSUPPORTED_SHAPE;
    return "none";
  }
  if (d->mask && d->mask_kind == CMPX_MASK_ADD) {  // 16-byte vector loads of each row's values
    if ((reinterpret_cast<uintptr_t>(d->mask) & 15u) != 0) {
      *status = CMPX_ERR_MISALIGNED;
      return "none";
    }
    for (int i = 0; i < 3; ++i)
      if (d->mask_stride[i] % 8 != 0) {
        *status = CMPX_ERR_MISALIGNED;
        return "none";
      }
  }
  if (fmha_short_eligible(d)) return fmha_short_name(d);
  // The name shows the schedule a call given cmpx_attn_workspace_size() bytes runs: "+tail-split"
  // when the last wave's items are split into key ranges (a second, merging kernel follows),
  // "+mask" when a boolean mask is packed to bits (a packing kernel runs first), "+addmask" for an
  // additive mask.
  const bool split = fmha_split_plan(d, current_num_sms()).split > 1;
  const bool bf = d->dtype == CMPX_BF16;
  static const std::array<std::string, 36> names = [] {
    std::array<std::string, 36> out;
    const char* const dims[3] = {"D64,2x128q,128kv,6st", "D128,2x128q,128kv,4st", "D192,2x128q,64kv,3st"};
    const char* const masks[3] = {"", "+mask", "+addmask"};
    for (int dd = 0; dd < 3; ++dd)
      for (int t = 0; t < 2; ++t)
        for (int sp = 0; sp < 2; ++sp)
          for (int mk = 0; mk < 3; ++mk)
            out[((dd * 2 + t) * 2 + sp) * 3 + mk] = std::string("fmha_sm100<") + (t ? "bf16," : "f16,") +
                                                    dims[dd] + ",persistent" + (sp ? "+tail-split" : "") +
                                                    masks[mk] + ">";
    return out;
  }();
  const int dd = d->head_dim <= 64 ? 0 : d->head_dim <= 128 ? 1 : 2;
  const int mk = !d->mask ? 0 : d->mask_kind == CMPX_MASK_BOOL ? 1 : 2;
  return names[((dd * 2 + (bf ? 1 : 0)) * 2 + (split ? 1 : 0)) * 3 + mk].c_str();
}

bool make_bhsd_map(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, int64_t D, int64_t L,
                   int64_t H, int64_t B, const int64_t* st, uint32_t box_rows) {
  const uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(L),
                            static_cast<uint64_t>(H), static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(st[2]) * 2, static_cast<uint64_t>(st[1]) * 2,
                               static_cast<uint64_t>(st[0]) * 2};
  const uint32_t box[4] = {64, box_rows, 1, 1};
  return encode_tmap(map, dt, 4, ptr, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

namespace {

template <int DP, bool BF16>
int launch_typed(const cmpx_attn_desc* d, const LaunchCtx& ctx) {
  using C = FmhaCfg<DP, fmha_bn<DP, 0>()>;        // plain and boolean-mask instantiations
  using C2 = FmhaCfg<DP, fmha_bn<DP, 2>()>;       // additive-mask instantiations
  const int mk = !d->mask ? 0 : d->mask_kind == CMPX_MASK_BOOL ? 1 : 2;
  const int bn = mk == 2 ? C2::BN : C::BN;
  const int smem_bytes = mk == 2 ? C2::SMEM_BYTES : C::SMEM_BYTES;
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv, to;
  if (!make_bhsd_map(&tq, dt, d->q, d->head_dim, d->len_q, d->heads, d->batch, d->q_stride, 128) ||
      !make_bhsd_map(&tk, dt, d->k, d->head_dim, d->len_k, attn_heads_kv(d), d->batch, d->k_stride, bn) ||
      !make_bhsd_map(&tv, dt, d->v, d->head_dim, d->len_k, attn_heads_kv(d), d->batch, d->v_stride, bn) ||
      !make_bhsd_map(&to, dt, d->o, d->head_dim, d->len_q, d->heads, d->batch, d->o_stride, 32))
    return CMPX_ERR_LAUNCH;

  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    void* const ptrs[6] = {fmha_kernel_ptr<DP, BF16, false, 0>(), fmha_kernel_ptr<DP, BF16, true, 0>(),
                           fmha_kernel_ptr<DP, BF16, false, 1>(), fmha_kernel_ptr<DP, BF16, true, 1>(),
                           fmha_kernel_ptr<DP, BF16, false, 2>(), fmha_kernel_ptr<DP, BF16, true, 2>()};
    const int bytes[6] = {C::SMEM_BYTES, C::SMEM_BYTES, C::SMEM_BYTES, C::SMEM_BYTES, C2::SMEM_BYTES, C2::SMEM_BYTES};
    for (int i = 0; i < 6; ++i)
      if (attr_err == cudaSuccess)
        attr_err = cudaFuncSetAttribute(ptrs[i], cudaFuncAttributeMaxDynamicSharedMemorySize, bytes[i]);
  });
  if (attr_err != cudaSuccess) return CMPX_ERR_LAUNCH;

  FmhaParams p;
  p.heads = static_cast<int>(d->heads);
  p.len_q = static_cast<int>(d->len_q);
  p.len_k = static_cast<int>(d->len_k);
  p.n_pairs = static_cast<int>((d->len_q + 255) / 256);
  p.n_items = static_cast<int>(p.n_pairs * d->heads * d->batch);
  p.lpt_first = p.n_items;
  p.lpt_heads = 1;
  if (d->causal && p.n_pairs > 1) {
    // enough slices that the sorted tail holds CMPX_FMHA_LPT items per CTA
    const long long slices = d->heads * d->batch;
    const long long ctas = std::min<long long>(p.n_items, std::max(1, ctx.num_sms));
    p.lpt_heads = static_cast<int>(std::min<long long>(slices, (CMPX_FMHA_LPT * ctas + p.n_pairs - 1) / p.n_pairs));
    if (p.lpt_heads > 0) p.lpt_first = static_cast<int>((slices - p.lpt_heads) * p.n_pairs);
    else p.lpt_heads = 1;
  }
  p.causal = d->causal ? 1 : 0;
  p.neg_scale = d->scale < 0 ? 1 : 0;
  p.scale_log2 = static_cast<float>(d->scale * 1.4426950408889634);
  p.o = d->o;
  p.os_b = d->o_stride[0];
  p.os_h = d->o_stride[1];
  p.os_s = d->o_stride[2];
  p.head_dim = static_cast<int>(d->head_dim);
  p.group = attn_group(d);
  p.work = static_cast<unsigned int*>(d->workspace);
  p.timeout_ns = ctx.timeout_ns;
  p.dev_flags = ctx.dev_flags;
  FmhaSplit sp = fmha_split_plan(d, ctx.num_sms);
  if (d->workspace_bytes < sp.bytes) sp = FmhaSplit{};  // too small a workspace: no split
  uint8_t* ws = static_cast<uint8_t*>(d->workspace);
  const MaskPack mp = mask_pack_plan(d);
  p.mask_bits = nullptr;
  p.mb_b = p.mb_h = p.mb_q = 0;
  p.mask_add = nullptr;
  p.ma_b = p.ma_h = p.ma_q = 0;
  p.mask_inv_scale = static_cast<float>(1.0 / d->scale);
  if (mk == 2) {
    p.mask_add = static_cast<const uint16_t*>(d->mask);
    p.ma_b = d->mask_stride[0];
    p.ma_h = d->mask_stride[1];
    p.ma_q = d->mask_stride[2];
  }
  if (mk == 1) {  // pack the mask to bits in the workspace, after the work counters
    uint32_t* bits = reinterpret_cast<uint32_t*>(ws + kAttnWorkspaceMin);
    const long long blocks = (mp.rows + 7) / 8;
    if (blocks > 0x7fffffffll) return CMPX_ERR_UNSUPPORTED_SHAPE;
    fmha_pack_mask_kernel<<<static_cast<unsigned int>(blocks), 256, 0, ctx.stream>>>(
        static_cast<const uint8_t*>(d->mask), d->mask_stride[0], d->mask_stride[1], d->mask_stride[2],
        static_cast<int>(mp.nh), static_cast<int>(mp.nq), static_cast<int>(d->len_k),
        static_cast<int>(mp.words), mp.rows, bits);
    if (cudaGetLastError() != cudaSuccess) return CMPX_ERR_LAUNCH;
    p.mask_bits = bits;
    p.mb_b = mp.wb;
    p.mb_h = mp.wh;
    p.mb_q = mp.wq;
  }
  p.n_whole = sp.split > 1 ? sp.n_whole : p.n_items;
  p.split = sp.split;
  p.n_work = sp.split > 1 ? sp.n_work : p.n_items;
  p.part_ml = sp.split > 1 ? reinterpret_cast<float*>(ws + sp.ml_off) : nullptr;
  p.part_o = sp.split > 1 ? reinterpret_cast<float*>(ws + sp.o_off) : nullptr;
  const int grid = std::min(p.n_work, std::max(1, ctx.num_sms));
  auto launch = [&](auto split_tag, auto mk_tag) {
    fmha_fwd_sm100_kernel<DP, BF16, decltype(split_tag)::value, decltype(mk_tag)::value>
        <<<grid, C::THREADS, smem_bytes, ctx.stream>>>(tq, tk, tv, to, p);
  };
  using Split = std::true_type;
  using NoSplit = std::false_type;
  using M0 = std::integral_constant<int, 0>;
  using M1 = std::integral_constant<int, 1>;
  using M2 = std::integral_constant<int, 2>;
  if (sp.split > 1) {
    if (mk == 1) launch(Split{}, M1{});
    else if (mk == 2) launch(Split{}, M2{});
    else launch(Split{}, M0{});
    if (cudaGetLastError() != cudaSuccess) return CMPX_ERR_LAUNCH;
    const int rows = (p.n_items - p.n_whole) * 256;
    fmha_split_merge_kernel<DP, BF16><<<(rows + 7) / 8, 128, 0, ctx.stream>>>(p);
  } else {
    if (mk == 1) launch(NoSplit{}, M1{});
    else if (mk == 2) launch(NoSplit{}, M2{});
    else launch(NoSplit{}, M0{});
  }
  return cudaGetLastError() == cudaSuccess ? CMPX_OK : CMPX_ERR_LAUNCH;
}

}  // namespace

int launch_fmha_sm100(const cmpx_attn_desc* d_in, const LaunchCtx& ctx) {
  int st = CMPX_OK;
  fmha_sm100_plan(d_in, &st);
  if (st != CMPX_OK) return st;
  cmpx_attn_desc fd;
  const cmpx_attn_desc* d = fmha_gqa_fold(d_in, &fd) ? &fd : d_in;
  if (d->len_q == 0) return CMPX_OK;
  if (fmha_short_eligible(d)) return launch_fmha_short(d, ctx);
  const bool bf = d->dtype == CMPX_BF16;
  if (d->head_dim <= 64) return bf ? launch_typed<64, true>(d, ctx) : launch_typed<64, false>(d, ctx);
  if (d->head_dim <= 128) return bf ? launch_typed<128, true>(d, ctx) : launch_typed<128, false>(d, ctx);
  return bf ? launch_typed<192, true>(d, ctx) : launch_typed<192, false>(d, ctx);
}

}  // namespace cmpx
