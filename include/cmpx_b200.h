/*
 * cmpx_b200.h -- C ABI of the B200 (sm_100a) attention / batched-matmul library.
 *
 * This is the drop-in boundary for the hot path of cmpext3 (WifiLast/torch-cmp-patch):
 * the native ops that the Python monkeypatch reaches for
 *   F.scaled_dot_product_attention  -> cmpext3.ops.attention(query, key, value, scale=None, causal=False)
 *   torch.bmm / matmul / einsum     -> cmpext3.ops.bmm(input, mat2)
 *   F.linear (nn.Linear)            -> cmpext3.ops.linear(input, weight, bias=None)
 * In the reference those are pybind11 functions over ATen tensors
 * (src/main.cpp:2307-2309 `bmm`, src/main.cpp:2353-2358 `attention`, implemented by
 * custom_bmm_forward src/main.cpp:363-441 and custom_attention_forward src/main.cpp:1603-1774).
 * Here the boundary is plain C: borrowed device pointers, element strides, sizes, a dtype tag,
 * the caller's cudaStream_t, and an int status.  Nothing in this header depends on torch.
 *
 * Conventions
 *  - Every entry point returns CMPX_OK (0) or a CMPX_ERR_* code.  A non-zero return means no
 *    kernel was launched and the output was not touched (the reference's launcher that declined
 *    silently and left the output unwritten, src/main.cpp:1742-1758, is exactly what this rules out).
 *  - Work is enqueued on `stream` (a cudaStream_t passed as void*) on the CURRENT device; the
 *    call does not synchronise and does not allocate device memory.
 *  - Strides are in elements.  For attention the head_dim must be contiguous (stride 1); for
 *    bmm one of the two matrix strides of each input must be 1 and C must be row-major.
 *  - Device-side waits are bounded.  A kernel whose wait runs out sets a bit in the device status
 *    word, stops early and returns; cmpx_device_status() reads (and clears) that word.
 */
#ifndef CMPX_B200_H
#define CMPX_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CMPX_API __attribute__((visibility("default")))
#else
#define CMPX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define CMPX_ABI_VERSION 7  /* 2: cmpx_attn_desc.heads_kv (grouped-query attention); 3: cmpx_linear;
                               4: cmpx_attn_desc.mask / mask_kind (boolean or additive attention mask);
                               5: cmpx_bmm_small / cmpx_bmm_small_plan;
                               6: cmpx_bmm_rowstats(_plan), cmpx_softmax_product(_plan);
                               7: cmpx_bmm_ws / cmpx_linear_ws and their workspace sizes */

/* Element type of every operand of one call (inputs and output share it, as in the reference:
 * dtype in == dtype out, src/main.cpp:1623-1627, :366-369). */
typedef enum cmpx_dtype {
  CMPX_F32 = 0,
  CMPX_F16 = 1,
  CMPX_BF16 = 2
} cmpx_dtype;

typedef enum cmpx_mask_kind {
  CMPX_MASK_BOOL = 0,  /* one byte per element, nonzero = the key takes part */
  CMPX_MASK_ADD = 1    /* added to the scaled scores, in the call's dtype */
} cmpx_mask_kind;

typedef enum cmpx_status {
  CMPX_OK = 0,
  CMPX_ERR_INVALID_ARGUMENT = 1,  /* null pointer, negative size, shape mismatch */
  CMPX_ERR_UNSUPPORTED_SHAPE = 2, /* outside the tile table (e.g. head_dim > 192) */
  CMPX_ERR_UNSUPPORTED_DTYPE = 3,
  CMPX_ERR_MISALIGNED = 4,        /* pointer/stride not 16-byte aligned for TMA */
  CMPX_ERR_WORKSPACE = 5,         /* workspace missing or too small */
  CMPX_ERR_LAUNCH = 6,            /* CUDA launch or tensor-map encode failed */
  CMPX_ERR_DEVICE = 7,            /* no sm_100 device current, or CUDA runtime error */
  CMPX_ERR_DEVICE_TIMEOUT = 8     /* reported by cmpx_device_status only */
} cmpx_status;

/* Scaled-dot-product attention forward:  O = softmax(Q K^T * scale [+ causal mask]) V
 * Tensors are [batch, heads, len, head_dim] with arbitrary batch/head/len strides and a
 * contiguous head_dim (the same strided-view contract as the reference's HFMA2 route,
 * src/main.cpp:1637-1666).  Causal masking is top-left aligned (key j is visible to query i
 * iff j <= i), which is what torch's is_causal does for len_q != len_k.
 * Grouped-query attention: k and v may have heads_kv heads (a divisor of heads); query head h then
 * reads key/value head h / (heads / heads_kv), as torch's enable_gqa=True does.
 * Attention mask, torch's attn_mask, broadcastable: mask_stride holds element strides
 * over batch, head, query row and key, 0 for a broadcast dimension; the key stride must be 1.
 *  - mask_kind CMPX_MASK_BOOL: one byte per element; key j takes part in query i's softmax only where
 *    mask[b, h, i, j] is nonzero.  A 16-bit call packs it to bits in the workspace
 *    (cmpx_attn_workspace_size counts that), so a masked 16-bit call needs the full workspace.
 *  - mask_kind CMPX_MASK_ADD: values in the call's dtype added to the scaled scores
 *    (softmax(q k^T * scale + mask)); -inf removes a key.  Rows must start on 16-byte boundaries
 *    (the query-row stride a multiple of 8 elements for 16-bit calls, 4 for fp32, or 0).
 *  - fp32 calls read the mask in place (no workspace): its pointer 16-byte aligned and every
 *    stride a multiple of 16 bytes (boolean: 16 elements; additive: 4), else
 *    CMPX_ERR_MISALIGNED.
 * With causal the mask applies on top of it (torch's math path ANDs them).  A query row with no key
 * left gets an all-zero output (torch's result), not NaN.
 * Replaces: custom_attention_forward (src/main.cpp:1603-1774) and its launchers
 * launch_flash_attention_hfma2 (src/cuda/fp16_flash_attention_hfma2.cu:269-286),
 * launch_attention_fp16 (src/cuda/fp16_attention.cu:328-386),
 * launch_attention_fp32 (src/cuda/fp32_attention.cu:200-221). */
typedef struct cmpx_attn_desc {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t batch, heads, len_q, len_k, head_dim;
  int64_t q_stride[3]; /* batch, head, row strides of q (elements) */
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int32_t dtype;       /* cmpx_dtype */
  int32_t causal;      /* 0 or 1 */
  double scale;        /* softmax scale; the reference default is 1/sqrt(head_dim) */
  void* workspace;     /* device scratch of cmpx_attn_workspace_size() bytes (may be NULL if 0) */
  size_t workspace_bytes;
  int64_t heads_kv;    /* heads of k and v: 0 or heads = one per query head, else a divisor of heads */
  const void* mask;    /* attention mask (see above); NULL = none */
  int64_t mask_stride[4]; /* batch, head, query-row, key strides of mask (elements; 0 = broadcast) */
  int32_t mask_kind;   /* cmpx_mask_kind */
  int32_t reserved2;
} cmpx_attn_desc;

/* Batched matmul  C[b] = A[b] @ B[b],  A: [batch, m, k], B: [batch, k, n], C: [batch, m, n].
 * Each operand has a batch stride and two matrix strides (row, col).  One of the two matrix
 * strides of A and of B must be 1 (row-major or column-major view: a transposed operand is
 * passed as a view, never copied); C must be row-major (col stride 1).
 * fp32 runs on the tensor cores as 3xTF32 (each operand split into a TF32 hi part and an fp32
 * remainder; a*b ~ a_hi*b_hi + a_hi*b_lo + a_lo*b_hi with fp32 accumulation), and needs K-major
 * operands: A contiguous along k (a_stride[2] == 1), B contiguous along k (b_stride[1] == 1), every
 * stride that is stepped a multiple of 4 elements and every pointer 16-byte aligned; other fp32
 * layouts return CMPX_ERR_MISALIGNED (copy B to a column-major view first).  The tensor core's fp32
 * accumulation error grows with k (2e-5 of the output's peak at k = 8192, 9e-5 at 32768), so an fp32
 * call with k > 8192 runs as several launches over k chunks of at most 8192 on the same stream: the
 * first stores C, the others add their partial products into it (the plan name ends in
 * "+k-chunks"); C must not alias A or B.
 * Replaces: custom_bmm_forward (src/main.cpp:363-441) and its per-batch host loop over
 * launch_matmul_fp32 (src/cuda/fp32_matmul.cu:236-265) / launch_matmul_fp16
 * (src/cuda/fp16_matmul.cu:373-427). */
typedef struct cmpx_bmm_desc {
  const void* a;
  const void* b;
  void* c;
  int64_t batch, m, n, k;
  int64_t a_stride[3]; /* batch, row (m), col (k) */
  int64_t b_stride[3]; /* batch, row (k), col (n) */
  int64_t c_stride[3]; /* batch, row (m), col (n); col must be 1 */
  int32_t dtype;       /* cmpx_dtype */
  int32_t reserved;
} cmpx_bmm_desc;

/* Attention forward.  Replaces cmpext3.ops.attention (src/main.cpp:2353-2358). */
CMPX_API int cmpx_attn_fwd(const cmpx_attn_desc* desc, void* stream);

/* Bytes of device workspace for the fastest schedule of this problem on the current device.  The
 * 16-bit kernels keep the two work counters of their persistent schedule in the first 256 bytes; a
 * non-causal call whose last wave of (256-row, head) items would leave most SMs idle also splits
 * those items into key ranges, whose partial results (fp32 O rows and per-row max / sum) take the
 * bytes after the counters and are merged by a second kernel.  Any 16-bit call accepts a workspace
 * of at least 256 bytes: one smaller than this size runs unsplit, with the same results up to fp32
 * summation order.  An fp32 call needs a workspace only for the same kind of split (its last wave's
 * 128-row items cut into key ranges, 8-bit per-item arrival counters in the first 256 bytes, the
 * partial rows after them, merged by the last range to finish); 0 when it runs unsplit, and given
 * less than this size it runs unsplit.  The workspace must be 16-byte aligned and its
 * first 256 bytes zero-filled before the first call; every call leaves them zeroed on return (the
 * rest is scratch, written before it is read), so a workspace can be reused by calls that do not
 * overlap on the GPU (one per stream).
 * No reference counterpart (the reference allocates nothing but the output). */
CMPX_API size_t cmpx_attn_workspace_size(const cmpx_attn_desc* desc);

/* Attention forward that allocates nothing, for callers that cannot obtain device memory at the
 * time of the call (a serving process whose pool owns the whole GPU, code running inside an
 * allocator callback, stacks that only allocate at start-up -- cudaMalloc may also synchronise the
 * device).  Same descriptor and results as cmpx_attn_fwd, but the workspace fields are ignored: the
 * kernel's scratch (its work counters) lives in a fixed 256-byte array inside the library, which
 * every GPU that loads the library keeps until the process exits; the 16-bit kernels then run the
 * schedule that needs no more than their 256 bytes of work counters (no tail split; additive masks
 * are served, but a call with a boolean mask returns CMPX_ERR_WORKSPACE, because that mask is packed
 * to bits in the workspace).  The call is checked against the tile table first, so an unsupported
 * call returns the same status as from cmpx_attn_fwd.  The first call on a device looks up that
 * array's device address (cudaGetSymbolAddress); make that first call before capturing the stream
 * into a graph.  A failed lookup returns CMPX_ERR_DEVICE and is retried by the next call.  Each call clears the counters it needs with an enqueued
 * memset.  All calls share the one array, so calls whose work overlaps on the GPU (different
 * streams without ordering between them) race on it: serialise them.
 * No counterpart in the reference. */
CMPX_API int cmpx_attn_fwd_noalloc(const cmpx_attn_desc* desc, void* stream);

/* Batched matmul.  Replaces cmpext3.ops.bmm (src/main.cpp:2307-2309). */
CMPX_API int cmpx_bmm(const cmpx_bmm_desc* desc, void* stream);

/* Batched product of many tiny matrices, same descriptor as cmpx_bmm: any dtype of the three, any
 * non-negative element strides for A, B and C (views are read and written in place), any m, n, k.
 * Each output element is a length-k dot product accumulated in fp32 and rounded once; there is no
 * intermediate tensor.  Meant for the per-item sizes the patched bmm / matmul route here
 * (m * k * n <= 32768 by default, CMPEXT3_SMALL_BMM_MAX_MKN), where a tiled GEMM wastes its tile.
 * Replaces: the eager broadcast multiply + sum of _small_bmm (cmpext3/__init__.py:440-464), which
 * materialises a [batch, m, k, n] intermediate. */
CMPX_API int cmpx_bmm_small(const cmpx_bmm_desc* desc, void* stream);
CMPX_API int cmpx_bmm_small_plan(const cmpx_bmm_desc* desc, char* buf, size_t buf_len);

/* Linear layer  y = x W^T (+ bias):  x [m, k], W [n, k] (the nn.Linear weight, read in place as the
 * K-major operand of the same GEMM as cmpx_bmm), bias [n] or NULL, y [m, n]; rows of x, W and y are
 * *_row_stride elements apart, columns contiguous.  fp16 / bf16: the bias is added to the fp32
 * accumulator before the one rounding to the output type; rows must start on 16-byte boundaries
 * (k, n and the strides multiples of 8) and the bias pointer must be 16-byte aligned.  fp32: the
 * 3xTF32 GEMM of cmpx_bmm, fp32 bias (4-byte aligned) added to the accumulator; k, n and the
 * strides multiples of 4.
 * Replaces: custom_linear_forward (src/main.cpp:195-346: bf16 converted to fp32 copies, W
 * transposed into a contiguous copy, an fp32 / fp16-accumulating GEMM, then a separate bias-add
 * kernel in the output type) behind cmpext3.ops.linear (the reference's _C.linear). */
typedef struct cmpx_linear_desc {
  const void* x;
  const void* w;
  const void* bias;    /* NULL: no bias */
  void* y;
  int64_t m, n, k;
  int64_t x_row_stride, w_row_stride, y_row_stride;
  int32_t dtype;       /* cmpx_dtype */
  int32_t reserved;
} cmpx_linear_desc;

CMPX_API int cmpx_linear(const cmpx_linear_desc* desc, void* stream);

/* cmpx_bmm / cmpx_linear with a device workspace, for the fp32 (3xTF32) products: given at least
 * cmpx_*_workspace_size bytes (16-byte aligned), a pass before the GEMM writes the low parts
 * (x - x truncated to TF32) of A and B, or of x and W, into the workspace once per call, and the
 * GEMM loads them beside the operands instead of splitting every shared-memory tile again (the
 * split's shared-memory traffic is what bounds the GEMM: 4096^3 measured 1.0 -> 0.6 ms).  The size
 * is 0 when the pass does not pay (m n / (m + n) < 512 per batch item, or k < 512), and for
 * fp16 / bf16 (which need none).
 * The results are the same as without a workspace, bit for bit.  cmpx_bmm_ws also takes an fp32 B
 * stored MN-major (a row-major [k, n] matrix: b_stride[2] == 1, rows 16-byte aligned), which
 * cmpx_bmm declines: the pass then writes B's hi and lo parts K-major into the workspace
 * (cmpx_bmm_workspace_size counts them), so no transposed copy of B is needed.  Bytes [0, 256) of the workspace
 * are neither read nor written, so the workspace of the attention calls (whose first 256 bytes
 * must stay zero) can be passed as it is; the rest is scratch, written before it is read.  Calls
 * that share a workspace must not overlap on the GPU.  A smaller or NULL workspace runs the
 * product as cmpx_bmm / cmpx_linear do.
 * No reference counterpart (the reference allocates nothing but the output). */
CMPX_API size_t cmpx_bmm_workspace_size(const cmpx_bmm_desc* desc);
CMPX_API int cmpx_bmm_ws(const cmpx_bmm_desc* desc, void* workspace, size_t workspace_bytes, void* stream);
CMPX_API size_t cmpx_linear_workspace_size(const cmpx_linear_desc* desc);
CMPX_API int cmpx_linear_ws(const cmpx_linear_desc* desc, void* workspace, size_t workspace_bytes, void* stream);

/* Row softmax over the last dimension:  y[r, :] = softmax(x[r, :]) for r < rows, computed in
 * fp32 (max, exp, sum) and rounded once to the output dtype (dtype in == dtype out), which is what
 * torch.softmax(x, dim=-1) returns for a fp16 / bf16 / fp32 tensor.  Rows are `cols` contiguous
 * elements apart by x_row_stride / y_row_stride (elements).
 * No counterpart among the reference's native ops: the reference leaves softmax stock
 * (cmpext3/__init__.py:133-138).  It serves the einsum-attention chain
 * einsum('bhid,bhjd->bhij') -> softmax(-1) -> einsum('bhij,bhjd->bhid') (cmpext3/einsum_ops.py:69-121),
 * whose softmax over the score tensor dominates that chain when it runs stock. */
typedef struct cmpx_softmax_desc {
  const void* x;
  void* y;
  int64_t rows, cols;
  int64_t x_row_stride, y_row_stride;
  int32_t dtype; /* cmpx_dtype */
  int32_t reserved;
} cmpx_softmax_desc;

CMPX_API int cmpx_softmax_rows(const cmpx_softmax_desc* desc, void* stream);

/* The einsum-attention chain einsum('bhid,bhjd->bhij') -> softmax(-1) -> einsum('bhij,bhjd->bhid')
 * (cmpext3/einsum_ops.py:69-121 in the reference, softmax left stock there,
 * cmpext3/__init__.py:133-138) with the score tensor written once and never read back: the scores
 * product also emits row statistics, and the softmax recomputes the scores from the product's
 * operands instead of reading them.  No counterpart among the reference's native ops.
 *
 * Row statistics of a 16-bit product C = A @ B: for every row r and every run of 64 columns
 * j*64 .. j*64+63 (the last one clipped at n), (max, sum) with max = the largest C[r, c] of the run
 * as stored (rounded to the 16-bit type) and sum = sum over the run of exp(C[r, c] - max), in fp32:
 * float stats[batch][ceil(n / 64)][m][2] (a run's rows contiguous), 8-byte aligned.
 *
 * cmpx_bmm_rowstats: cmpx_bmm (same descriptor, same result, bit for bit) for 16-bit A and B that
 * are both K-major (a_stride[2] == 1, b_stride[1] == 1), writing the statistics as well. */
CMPX_API int cmpx_bmm_rowstats(const cmpx_bmm_desc* desc, float* stats, void* stream);
CMPX_API int cmpx_bmm_rowstats_plan(const cmpx_bmm_desc* desc, const float* stats, char* buf, size_t buf_len);

/* cmpx_softmax_product: y = softmax(A @ B, dim=-1), A [batch, m, k] and B [batch, k, n] as in
 * cmpx_bmm_desc (16-bit, both K-major; 1 <= k <= 128), y [batch, m, n] with the strides in c_stride
 * (columns contiguous, rows 16-byte aligned; desc->c is not used), stats the product's row
 * statistics as cmpx_bmm_rowstats wrote them.  The scores are recomputed on the tensor cores with
 * the same instruction shape and k order as cmpx_bmm and rounded to the 16-bit type as cmpx_bmm
 * rounds them, so y is the softmax of exactly the tensor cmpx_bmm returns for (A, B); the
 * [batch, m, n] score tensor is never read.  Each y is exp(s - max) / sum in fp32, rounded once. */
CMPX_API int cmpx_softmax_product(const cmpx_bmm_desc* desc, const float* stats, void* y, void* stream);
CMPX_API int cmpx_softmax_product_plan(const cmpx_bmm_desc* desc, const float* stats, const void* y, char* buf,
                                       size_t buf_len);

/* Name of the tile-table entry a call would use, written into buf (NUL-terminated).
 * Returns CMPX_OK or the status the call itself would return.  Replaces the per-signature
 * decision record of the reference's runtime autoselect (cmpext3/autoselect.py:290-364),
 * which this library does not need: the kernel choice is a fixed function of the shape. */
CMPX_API int cmpx_attn_plan(const cmpx_attn_desc* desc, char* buf, size_t buf_len);
CMPX_API int cmpx_bmm_plan(const cmpx_bmm_desc* desc, char* buf, size_t buf_len);
CMPX_API int cmpx_linear_plan(const cmpx_linear_desc* desc, char* buf, size_t buf_len);

/* Human-readable text for a status code (static storage). */
CMPX_API const char* cmpx_status_str(int status);

/* Reads and clears the device status word of the current device after synchronising it.
 * *flags receives the OR of CMPX_DEVFLAG_* bits raised since the last call.
 * No reference counterpart (the reference's kernels have no bounded waits). */
#define CMPX_DEVFLAG_WAIT_TIMEOUT 1u   /* an mbarrier / pipeline wait ran out */
#define CMPX_DEVFLAG_BAD_ARGS 2u       /* a kernel rejected its own launch arguments */
CMPX_API int cmpx_device_status(unsigned int* flags);

/* Self-test of the bounded-wait path: launches one CTA that waits on an mbarrier nothing ever
 * arrives on, for at most timeout_ns nanoseconds, then records CMPX_DEVFLAG_WAIT_TIMEOUT and
 * returns.  Used by the failure-detection test; never faults, traps or hangs.
 * No reference counterpart. */
CMPX_API int cmpx_selftest_wait_timeout(uint64_t timeout_ns, void* stream);

/* Library ABI version (CMPX_ABI_VERSION). */
CMPX_API int cmpx_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CMPX_B200_H */
