"""cmpext3._native -- the native ops of this path, bound to the C-ABI library with ctypes.

Mirrors the reference's pybind11 module ``cmpext3._native`` for the two ops on this path
(src/main.cpp:2307-2309 ``bmm(input, mat2)``, src/main.cpp:2353-2358
``attention(query, key, value, scale=None, causal=False)``): same names, argument names, defaults,
positional order, dtype in == dtype out, and ``RuntimeError`` for anything the kernels do not
cover (the monkeypatch turns that into a stock-torch call, as in the reference).

The work is done by ``libcmpx_b200.so`` (include/cmpx_b200.h): this module only checks
arguments, allocates the output with torch's caching allocator, and passes raw device pointers,
element strides and the current CUDA stream.  There is no CPU or library fallback in here: if the
library is missing, importing this module raises ``ImportError``; if a call is outside the tile
table, it raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import functools
import math
import os
from pathlib import Path

import torch

__all__ = ["attention", "bmm", "attention_plan", "bmm_plan", "device_status", "LIBRARY_PATH",
           "lib", "CmpxError"]

LIBRARY_PATH = Path(os.environ.get("CMPX_LIBRARY", Path(__file__).with_name("libcmpx_b200.so")))

# Status codes (include/cmpx_b200.h)
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED_SHAPE = 2
ERR_UNSUPPORTED_DTYPE = 3
ERR_MISALIGNED = 4
ERR_WORKSPACE = 5
ERR_LAUNCH = 6
ERR_DEVICE = 7
ERR_DEVICE_TIMEOUT = 8

DEVFLAG_WAIT_TIMEOUT = 1
DEVFLAG_BAD_ARGS = 2

_DTYPE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


class CmpxError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, what: str, status: int):
        self.status = status
        super().__init__(f"cmpext3 {what}: {_status_str(status)} (status {status})")


class AttnDesc(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("o", ctypes.c_void_p),
        ("batch", ctypes.c_int64), ("heads", ctypes.c_int64), ("len_q", ctypes.c_int64),
        ("len_k", ctypes.c_int64), ("head_dim", ctypes.c_int64),
        ("q_stride", ctypes.c_int64 * 3), ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3), ("o_stride", ctypes.c_int64 * 3),
        ("dtype", ctypes.c_int32), ("causal", ctypes.c_int32), ("scale", ctypes.c_double),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("heads_kv", ctypes.c_int64),
        ("mask", ctypes.c_void_p), ("mask_stride", ctypes.c_int64 * 4),
        ("mask_kind", ctypes.c_int32), ("reserved2", ctypes.c_int32),
    ]


class BmmDesc(ctypes.Structure):
    _fields_ = [
        ("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("c", ctypes.c_void_p),
        ("batch", ctypes.c_int64), ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
        ("a_stride", ctypes.c_int64 * 3), ("b_stride", ctypes.c_int64 * 3),
        ("c_stride", ctypes.c_int64 * 3),
        ("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
    ]


class LinearDesc(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("bias", ctypes.c_void_p), ("y", ctypes.c_void_p),
        ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
        ("x_row_stride", ctypes.c_int64), ("w_row_stride", ctypes.c_int64), ("y_row_stride", ctypes.c_int64),
        ("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
    ]


class SoftmaxDesc(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("y", ctypes.c_void_p),
                ("rows", ctypes.c_int64), ("cols", ctypes.c_int64),
                ("x_row_stride", ctypes.c_int64), ("y_row_stride", ctypes.c_int64),
                ("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32)]


# CMPX_ABI_VERSION of include/cmpx_b200.h that the ctypes structures above mirror.
ABI_VERSION = 7


def _load() -> ctypes.CDLL:
    if not LIBRARY_PATH.exists():
        raise ImportError(
            f"cmpext3 native library not built ({LIBRARY_PATH}). "
            "Run: python torch-cmp-patch_b200/build.py")
    L = ctypes.CDLL(str(LIBRARY_PATH))
    L.cmpx_attn_fwd.argtypes = [ctypes.POINTER(AttnDesc), ctypes.c_void_p]
    L.cmpx_attn_fwd.restype = ctypes.c_int
    L.cmpx_attn_fwd_noalloc.argtypes = [ctypes.POINTER(AttnDesc), ctypes.c_void_p]
    L.cmpx_attn_fwd_noalloc.restype = ctypes.c_int
    L.cmpx_attn_workspace_size.argtypes = [ctypes.POINTER(AttnDesc)]
    L.cmpx_attn_workspace_size.restype = ctypes.c_size_t
    L.cmpx_bmm.argtypes = [ctypes.POINTER(BmmDesc), ctypes.c_void_p]
    L.cmpx_bmm.restype = ctypes.c_int
    L.cmpx_attn_plan.argtypes = [ctypes.POINTER(AttnDesc), ctypes.c_char_p, ctypes.c_size_t]
    L.cmpx_attn_plan.restype = ctypes.c_int
    L.cmpx_bmm_plan.argtypes = [ctypes.POINTER(BmmDesc), ctypes.c_char_p, ctypes.c_size_t]
    L.cmpx_bmm_plan.restype = ctypes.c_int
    L.cmpx_bmm_small.argtypes = [ctypes.POINTER(BmmDesc), ctypes.c_void_p]
    L.cmpx_bmm_small.restype = ctypes.c_int
    L.cmpx_bmm_small_plan.argtypes = [ctypes.POINTER(BmmDesc), ctypes.c_char_p, ctypes.c_size_t]
    L.cmpx_bmm_small_plan.restype = ctypes.c_int
    L.cmpx_linear.argtypes = [ctypes.POINTER(LinearDesc), ctypes.c_void_p]
    L.cmpx_bmm_workspace_size.restype = ctypes.c_size_t
    L.cmpx_bmm_workspace_size.argtypes = [ctypes.POINTER(BmmDesc)]
    L.cmpx_bmm_ws.restype = ctypes.c_int
    L.cmpx_bmm_ws.argtypes = [ctypes.POINTER(BmmDesc), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    L.cmpx_linear_workspace_size.restype = ctypes.c_size_t
    L.cmpx_linear_workspace_size.argtypes = [ctypes.POINTER(LinearDesc)]
    L.cmpx_linear_ws.restype = ctypes.c_int
    L.cmpx_linear_ws.argtypes = [ctypes.POINTER(LinearDesc), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    L.cmpx_linear.restype = ctypes.c_int
    L.cmpx_linear_plan.argtypes = [ctypes.POINTER(LinearDesc), ctypes.c_char_p, ctypes.c_size_t]
    L.cmpx_linear_plan.restype = ctypes.c_int
    L.cmpx_softmax_rows.argtypes = [ctypes.POINTER(SoftmaxDesc), ctypes.c_void_p]
    L.cmpx_softmax_rows.restype = ctypes.c_int
    L.cmpx_bmm_rowstats.argtypes = [ctypes.POINTER(BmmDesc), ctypes.c_void_p, ctypes.c_void_p]
    L.cmpx_bmm_rowstats.restype = ctypes.c_int
    L.cmpx_bmm_rowstats_plan.argtypes = [ctypes.POINTER(BmmDesc), ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    L.cmpx_bmm_rowstats_plan.restype = ctypes.c_int
    L.cmpx_softmax_product.argtypes = [ctypes.POINTER(BmmDesc), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    L.cmpx_softmax_product.restype = ctypes.c_int
    L.cmpx_softmax_product_plan.argtypes = [ctypes.POINTER(BmmDesc), ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_char_p, ctypes.c_size_t]
    L.cmpx_softmax_product_plan.restype = ctypes.c_int
    L.cmpx_status_str.argtypes = [ctypes.c_int]
    L.cmpx_status_str.restype = ctypes.c_char_p
    L.cmpx_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    L.cmpx_device_status.restype = ctypes.c_int
    L.cmpx_selftest_wait_timeout.argtypes = [ctypes.c_uint64, ctypes.c_void_p]
    L.cmpx_selftest_wait_timeout.restype = ctypes.c_int
    L.cmpx_abi_version.argtypes = []
    L.cmpx_abi_version.restype = ctypes.c_int
    if L.cmpx_abi_version() != ABI_VERSION:
        raise ImportError(
            f"{LIBRARY_PATH} has ABI version {L.cmpx_abi_version()}, this binding expects "
            f"{ABI_VERSION} (the descriptor layouts above). Rebuild: python torch-cmp-patch_b200/build.py")
    return L


lib = _load()

# Debug switch: synchronise after every call and raise if a device-side wait timed out.
_CHECK = os.environ.get("CMPEXT3_CHECK", "0") not in ("0", "", "false", "False")
_NVTX = os.environ.get("CMPEXT3_NVTX", "0") not in ("0", "", "false", "False")


def _traced(name: str):
    """With CMPEXT3_NVTX=1 (read at import), an NVTX range ``cmpx.<name>`` around every call of the
    op -- the binding's host work and the kernels it enqueues -- so that profiler timelines (nsys,
    ncu --nvtx) name the native calls.  Otherwise the op is returned unchanged (no cost)."""
    def wrap(fn):
        if not _NVTX:
            return fn

        @functools.wraps(fn)
        def inner(*args, **kwargs):
            torch.cuda.nvtx.range_push(f"cmpx.{name}")
            try:
                return fn(*args, **kwargs)
            finally:
                torch.cuda.nvtx.range_pop()
        return inner
    return wrap


def _status_str(status: int) -> str:
    return lib.cmpx_status_str(int(status)).decode()


def _stream_handle(device: torch.device) -> int:
    """Raw cudaStream_t of the current torch stream on `device` (no Stream object is built)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return torch._C._cuda_getCurrentRawStream(idx)


def device_status() -> int:
    """Synchronise the current device, return (and clear) its CMPX_DEVFLAG_* bits."""
    flags = ctypes.c_uint(0)
    st = lib.cmpx_device_status(ctypes.byref(flags))
    if st != OK:
        raise CmpxError("device_status", st)
    return int(flags.value)


def _post_check() -> None:
    if _CHECK:
        flags = device_status()
        if flags:
            raise CmpxError(f"device flags 0x{flags:x}", ERR_DEVICE_TIMEOUT)


# ---------------------------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------------------------

def _tma_ok(t: torch.Tensor) -> bool:
    """Strides usable by the 16-bit TMA path: head dim contiguous, other strides 16-byte multiples."""
    s0, s1, s2, s3 = t.stride()
    if s3 != 1 or t.data_ptr() % 16 != 0:
        return False
    es = t.element_size()
    return s0 > 0 and s1 > 0 and s2 > 0 and (s0 * es) % 16 == 0 and (s1 * es) % 16 == 0 and (s2 * es) % 16 == 0


def _attn_desc(q, k, v, o, scale: float, causal: bool, workspace=None, mask=None) -> AttnDesc:
    B, H, Lq, D = q.shape
    qs, ks, vs, os_ = q.stride(), k.stride(), v.stride(), o.stride()
    return AttnDesc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, Lq, k.shape[2], D,
                    (ctypes.c_int64 * 3)(*qs[:3]), (ctypes.c_int64 * 3)(*ks[:3]),
                    (ctypes.c_int64 * 3)(*vs[:3]), (ctypes.c_int64 * 3)(*os_[:3]),
                    _DTYPE[q.dtype], 1 if causal else 0, float(scale),
                    None if workspace is None else workspace.data_ptr(),
                    0 if workspace is None else workspace.numel(), k.shape[1],
                    None if mask is None else mask.data_ptr(),
                    (ctypes.c_int64 * 4)(*(mask.stride() if mask is not None else (0, 0, 0, 0))),
                    0 if mask is None or mask.dtype == torch.bool else 1, 0)


def _prepare_mask(attn_mask, query, key):
    """attn_mask broadcast to [B, H, Lq, Lk] as a strided view (0 along broadcast dims, the key
    dimension contiguous), or None.  Boolean masks and additive masks in the query's dtype are in
    the tile table; an additive mask of another dtype is not (stock serves it).  Rows are padded to
    16-byte boundaries where the kernel reads them with vector loads: additive masks, and every
    mask of an fp32 call (which reads the mask in place instead of packing it)."""
    if attn_mask is None:
        return None
    if not isinstance(attn_mask, torch.Tensor):
        raise TypeError("attn_mask must be a Tensor")
    additive = attn_mask.dtype != torch.bool
    if additive and attn_mask.dtype != query.dtype:
        raise RuntimeError("attention: an additive attn_mask runs on the kernels only in the query's dtype")
    if attn_mask.device != query.device:
        raise RuntimeError("attn_mask must be on the query's device")
    if attn_mask.dim() > 4:
        raise RuntimeError("attn_mask has more than 4 dimensions")
    B, H, Lq, _ = query.shape
    Lk = key.shape[2]
    m = attn_mask.reshape((1,) * (4 - attn_mask.dim()) + tuple(attn_mask.shape))
    if m.stride(3) != 1 and m.size(3) != 1:
        m = m.contiguous()
    if m.size(3) == 1 and Lk != 1:  # broadcast along keys: materialise its rows
        m = m.expand(*m.shape[:3], Lk).contiguous()
    if additive or query.dtype == torch.float32:
        # 16-byte vector loads: base and every non-broadcast row / head / batch stride aligned
        unit = 16 // m.element_size()

        def aligned(t):
            return t.data_ptr() % 16 == 0 and all(
                t.size(i) == 1 or t.stride(i) % unit == 0 for i in range(3))
        if not aligned(m):
            lk_pad = (m.size(3) + unit - 1) // unit * unit
            padded = torch.zeros(*m.shape[:3], lk_pad, dtype=m.dtype, device=m.device)
            padded[..., :m.size(3)] = m
            m = padded[..., :m.size(3)]
    try:
        m = m.expand(B, H, Lq, Lk)
    except RuntimeError as exc:
        raise RuntimeError(f"attn_mask {tuple(attn_mask.shape)} does not broadcast to {(B, H, Lq, Lk)}") from exc
    return m


def _check_attention_args(query, key, value) -> None:
    for name, t in (("query", query), ("key", key), ("value", value)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a Tensor")
        if t.dim() != 4:
            raise RuntimeError(f"{name} must be 4D (batch, heads, seq, head_dim)")
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor")
    if query.dtype not in _DTYPE or key.dtype != query.dtype or value.dtype != query.dtype:
        raise RuntimeError("query/key/value must share one dtype among float32/float16/bfloat16")
    if not (query.device == key.device == value.device):
        raise RuntimeError("query/key/value must be on one device")
    B, H, _, D = query.shape
    Hkv = key.shape[1]
    # Hkv < H: grouped-query attention (query head h reads key/value head h // (H // Hkv)), the
    # semantics of torch's enable_gqa=True; the reference's op takes equal head counts only.
    if key.shape[0] != B or key.shape[3] != D or Hkv < 1 or H % Hkv != 0:
        raise RuntimeError(f"key shape {tuple(key.shape)} does not match query {tuple(query.shape)}")
    if tuple(value.shape) != (B, Hkv, key.shape[2], D):
        raise RuntimeError(f"value shape {tuple(value.shape)} does not match key {tuple(key.shape)}")


def _f32_attn_ok(t: torch.Tensor) -> bool:
    return (t.stride(3) == 1 and t.data_ptr() % 16 == 0
            and all(st > 0 and st % 4 == 0 for st in t.stride()[:3]))


def _padded_f32(t: torch.Tensor) -> torch.Tensor:
    B, H, L, D = t.shape
    buf = torch.empty((B, H, L, (D + 3) // 4 * 4), dtype=t.dtype, device=t.device)
    buf[..., :D].copy_(t)
    return buf[..., :D]


def _prepare_attention(query, key, value, scale, causal):
    _check_attention_args(query, key, value)
    B, H, Lq, D = query.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if query.dtype != torch.float32:
        # TMA needs 16-byte aligned rows; copy a view that does not have them (the reference makes
        # such inputs contiguous too, src/main.cpp:1693-1698).
        query, key, value = (t if _tma_ok(t) else t.contiguous() for t in (query, key, value))
    else:
        # The 3xTF32 kernel reads with TMA too: pointer and batch / head / row strides 16-byte
        # aligned, head dim contiguous; other views are copied into buffers whose rows are padded
        # to a multiple of 4 elements (the padding is never read).
        query, key, value = (t if _f32_attn_ok(t) else _padded_f32(t) for t in (query, key, value))
    # Output in [B, Lq, H, D] memory viewed as [B, H, Lq, D] -- the layout torch's own CUDA SDPA
    # returns and the one a model's transpose(1, 2).reshape(B, Lq, H*D) wants.
    out = torch.empty((B, Lq, H, D), dtype=query.dtype, device=query.device).transpose(1, 2)
    return query, key, value, out, float(scale)


# Zero-filled workspaces, one per (device, stream): the kernels leave them zeroed, and calls on one
# stream never overlap, so each stream reuses its own.
_WORKSPACES: dict = {}


def release_workspaces() -> None:
    """Drop the cached per-stream workspaces (they grow to the largest call seen: an fp32 GEMM's
    split operands take 4 (m + n) k bytes per batch item).  The next call allocates afresh."""
    _WORKSPACES.clear()


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    key = (device.index, stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


@_traced("attention")
def attention(query, key, value, scale=None, causal=False, attn_mask=None):
    """SDPA forward on the sm_100a kernels.  Same contract as the reference's ops.attention, plus an
    optional boolean attn_mask (torch's meaning: True = the key takes part; with causal the two
    are ANDed; a row left with no key outputs 0)."""
    q, k, v, out, scale = _prepare_attention(query, key, value, scale, causal)
    mask = _prepare_mask(attn_mask, q, k)
    dev = q.device
    stream = _stream_handle(dev)
    # The 16-bit kernels keep their work counters (and the packed mask, and for a non-causal call
    # whose last wave of work is partial the split key ranges' partial results) in a workspace; the
    # fp32 ones need none.  One zero-filled buffer per (device, stream), grown on demand.
    desc = _attn_desc(q, k, v, out, scale, bool(causal), mask=mask)
    nbytes = lib.cmpx_attn_workspace_size(ctypes.byref(desc))
    if nbytes:
        ws = _workspace(dev, stream, nbytes)
        desc.workspace, desc.workspace_bytes = ws.data_ptr(), ws.numel()
    if dev.index == torch.cuda.current_device():
        st = lib.cmpx_attn_fwd(ctypes.byref(desc), stream)
    else:
        with torch.cuda.device(dev):
            st = lib.cmpx_attn_fwd(ctypes.byref(desc), stream)
    if st != OK:
        raise CmpxError("attention", st)
    _post_check()
    return out


def attention_plan(query, key, value, scale=None, causal=False, attn_mask=None) -> str:
    """Name of the tile-table entry ``attention`` would run for these arguments."""
    q, k, v, out, scale = _prepare_attention(query, key, value, scale, causal)
    mask = _prepare_mask(attn_mask, q, k)
    desc = _attn_desc(q, k, v, out, scale, bool(causal), mask=mask)
    buf = ctypes.create_string_buffer(128)
    st = lib.cmpx_attn_plan(ctypes.byref(desc), buf, 128)
    if st != OK:
        raise CmpxError("attention plan", st)
    return buf.value.decode()


# ---------------------------------------------------------------------------------------------
# bmm
# ---------------------------------------------------------------------------------------------

def _mat_ok(t: torch.Tensor) -> bool:
    """A [batch, r, c] operand the 16-bit TMA path reads in place: row- or column-major matrices
    with 16-byte aligned leading and batch strides."""
    if t.data_ptr() % 16 != 0:
        return False
    es = t.element_size()
    s0, s1, s2 = t.stride()
    lead_ok = (s2 == 1 and (t.shape[1] == 1 or (s1 > 0 and (s1 * es) % 16 == 0))) or \
              (s1 == 1 and (t.shape[2] == 1 or (s2 > 0 and (s2 * es) % 16 == 0)))
    batch_ok = t.shape[0] == 1 or (s0 > 0 and (s0 * es) % 16 == 0)
    return lead_ok and batch_ok


def _check_bmm_args(a, b) -> None:
    for name, t in (("input", a), ("mat2", b)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a Tensor")
        if t.dim() != 3:
            raise RuntimeError(f"{name} must be 3D")
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor")
    if a.dtype not in _DTYPE or b.dtype != a.dtype:
        raise RuntimeError("input/mat2 must share one dtype among float32/float16/bfloat16")
    if a.device != b.device:
        raise RuntimeError("input/mat2 must be on one device")
    if a.shape[0] != b.shape[0]:
        raise RuntimeError("Batch size mismatch")
    if a.shape[2] != b.shape[1]:
        raise RuntimeError("Contracting dimension (K) mismatch")


def _kmajor_f32(t: torch.Tensor) -> torch.Tensor:
    """A [batch, r, k] fp32 operand as the 3xTF32 GEMM reads it: contiguous along k, rows and batch
    items on 16-byte boundaries.  Returned as is when it already is; otherwise copied into a buffer
    whose rows are padded to a multiple of 4 elements (the padding is never read)."""
    nb, r, k = t.shape
    s0, s1, s2 = t.stride()
    if (t.data_ptr() % 16 == 0 and s2 == 1 and (r == 1 or (s1 > 0 and s1 % 4 == 0))
            and (nb == 1 or (s0 > 0 and s0 % 4 == 0))):
        return t
    buf = torch.empty((nb, r, (k + 3) // 4 * 4), dtype=t.dtype, device=t.device)
    buf[..., :k].copy_(t)
    return buf[..., :k]


def _out_rows(nb: int, m: int, n: int, dtype, device) -> torch.Tensor:
    """The [nb, m, n] output; for fp32, rows padded to 16 bytes when n is not a multiple of 4 and a
    row or batch stride is stepped (the caller returns a contiguous copy of the view)."""
    if dtype != torch.float32 or n % 4 == 0 or (m <= 1 and nb <= 1):
        return torch.empty((nb, m, n), dtype=dtype, device=device)
    return torch.empty((nb, m, (n + 3) // 4 * 4), dtype=dtype, device=device)[..., :n]


def _mn_f32_ok(b: torch.Tensor) -> bool:
    """An fp32 [batch, k, n] B stored contiguous along n with 16-byte aligned rows: cmpx_bmm_ws reads
    it through its workspace pass (no transposed copy)."""
    nb, k, _ = b.shape
    s0, s1, s2 = b.stride()
    return (b.data_ptr() % 16 == 0 and s2 == 1 and (k == 1 or (s1 > 0 and s1 % 4 == 0))
            and (nb == 1 or (s0 > 0 and s0 % 4 == 0)))


def _prepare_bmm(a, b, keep_mn_b=False):
    _check_bmm_args(a, b)
    if a.dtype != torch.float32:
        a = a if _mat_ok(a) else a.contiguous()
        b = b if _mat_ok(b) else b.contiguous()
    else:  # K-major A and B (B as the transpose of a k-contiguous [batch, n, k] buffer)
        a = _kmajor_f32(a)
        if not (keep_mn_b and _mn_f32_ok(b)):
            b = _kmajor_f32(b.transpose(1, 2)).transpose(1, 2)
    nb, m, _ = a.shape
    n = b.shape[2]
    c = _out_rows(nb, m, n, a.dtype, a.device)
    return a, b, c


def _bmm_desc(a, b, c) -> BmmDesc:
    d = BmmDesc()
    d.a, d.b, d.c = a.data_ptr(), b.data_ptr(), c.data_ptr()
    d.batch, d.m, d.k = a.shape
    d.n = b.shape[2]
    d.a_stride[:] = a.stride()
    d.b_stride[:] = b.stride()
    d.c_stride[:] = c.stride()
    d.dtype = _DTYPE[a.dtype]
    d.reserved = 0
    return d


@_traced("bmm")
def bmm(input, mat2):
    """Batched matmul on the sm_100a kernels.  Same contract as the reference's ops.bmm."""
    # fp32 with B stored MN-major: kept as it is when the workspace schedule takes it (its pass
    # writes B K-major), copied K-major otherwise
    a, b, c = _prepare_bmm(input, mat2, keep_mn_b=True)
    if c.numel() == 0:
        return c
    if a.shape[2] == 0:
        return c.zero_()
    desc = _bmm_desc(a, b, c)
    if a.dtype == torch.float32 and b.stride(1) != 1 and lib.cmpx_bmm_workspace_size(ctypes.byref(desc)) == 0:
        a, b, c = _prepare_bmm(input, mat2)
        desc = _bmm_desc(a, b, c)
    with torch.cuda.device(a.device):
        stream = _stream_handle(a.device)
        # fp32: the split-operand schedule when the product is large enough (same results)
        nbytes = lib.cmpx_bmm_workspace_size(ctypes.byref(desc))
        if nbytes:
            ws = _workspace(a.device, stream, nbytes)
            st = lib.cmpx_bmm_ws(ctypes.byref(desc), ws.data_ptr(), ws.numel(), stream)
        else:
            st = lib.cmpx_bmm(ctypes.byref(desc), stream)
    if st != OK:
        raise CmpxError("bmm", st)
    _post_check()
    return c if c.is_contiguous() else c.contiguous()


def bmm_plan(input, mat2) -> str:
    """Name of the tile-table entry ``bmm`` would run for these arguments."""
    a, b, c = _prepare_bmm(input, mat2)
    desc = _bmm_desc(a, b, c)
    buf = ctypes.create_string_buffer(128)
    st = lib.cmpx_bmm_plan(ctypes.byref(desc), buf, 128)
    if st != OK:
        raise CmpxError("bmm plan", st)
    return buf.value.decode()


def _prepare_small(input, mat2):
    _check_bmm_args(input, mat2)
    c = torch.empty((input.shape[0], input.shape[1], mat2.shape[2]), dtype=input.dtype, device=input.device)
    return _bmm_desc(input, mat2, c), c


@_traced("bmm_small")
def bmm_small(input, mat2):
    """Batched product of many tiny matrices (the reference's _small_bmm route): one fp32 dot
    product per output element on the GPU, operands read in place through their strides."""
    desc, c = _prepare_small(input, mat2)
    if c.numel() == 0:
        return c
    with torch.cuda.device(input.device):
        st = lib.cmpx_bmm_small(ctypes.byref(desc), _stream_handle(input.device))
    if st != OK:
        raise CmpxError("bmm_small", st)
    _post_check()
    return c


def bmm_small_plan(input, mat2) -> str:
    """Name of the kernel ``bmm_small`` runs for these arguments."""
    desc, _ = _prepare_small(input, mat2)
    buf = ctypes.create_string_buffer(128)
    st = lib.cmpx_bmm_small_plan(ctypes.byref(desc), buf, 128)
    if st != OK:
        raise CmpxError("bmm_small plan", st)
    return buf.value.decode()


# ---------------------------------------------------------------------------------------------
# linear  y = x W^T + b  (the reference's _C.linear, src/main.cpp:195-346)
# ---------------------------------------------------------------------------------------------

def _rows_ok(t: torch.Tensor) -> bool:
    """A 2-D operand the 16-bit TMA path reads in place: unit column stride, 16-byte aligned rows."""
    es = t.element_size()
    return (t.data_ptr() % 16 == 0 and t.stride(1) == 1
            and (t.shape[0] == 1 or (t.stride(0) > 0 and (t.stride(0) * es) % 16 == 0)))


def _prepare_linear(input, weight, bias):
    for name, t in (("input", input), ("weight", weight)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a Tensor")
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor")
    if input.dim() < 2:
        raise RuntimeError("Input dim >= 2")
    if weight.dim() != 2:
        raise RuntimeError("Weight dim == 2")
    if input.device != weight.device:
        raise RuntimeError("Device mismatch")
    n, k = weight.shape
    if input.shape[-1] != k:
        raise RuntimeError("Input shape mismatch with Weight")
    if input.dtype not in _DTYPE or weight.dtype != input.dtype:
        raise RuntimeError("linear: input/weight must share one dtype among float32/float16/bfloat16")
    if bias is not None:
        if not isinstance(bias, torch.Tensor) or bias.dim() != 1 or bias.shape[0] != n:
            raise RuntimeError("Bias must be 1D of size out_features")
        if bias.dtype != input.dtype or bias.device != input.device:
            raise RuntimeError("Bias dtype/device mismatch")
        bias = bias if (bias.stride(0) == 1 and bias.data_ptr() % 16 == 0) else bias.contiguous()
        if bias.data_ptr() % 16 != 0:
            bias = bias.clone()
    x = input.reshape(-1, k)
    if input.dtype == torch.float32:  # rows padded to 16 bytes where needed (3xTF32 GEMM)
        x = _kmajor_f32(x.unsqueeze(0))[0]
        w = _kmajor_f32(weight.unsqueeze(0))[0]
        y = _out_rows(1, x.shape[0], n, input.dtype, input.device)[0]
        return x, w, bias, y
    x = x if _rows_ok(x) else x.contiguous()
    w = weight if _rows_ok(weight) else weight.contiguous()
    y = torch.empty((x.shape[0], n), dtype=input.dtype, device=input.device)
    return x, w, bias, y


def _linear_desc(x, w, bias, y) -> LinearDesc:
    return LinearDesc(x.data_ptr(), w.data_ptr(), None if bias is None else bias.data_ptr(), y.data_ptr(),
                      x.shape[0], w.shape[0], w.shape[1], x.stride(0), w.stride(0), y.stride(0),
                      _DTYPE[x.dtype], 0)


@_traced("linear")
def linear(input, weight, bias=None):
    """F.linear on the sm_100a GEMM with the bias added in its epilogue.  Same contract as the
    reference's ops.linear (input [..., K], weight [N, K], bias [N] -> [..., N])."""
    x, w, b, y = _prepare_linear(input, weight, bias)
    out_shape = tuple(input.shape[:-1]) + (w.shape[0],)
    if y.numel() == 0:
        return y.contiguous().view(out_shape)
    if w.shape[1] == 0:
        return (y.zero_() if b is None else y.copy_(b.expand_as(y))).contiguous().view(out_shape)
    desc = _linear_desc(x, w, b, y)
    dev = x.device

    def run():
        stream = _stream_handle(dev)
        nbytes = lib.cmpx_linear_workspace_size(ctypes.byref(desc))  # fp32 split operands (same results)
        if nbytes:
            ws = _workspace(dev, stream, nbytes)
            return lib.cmpx_linear_ws(ctypes.byref(desc), ws.data_ptr(), ws.numel(), stream)
        return lib.cmpx_linear(ctypes.byref(desc), stream)
    if dev.index == torch.cuda.current_device():
        st = run()
    else:
        with torch.cuda.device(dev):
            st = run()
    if st != OK:
        raise CmpxError("linear", st)
    _post_check()
    return (y if y.is_contiguous() else y.contiguous()).view(out_shape)


def linear_plan(input, weight, bias=None) -> str:
    """Name of the tile-table entry ``linear`` would run for these arguments."""
    x, w, b, y = _prepare_linear(input, weight, bias)
    desc = _linear_desc(x, w, b, y)
    buf = ctypes.create_string_buffer(128)
    st = lib.cmpx_linear_plan(ctypes.byref(desc), buf, 128)
    if st != OK:
        raise CmpxError("linear plan", st)
    return buf.value.decode()


# ---------------------------------------------------------------------------------------------
# softmax over the last dimension (the einsum-attention chain's middle step)
# ---------------------------------------------------------------------------------------------

@_traced("softmax")
def softmax(input, dim=-1):
    """torch.softmax(input, dim=-1) on the sm_100a row-softmax kernel (fp32 arithmetic, output in
    the input's dtype).  Only the last dimension; the rows must be contiguous."""
    if not isinstance(input, torch.Tensor):
        raise TypeError("input must be a Tensor")
    if not input.is_cuda or input.dtype not in _DTYPE:
        raise RuntimeError("input must be a CUDA float32/float16/bfloat16 tensor")
    if input.dim() == 0 or dim not in (-1, input.dim() - 1):
        raise RuntimeError("only the last dimension is supported")
    x = input if input.is_contiguous() else input.contiguous()
    y = torch.empty_like(x, memory_format=torch.contiguous_format)
    if x.numel() == 0:
        return y
    cols = x.shape[-1]
    d = SoftmaxDesc()
    d.x, d.y = x.data_ptr(), y.data_ptr()
    d.rows, d.cols = x.numel() // cols, cols
    d.x_row_stride = d.y_row_stride = cols
    d.dtype = _DTYPE[x.dtype]
    d.reserved = 0
    with torch.cuda.device(x.device):
        st = lib.cmpx_softmax_rows(ctypes.byref(d), _stream_handle(x.device))
    if st != OK:
        raise CmpxError("softmax", st)
    _post_check()
    return y


def _prepare_rowstats(input, mat2):
    _check_bmm_args(input, mat2)
    if input.dtype == torch.float32:
        raise RuntimeError("bmm_rowstats: 16-bit operands only")
    nb, m, _ = input.shape
    n = mat2.shape[2]
    c = _out_rows(nb, m, n, input.dtype, input.device)
    stats = torch.empty((nb, (n + 63) // 64, m, 2), dtype=torch.float32, device=input.device)
    return _bmm_desc(input, mat2, c), c, stats


@_traced("bmm_rowstats")
def bmm_rowstats(input, mat2):
    """(c, stats): ``bmm(input, mat2)`` bit for bit (16-bit, both operands contiguous along k), and
    the row statistics of c: stats [batch, ceil(n / 64), m, 2] fp32, for every row and 64-column run
    the max of the stored values and the sum of exp(value - max) over the run."""
    d, c, stats = _prepare_rowstats(input, mat2)
    if c.numel():
        with torch.cuda.device(input.device):
            st = lib.cmpx_bmm_rowstats(ctypes.byref(d), stats.data_ptr(), _stream_handle(input.device))
        if st != OK:
            raise CmpxError("bmm_rowstats", st)
        _post_check()
    return c, stats


def bmm_rowstats_plan(input, mat2) -> str:
    """Name of the kernel ``bmm_rowstats`` runs for these operands."""
    d, _, stats = _prepare_rowstats(input, mat2)
    buf = ctypes.create_string_buffer(128)
    st = lib.cmpx_bmm_rowstats_plan(ctypes.byref(d), stats.data_ptr(), buf, 128)
    if st != OK:
        raise CmpxError("bmm_rowstats plan", st)
    return buf.value.decode()


def _prepare_softmax_product(a, b, stats):
    _check_bmm_args(a, b)
    if a.dtype == torch.float32:
        raise RuntimeError("softmax_product: 16-bit operands only")
    runs = (b.shape[2] + 63) // 64
    if (not isinstance(stats, torch.Tensor) or stats.dtype != torch.float32 or stats.device != a.device
            or tuple(stats.shape) != (a.shape[0], runs, a.shape[1], 2) or not stats.is_contiguous()):
        raise RuntimeError("softmax_product: stats must be the contiguous fp32 [batch, ceil(n / 64), m, 2] "
                           "row statistics of a @ b (bmm_rowstats)")
    y = torch.empty((a.shape[0], a.shape[1], b.shape[2]), dtype=a.dtype, device=a.device)
    d = _bmm_desc(a, b, y)
    d.c = None
    return d, y


@_traced("softmax_product")
def softmax_product(a, b, stats):
    """softmax(a @ b, dim=-1) computed from the operands (16-bit, a [batch, m, k] and b
    [batch, k, n] both contiguous along k, k <= 128) and the product's row statistics as
    ``bmm_rowstats`` returned them: the scores are recomputed on the tensor cores exactly as ``bmm``
    computes and rounds them, and never read back from memory."""
    d, y = _prepare_softmax_product(a, b, stats)
    if y.numel():
        with torch.cuda.device(a.device):
            st = lib.cmpx_softmax_product(ctypes.byref(d), stats.data_ptr(), y.data_ptr(), _stream_handle(a.device))
        if st != OK:
            raise CmpxError("softmax_product", st)
        _post_check()
    return y


def softmax_product_plan(a, b, stats) -> str:
    """Name of the kernel ``softmax_product`` runs for these operands."""
    d, y = _prepare_softmax_product(a, b, stats)
    buf = ctypes.create_string_buffer(128)
    st = lib.cmpx_softmax_product_plan(ctypes.byref(d), stats.data_ptr(), y.data_ptr(), buf, 128)
    if st != OK:
        raise CmpxError("softmax_product plan", st)
    return buf.value.decode()


def selftest_wait_timeout(timeout_ns: int, device=None) -> None:
    """Launch the bounded-wait self-test kernel (see cmpx_selftest_wait_timeout)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        st = lib.cmpx_selftest_wait_timeout(int(timeout_ns), _stream_handle(dev))
    if st != OK:
        raise CmpxError("selftest", st)
