"""cmpext3 (B200 edition) -- drop-in replacement for the attention / batched-matmul hot path of
cmpext3 (WifiLast/torch-cmp-patch), running hand-written sm_100a kernels.

Importing the package monkeypatches, exactly where the reference does (cmpext3/__init__.py:741-781,
auto-run at :822-823 of the reference):

    F.scaled_dot_product_attention  -> cmpext3.ops.attention(query, key, value, scale, is_causal)
    torch.bmm                       -> cmpext3.ops.bmm(input, mat2)
    torch.matmul (2D / 3D)          -> cmpext3.ops.bmm
    torch.einsum                    -> einsum_ops planner -> torch.bmm (patched)
    F.linear (so nn.Linear)         -> cmpext3.ops.linear(input, weight, bias)

and, beyond the reference, the middle step of an einsum / bmm attention chain
(``einsum('bhid,bhjd->bhij') -> softmax(-1) -> einsum('bhij,bhjd->bhid')``):

    torch.softmax / F.softmax / Tensor.softmax over the last dimension of a tensor that one of the
    patched einsum / bmm / matmul calls above returned -> cmpext3.ops.softmax

(every other softmax stays stock, as in the reference, which does not patch softmax at all).

with the reference's wrapper signatures, gates and stock bail-outs: stock PyTorch runs when autograd
is live for an input, when a tensor is not a CUDA fp16/fp32/bf16 tensor, when SDPA gets an
``attn_mask`` that is neither boolean nor in the query's dtype, ``dropout_p > 0`` or a non-4D
query (masks run natively beyond the reference, which sent every masked call to stock), when bmm/matmul get ``out=`` or mixed dtypes, and
whenever the native op raises ``RuntimeError``/``TypeError`` for an argument outside its tile table.

What changed underneath: the kernels are tcgen05/TMA/TMEM kernels for B200 in a C-ABI library
(include/cmpx_b200.h), bf16 is computed natively (the reference converted it to fp16 for attention
and to fp32 for bmm), and the runtime native-versus-stock race is replaced by a fixed tile table
(see cmpext3.autoselect).  The rest of the reference (conv, norms, activations, TensorRT, NVML
clock/power changes) is not part of this package; in particular nothing here changes GPU clocks or
power limits.  fp32 bmm / matmul / einsum / linear run on a 3xTF32 tensor-core GEMM (k > 8192 in
chunks of at most 8192, summed in fp32).

    import cmpext3            # patches on import
    cmpext3.disable(); cmpext3.enable()

Set CMPEXT3_AUTOPATCH=0 to import without patching; CMPEXT3_DISABLE_OPS=attention,bmm,matmul,einsum,
softmax,linear pins named ops to stock; CMPEXT3_VERBOSE=1 logs each new signature's tile-table entry;
cmpext3.autoselect_report() lists them; CMPEXT3_NVTX=1 puts an NVTX range around every native call.

SAFETY: the kernels are forward-only (no autograd); every patched call falls back to stock when
autograd is live, as in the reference.
"""
from __future__ import annotations

import os
import weakref
from typing import Any, Callable

import torch
import torch.nn.functional as F

try:
    from . import _native as _C
except ImportError as exc:  # pragma: no cover
    raise ImportError(
        "cmpext3 native library not built. Run: python torch-cmp-patch_b200/build.py"
    ) from exc

# Raw, unpatched access to the native ops (attention, bmm) for manual use.
ops = _C

from . import autoselect  # noqa: E402
from . import einsum_ops  # noqa: E402

_SUPPORTED_DTYPES = (torch.float16, torch.float32, torch.bfloat16)
_ORIGINALS: dict[tuple[Any, str], Callable] = {}
_ENABLED = False


def _grad_safe(*tensors: Any) -> bool:
    """True if swapping in a kernel with no autograd support is safe."""
    if hasattr(torch, "is_inference_mode_enabled") and torch.is_inference_mode_enabled():
        return True
    if not torch.is_grad_enabled():
        return True
    return not any(isinstance(t, torch.Tensor) and t.requires_grad for t in tensors)


def _usable(*tensors: Any) -> bool:
    """True if every tensor argument is a CUDA fp16/fp32/bf16 tensor."""
    for t in tensors:
        if isinstance(t, torch.Tensor) and (not t.is_cuda or t.dtype not in _SUPPORTED_DTYPES):
            return False
    return True


# CMPEXT3_DISABLE_OPS=attention,bmm pins named ops to stock ("attention" is the op name of
# F.scaled_dot_product_attention, as in the reference).
_OP_ALIASES = {"scaled_dot_product_attention": "attention"}
_DISABLED_OPS = frozenset(
    part.strip() for part in os.environ.get("CMPEXT3_DISABLE_OPS", "").split(",") if part.strip()
)


def _install(target: Any, name: str, wrapper: Callable) -> None:
    if name in _DISABLED_OPS or _OP_ALIASES.get(name, name) in _DISABLED_OPS:
        return
    key = (target, name)
    if key not in _ORIGINALS:
        _ORIGINALS[key] = getattr(target, name)
    _keep_scriptable(wrapper, _ORIGINALS[key])
    setattr(target, name, wrapper)


def _keep_scriptable(wrapper: Callable, original: Callable) -> None:
    """Make torch.jit.script treat ``wrapper`` as the stock ``original``.

    TorchScript resolves torch.bmm & co. by object identity; a scripted function that calls a
    patched op would otherwise try to compile the Python wrapper.  C++ builtins are aliased to the
    wrapper; Python functions get their compiled original (or overloads) cached for the wrapper.
    """
    from torch.jit import _builtins, _state
    op = _builtins._find_builtin(original)
    if op is not None:
        _builtins._register_builtin(wrapper, op)
        return
    from torch import _jit_internal
    from torch.jit import _script
    try:
        if _jit_internal._get_fn_overloads(_jit_internal._qualified_name(original)):
            _state._set_jit_overload_cache(wrapper, _script._get_overloads(original))
        else:
            _state._set_jit_function_cache(wrapper, torch.jit.script(original))
    except Exception:  # noqa: BLE001 -- an original that does not script stays as it is
        pass


def _restore(target: Any, name: str) -> None:
    original = _ORIGINALS.pop((target, name), None)
    if original is not None:
        setattr(target, name, original)


_DTYPE_TAG = {torch.float16: "fp16", torch.float32: "fp32", torch.bfloat16: "bf16"}


def _dispatch(op: str, ref: torch.Tensor, key: tuple, native_call: Callable,
              stock_call: Callable, plan: Callable[[], str] | None = None) -> Any:
    """Run the native op for this signature (stock if it declines).

    With the record on (default) the first call per signature notes the tile-table entry, and a
    signature the kernels decline is remembered as stock (cmpext3.autoselect).  With
    CMPEXT3_AUTOSELECT=0: kernel, and stock only if it raises.
    """
    if autoselect.enabled():
        try:
            return autoselect.choose(f"{op} {_DTYPE_TAG.get(ref.dtype, ref.dtype)}", key,
                                     native_call, stock_call, plan)
        except TypeError as exc:
            if "unhashable" not in str(exc):
                raise
    try:
        return native_call()
    except (RuntimeError, TypeError):
        return stock_call()


# ---------------------------------------------------------------------------------------------
# Wrappers (signatures and gates as in the reference: __init__.py:423-501, :609-633)
# ---------------------------------------------------------------------------------------------

def _patched_linear(input, weight, bias=None):
    """F.linear with the reference's gates (__init__.py:410-420): stock under live autograd, for
    non-CUDA / unsupported dtypes, for input.dim() < 2 or a non-2-D weight, for fp16 with an odd
    out_features; the native op raising (misaligned 16-bit rows) also serves the call from stock."""
    orig = _ORIGINALS[(F, "linear")]
    if not (_grad_safe(input, weight, bias) and _usable(input, weight)):
        return orig(input, weight, bias)
    if input.dim() < 2 or weight.dim() != 2:
        return orig(input, weight, bias)
    if input.dtype == torch.float16 and weight.size(0) % 2 != 0:
        return orig(input, weight, bias)
    return _dispatch("linear", input, (input.shape, input.dtype, weight.shape, bias is not None),
                     lambda: _C.linear(input, weight, bias),
                     lambda: orig(input, weight, bias),
                     lambda: _C.linear_plan(input, weight, bias))


def _patched_matmul(input, other, *, out=None):
    orig = _ORIGINALS[(torch, "matmul")]
    if out is not None or not (_grad_safe(input, other) and _usable(input, other)):
        return orig(input, other) if out is None else orig(input, other, out=out)
    if input.dtype != other.dtype:
        return orig(input, other)
    if input.dim() == 2 and other.dim() == 2:
        native = lambda: _C.bmm(input.unsqueeze(0), other.unsqueeze(0)).squeeze(0)  # noqa: E731
        plan = lambda: _C.bmm_plan(input.unsqueeze(0), other.unsqueeze(0))  # noqa: E731
    elif input.dim() == 3 and other.dim() == 3:
        if _small_bmm_eligible(input, other):
            return _dispatch("bmm_small", input, (input.shape, input.dtype, other.shape),
                             lambda: _small_bmm(input, other), lambda: orig(input, other),
                             lambda: _C.bmm_small_plan(input, other))
        native = lambda: _C.bmm(input, other)  # noqa: E731
        plan = lambda: _C.bmm_plan(input, other)  # noqa: E731
    else:
        return orig(input, other)
    return _note_product(_dispatch("matmul", input, (input.shape, input.dtype, other.shape),
                                   native, lambda: orig(input, other), plan))


# Many tiny matrices (M*K*N <= 32768 per item): routed as in the reference (__init__.py:440-464),
# with the same threshold variable, but computed by the native small-matrix kernel (one fp32 dot
# product per output element, no [batch, M, K, N] intermediate) instead of an eager broadcast
# multiply + sum.  CMPEXT3_SMALL_BMM_CHUNK, which bounded that intermediate, is still read for
# compatibility and has nothing left to bound.
_SMALL_BMM_MAX_MKN = int(os.environ.get("CMPEXT3_SMALL_BMM_MAX_MKN", "32768"))
_SMALL_BMM_CHUNK = int(os.environ.get("CMPEXT3_SMALL_BMM_CHUNK", str(1 << 25)))


def _small_bmm_eligible(a: torch.Tensor, b: torch.Tensor) -> bool:
    return (a.dim() == 3 and b.dim() == 3 and a.size(0) == b.size(0) and a.size(2) == b.size(1)
            and a.size(1) * a.size(2) * b.size(2) <= _SMALL_BMM_MAX_MKN)


def _small_bmm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return _C.bmm_small(a, b)


def _patched_bmm(input, mat2, *, out=None):
    orig = _ORIGINALS[(torch, "bmm")]
    if out is not None or not (_grad_safe(input, mat2) and _usable(input, mat2)):
        return orig(input, mat2) if out is None else orig(input, mat2, out=out)
    if input.dtype != mat2.dtype:
        return orig(input, mat2)
    if _small_bmm_eligible(input, mat2):
        return _dispatch("bmm_small", input, (input.shape, input.dtype, mat2.shape),
                         lambda: _small_bmm(input, mat2),
                         lambda: orig(input, mat2),
                         lambda: _C.bmm_small_plan(input, mat2))
    made = {}
    if _fusable(input, mat2):
        # a product a softmax may follow: the same product, with its row statistics
        def native():
            made["native"], made["stats"] = _C.bmm_rowstats(input, mat2)
            return made["native"]

        def plan():
            return _C.bmm_rowstats_plan(input, mat2)
    else:
        def native():
            made["native"] = r = _C.bmm(input, mat2)
            return r

        def plan():
            return _C.bmm_plan(input, mat2)
    c = _note_product(_dispatch("bmm", input, (input.shape, input.dtype, mat2.shape), native,
                                lambda: orig(input, mat2), plan))
    if made.get("native") is c and "stats" in made:
        _note_operands(c, input, mat2, made["stats"])
    return c


# Tensors returned by the patched einsum / bmm / matmul, keyed by id and held weakly: a softmax
# over the last dimension of one of them is the middle step of an attention chain, and only such a
# softmax is diverted to the native row-softmax kernel.
_PRODUCED: dict[int, weakref.ref] = {}


def _note_product(t: Any) -> Any:
    if isinstance(t, torch.Tensor):
        key = id(t)

        def _forget(ref, key=key):
            if _PRODUCED.get(key) is ref:
                del _PRODUCED[key]
        _PRODUCED[key] = weakref.ref(t, _forget)
    return t


def _is_product(t: Any) -> bool:
    ref = _PRODUCED.get(id(t))
    return ref is not None and ref() is t


# Operands and row statistics of a product the native bmm kernel computed, kept (with the in-place
# version counters) while the product lives, when a softmax over the product's last dimension can be
# recomputed from them instead of reading the product back: 16-bit, both operands contiguous along
# the contracted dimension, k <= 128, a product row of at least 128 elements (what attention scores
# look like).  Off by default (CMPEXT3_FUSED_SOFTMAX=1 turns it on): on a B200 the statistics cost
# the scores product one exponential per element, which takes longer than the softmax's read of the
# score tensor that the recompute saves (the C3 chain: 0.401 ms fused against 0.393 ms with the
# row-softmax kernel).
_FUSED_SOFTMAX = os.environ.get("CMPEXT3_FUSED_SOFTMAX", "0") not in ("0", "", "false", "False")
_OPERANDS: dict[int, tuple] = {}


def _fusable(a: torch.Tensor, b: torch.Tensor) -> bool:
    return (_FUSED_SOFTMAX and a.dtype in (torch.float16, torch.bfloat16) and a.dim() == 3 and b.dim() == 3
            and 1 <= a.shape[2] <= 128 and b.shape[2] >= 128 and b.shape[2] % 8 == 0
            and a.stride(2) == 1 and b.stride(1) == 1)


def _note_operands(t: torch.Tensor, a: torch.Tensor, b: torch.Tensor, stats: torch.Tensor) -> None:
    if not _fusable(a, b):
        return
    key = id(t)

    def _forget(ref, key=key):
        rec = _OPERANDS.get(key)
        if rec is not None and rec[0] is ref:
            del _OPERANDS[key]
    _OPERANDS[key] = (weakref.ref(t, _forget), a, b, stats, t._version, a._version, b._version)


def _operands_of(t: torch.Tensor):
    """(a, b, stats) with t == a @ b unchanged since it was computed (t contiguous, [.., m, n] rows
    of the [batch, m, n] product) and stats its row statistics, or None."""
    rec = _OPERANDS.get(id(t))
    if rec is None or rec[0]() is not t or not t.is_contiguous():
        return None
    _, a, b, stats, tv, av, bv = rec
    if t._version != tv or a._version != av or b._version != bv:
        return None
    return a, b, stats


def _patched_einsum(*args, **kwargs):
    """torch.einsum planned as batched matmuls (einsum_ops) so the bmm patch applies."""
    orig = _ORIGINALS[(torch, "einsum")]
    if kwargs or len(args) < 2 or not isinstance(args[0], str):
        return orig(*args, **kwargs)
    eq = args[0]
    operands = args[1:]
    if len(operands) == 1 and isinstance(operands[0], (list, tuple)):
        operands = tuple(operands[0])
    if not operands or not all(isinstance(t, torch.Tensor) for t in operands):
        return orig(*args)
    if not (_grad_safe(*operands) and _usable(*operands)) or len({t.dtype for t in operands}) != 1:
        return orig(*args)
    if einsum_ops.supported(eq, operands) is not None:
        return orig(*args)
    last = {}

    def bmm_noting(x, y):  # the planner's products go through the patched bmm; keep the last one
        last["r"] = r = torch.bmm(x, y)
        return r
    out = _note_product(_dispatch("einsum", operands[0],
                                  (eq.replace(" ", ""), tuple(tuple(t.shape) for t in operands)),
                                  lambda: einsum_ops.einsum(eq, operands, bmm=bmm_noting),
                                  lambda: orig(*args)))
    # An output that is the last product itself, reshaped (same memory, same rows), keeps that
    # product's operands: e.g. 'bhid,bhjd->bhij' returns bmm([bh,i,d], [bh,d,j]).view(b,h,i,j).
    r = last.get("r")
    if (r is not None and isinstance(out, torch.Tensor) and out is not r and out.is_contiguous()
            and r.is_contiguous() and out.data_ptr() == r.data_ptr() and out.numel() == r.numel()
            and out.dim() > 0 and r.dim() > 0 and out.shape[-1] == r.shape[-1]):
        ops = _operands_of(r)
        if ops is not None:
            _note_operands(out, *ops)
    return out


def _softmax(input, dim, dtype, stock_call: Callable):
    """Native softmax for the last dimension of a tensor a patched einsum / bmm / matmul returned
    (same dtype out): recomputed from the product's operands and row statistics when they describe
    it, else the row kernel reading it; stock otherwise."""
    if (isinstance(input, torch.Tensor) and dim is not None and (dtype is None or dtype == input.dtype)
            and input.dim() > 0 and isinstance(dim, int) and dim in (-1, input.dim() - 1)
            and _is_product(input) and _grad_safe(input) and _usable(input)):
        ops = _operands_of(input)
        if ops is not None:
            # the scores are recomputed from the product's operands instead of read back
            a, b, stats = ops
            return _dispatch("softmax_product", input, (tuple(input.shape), input.dtype, tuple(a.shape)),
                             lambda: _C.softmax_product(a, b, stats).view(input.shape), stock_call,
                             lambda: _C.softmax_product_plan(a, b, stats))
        return _dispatch("softmax", input, (tuple(input.shape), input.dtype),
                         lambda: _C.softmax(input, -1), stock_call)
    return stock_call()


def _patched_torch_softmax(input, dim, dtype=None, **kwargs):
    orig = _ORIGINALS[(torch, "softmax")]
    if kwargs:
        return orig(input, dim, dtype=dtype, **kwargs)
    return _softmax(input, dim, dtype, lambda: orig(input, dim, dtype=dtype))


def _patched_f_softmax(input, dim=None, _stacklevel=3, dtype=None):
    orig = _ORIGINALS[(F, "softmax")]
    return _softmax(input, dim, dtype,
                    lambda: orig(input, dim=dim, _stacklevel=_stacklevel, dtype=dtype))


def _patched_tensor_softmax(self, dim, dtype=None):
    orig = _ORIGINALS[(torch.Tensor, "softmax")]
    return _softmax(self, dim, dtype, lambda: orig(self, dim, dtype=dtype))


def _patched_sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False,
                  scale=None, **kwargs):
    orig = _ORIGINALS[(F, "scaled_dot_product_attention")]
    # Gates as in the reference (__init__.py:609-633), except that an attn_mask on the query's device
    # runs natively too -- boolean, or additive in the query's dtype; other masks stay stock.
    mask_ok = attn_mask is None or (
        isinstance(attn_mask, torch.Tensor) and attn_mask.device == query.device
        and attn_mask.dtype in (torch.bool, query.dtype))
    if (not mask_ok or dropout_p != 0.0
            or query.dim() != 4 or not _grad_safe(query, key, value)
            or not _usable(query, key, value)):
        return orig(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                    is_causal=is_causal, scale=scale, **kwargs)
    if key.dim() == 4 and key.size(1) != query.size(1) and not kwargs.get("enable_gqa"):
        # unequal head counts without enable_gqa: torch's own error / behaviour
        return orig(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                    is_causal=is_causal, scale=scale, **kwargs)
    if attn_mask is None:
        return _dispatch("attention", query,
                         (query.shape, query.dtype, key.shape, value.shape, scale, is_causal),
                         lambda: _C.attention(query, key, value, scale, is_causal),
                         lambda: orig(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                                      is_causal=is_causal, scale=scale, **kwargs),
                         lambda: _C.attention_plan(query, key, value, scale, is_causal))
    return _dispatch("attention", query,
                     (query.shape, query.dtype, key.shape, value.shape, scale, is_causal,
                      tuple(attn_mask.shape), attn_mask.dtype),
                     lambda: _C.attention(query, key, value, scale, is_causal, attn_mask),
                     lambda: orig(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                                  is_causal=is_causal, scale=scale, **kwargs),
                     lambda: _C.attention_plan(query, key, value, scale, is_causal, attn_mask))


def enable() -> None:
    """Patch torch / torch.nn.functional so eligible calls run on the sm_100a kernels."""
    global _ENABLED
    if _ENABLED:
        return
    _install(F, "linear", _patched_linear)
    _install(torch, "matmul", _patched_matmul)
    _install(torch, "bmm", _patched_bmm)
    _install(torch, "einsum", _patched_einsum)
    if hasattr(F, "scaled_dot_product_attention"):
        _install(F, "scaled_dot_product_attention", _patched_sdpa)
    _install(torch, "softmax", _patched_torch_softmax)
    _install(F, "softmax", _patched_f_softmax)
    _install(torch.Tensor, "softmax", _patched_tensor_softmax)
    _ENABLED = True


def disable() -> None:
    """Restore every patched function to the stock PyTorch implementation."""
    global _ENABLED
    for target, name in list(_ORIGINALS.keys()):
        _restore(target, name)
    _ENABLED = False


def is_enabled() -> bool:
    return _ENABLED


def autoselect_report() -> str:
    """Every signature seen so far with the tile-table entry (or stock) that served it."""
    return autoselect.format_report()


if os.environ.get("CMPEXT3_AUTOPATCH", "1") != "0":
    enable()
