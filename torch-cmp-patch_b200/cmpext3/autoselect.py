"""Per-signature dispatch record: which tile-table entry serves each (op, shape, dtype) signature.

The reference decided native-versus-stock at run time: the first call per signature ran both, compared
outputs, timed both and kept the faster one (cmpext3/autoselect.py:290-364 in the reference).  On a
B200 the choice is not a bet: the sm_100a kernels are built for these shapes, and the kernel and its
tile configuration are a fixed function of dtype, shape and layout, chosen inside the native library
(``cmpx_attn_plan`` / ``cmpx_bmm_plan`` in include/cmpx_b200.h).  What is kept from the reference is
the bookkeeping its callers rely on:

* ``enabled()``, ``reset()``, ``report()``, ``format_report()`` and ``cmpext3.autoselect_report()``
  still work; a decision now records the tile-table entry that ran (or why the native op declined);
* a signature whose native call raised ``RuntimeError``/``TypeError`` on first use is served by stock
  from then on without re-trying the kernel (reference ``choose``, :302-308, :319-322); a one-off
  failure after a good first call is served by stock for that call only (reference :302-308);
* the table of signatures is capped per op (reference ``_MAX_SIGNATURES_PER_OP``, :84); past the cap
  calls run the kernel directly without being recorded.
* ``_mismatch`` / ``_TOLERANCE`` (reference :93-97, :229-261) stay as the correctness rule the tests
  apply -- not on the hot path, which does not run stock next to the kernel any more.

Knobs: ``CMPEXT3_AUTOSELECT=0`` turns the record off (every call runs the kernel, stock only if it
raises -- the same routing); ``CMPEXT3_VERBOSE=1`` prints each new decision to stderr.
"""
from __future__ import annotations

import math
import os
import sys
from typing import Any, Callable

import torch


def _flag(name: str, default: str = "0") -> bool:
    return os.environ.get(name, default) not in ("0", "", "false", "False")


_ENABLED = _flag("CMPEXT3_AUTOSELECT", "1")
_VERBOSE = _flag("CMPEXT3_VERBOSE", "0")

# Signatures recorded per op before the record stops growing (dynamic shapes, e.g. attention over a
# variable sequence length, would otherwise grow the table without bound).
_MAX_SIGNATURES_PER_OP = 4096

# Correctness rule of the reference (max |native - stock| / max |stock|), kept for the tests.
_TOLERANCE = {
    torch.float32: 1e-3,
    torch.float16: 3e-2,
    torch.bfloat16: 5e-2,
}


class Decision:
    """Which implementation serves one call signature, and (for the kernel) which table entry."""

    __slots__ = ("op", "use_native", "entry", "note")

    def __init__(self, op: str, use_native: bool, entry: str | None = None, note: str = ""):
        self.op = op
        self.use_native = use_native
        self.entry = entry
        self.note = note

    def __repr__(self) -> str:
        which = "cmpext3" if self.use_native else "stock"
        detail = self.entry or self.note
        return f"<{self.op}: {which} ({detail})>"


_decisions: dict[Any, Decision] = {}
_counts: dict[str, int] = {}


def enabled() -> bool:
    return _ENABLED


def reset() -> None:
    """Forget every recorded decision."""
    _decisions.clear()
    _counts.clear()


def report() -> list[Decision]:
    """Every decision recorded so far: stock-served signatures first, then by op name."""
    return sorted(_decisions.values(), key=lambda d: (d.use_native, d.op, d.entry or ""))


def format_report() -> str:
    if not _decisions:
        return "cmpext3: no kernel decisions made yet (no eligible op has run)."
    lines = [f"cmpext3: {len(_decisions)} signature(s), tile-table entries:"]
    for d in report():
        lines.append(f"  {'cmpext3' if d.use_native else 'stock  '}  {d.op:<16} {d.entry or d.note}")
    return "\n".join(lines)


def _log(message: str) -> None:
    if _VERBOSE:
        sys.stderr.write(f"[cmpext3] {message}\n")
        sys.stderr.flush()


def choose(op: str, key: Any, native_call: Callable, stock_call: Callable,
           plan: Callable[[], str] | None = None) -> Any:
    """Serve one call: the kernel if this signature runs natively, stock otherwise."""
    decision = _decisions.get(key)
    if decision is not None:
        if not decision.use_native:
            return stock_call()
        try:
            return native_call()
        except (RuntimeError, TypeError):
            return stock_call()  # one-off failure: keep the decision, serve this call from stock

    if _counts.get(op, 0) >= _MAX_SIGNATURES_PER_OP:
        try:
            return native_call()
        except (RuntimeError, TypeError):
            return stock_call()

    _counts[op] = _counts.get(op, 0) + 1
    try:
        out = native_call()
    except (RuntimeError, TypeError) as exc:
        _decisions[key] = Decision(op, False, note=f"native kernel raised {type(exc).__name__}: {exc}")
        _log(f"{op}: stock -- {_decisions[key].note}")
        return stock_call()
    entry = None
    if plan is not None:
        try:
            entry = plan()
        except Exception as exc:  # noqa: BLE001 -- the name is informational only
            entry = f"(plan unavailable: {exc})"
    _decisions[key] = Decision(op, True, entry=entry or "native")
    _log(f"{op}: cmpext3 -- {_decisions[key].entry}")
    return out


def _mismatch(native_out: Any, stock_out: Any, tol: float | None = None) -> str | None:
    """None if the two agree within the reference's rule; else a short reason."""
    if not isinstance(native_out, torch.Tensor) or not isinstance(stock_out, torch.Tensor):
        return None
    if tuple(native_out.shape) != tuple(stock_out.shape):
        return f"shape {tuple(native_out.shape)} vs stock {tuple(stock_out.shape)}"
    a = native_out.detach().reshape(-1).double().cpu()
    b = stock_out.detach().reshape(-1).double().cpu()
    if not torch.isfinite(a).all().item():
        return "native output contains NaN/Inf"
    diff = (a - b).abs().max().item() if a.numel() else 0.0
    scale = b.abs().max().item() if b.numel() else 0.0
    if not math.isfinite(diff):
        return "native output contains NaN/Inf"
    rel = diff / scale if scale > 0.0 else diff
    limit = tol if tol is not None else _TOLERANCE.get(stock_out.dtype, 1e-3)
    if rel > limit:
        return f"max relative difference {rel:.2e} exceeds {limit:.0e}"
    return None
