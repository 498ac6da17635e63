"""torch.einsum planned as batched matrix products, so the bmm patch (and its sm_100a kernel) applies.

This module restates the reference's planner (cmpext3/einsum_ops.py:25-131 in the reference):
its identifiers (``Unsupported``, ``parse``, ``_sizes``, ``_pair``, ``einsum``, ``supported``) and
its step order are kept on purpose, because the planner's results and its fall-back decisions are
part of the drop-in contract (the same equations must reach the same bmm calls, and the same ones
must go back to stock einsum).  The steps:

* operands are contracted left to right, two at a time;
* in each pair, indices that appear in only one operand and are not needed later are summed out
  first; the remaining indices split into batch (in both operands and kept), contracted (in both,
  not kept), and free-left / free-right (kept, one operand only);
* the pair becomes one ``bmm([batch, M, K], [batch, K, N])`` over permuted views, reshaped and
  permuted back to the requested output order; size-1 dimensions broadcast;
* unsupported forms raise ``Unsupported`` (so the caller falls back to stock einsum): an ellipsis,
  an index repeated inside one operand, a repeated or unknown output index, an operand count or
  rank that does not match the equation, or incompatible sizes.

Unlike the reference's native bmm, the bmm this feeds (``cmpext3.ops.bmm``) reads a permuted operand
in place: the ``bhjd -> (bh, d, j)`` view of K in an attention-score einsum reaches the kernel as a
K-major operand without a copy.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch


class Unsupported(Exception):
    """The equation is outside what this planner handles; use stock einsum."""


def parse(equation: str, n_operands: int) -> Tuple[List[str], str]:
    """Split an equation into operand terms and the output term (implicit output resolved)."""
    eq = equation.replace(" ", "")
    if "." in eq:
        raise Unsupported("ellipsis")
    if "->" in eq:
        lhs, out = eq.split("->", 1)
        if "->" in out:
            raise Unsupported("bad output")
    else:
        lhs = eq
        seen: dict[str, int] = {}
        for ch in lhs:
            if ch != ",":
                seen[ch] = seen.get(ch, 0) + 1
        out = "".join(sorted(ch for ch, n in seen.items() if n == 1))
    terms = lhs.split(",")
    if len(terms) != n_operands:
        raise Unsupported("operand count")
    if any(len(set(t)) != len(t) for t in terms):
        raise Unsupported("repeated index in one operand")
    if len(set(out)) != len(out) or not set(out) <= set(lhs.replace(",", "")):
        raise Unsupported("bad output")
    return terms, out


def _sizes(terms: Sequence[str], operands: Sequence[torch.Tensor]) -> dict:
    """Size of every index; 1 broadcasts against any size."""
    size: dict[str, int] = {}
    for term, x in zip(terms, operands):
        if x.dim() != len(term):
            raise Unsupported("rank mismatch")
        for ch, n in zip(term, x.shape):
            n = int(n)
            prev = size.get(ch)
            if prev is not None and prev != n and prev != 1 and n != 1:
                raise Unsupported("size mismatch")
            size[ch] = n if prev is None else max(prev, n)
    return size


def _sum_out(x: torch.Tensor, term: str, keep: set) -> Tuple[torch.Tensor, str]:
    """Sum over the indices of ``term`` that are not in ``keep``."""
    gone = [i for i, ch in enumerate(term) if ch not in keep]
    if not gone:
        return x, term
    return x.sum(dim=gone), "".join(ch for ch in term if ch in keep)


def _prod(size: dict, idx: Sequence[str]) -> int:
    p = 1
    for ch in idx:
        p *= size[ch]
    return p


def _pair(a: torch.Tensor, ta: str, b: torch.Tensor, tb: str, out: str, size: dict,
          bmm: Callable) -> torch.Tensor:
    """Contract a[ta] with b[tb] into [out] with one batched matmul."""
    a, ta = _sum_out(a, ta, set(tb) | set(out))
    b, tb = _sum_out(b, tb, set(ta) | set(out))
    batch = [ch for ch in out if ch in ta and ch in tb]
    left = [ch for ch in out if ch in ta and ch not in tb]
    right = [ch for ch in out if ch in tb and ch not in ta]
    contract = [ch for ch in ta if ch in tb and ch not in out]
    a = a.expand(tuple(size[ch] for ch in ta)).permute(tuple(ta.index(ch) for ch in batch + left + contract))
    b = b.expand(tuple(size[ch] for ch in tb)).permute(tuple(tb.index(ch) for ch in batch + contract + right))
    nb, m, k, n = _prod(size, batch), _prod(size, left), _prod(size, contract), _prod(size, right)
    r = bmm(a.reshape(nb, m, k), b.reshape(nb, k, n))
    order = batch + left + right
    r = r.reshape(tuple(size[ch] for ch in order))
    if order == list(out):
        return r
    return r.permute(tuple(order.index(ch) for ch in out))


def einsum(equation: str, operands: Sequence[torch.Tensor], bmm: Optional[Callable] = None) -> torch.Tensor:
    """Evaluate ``equation`` as a chain of batched matmuls (reference einsum_ops.py:101-121);
    an equation outside the planner raises ``Unsupported``."""
    bmm = bmm or torch.bmm
    terms, out = parse(equation, len(operands))
    size = _sizes(terms, operands)
    if len(operands) == 1:
        x, t = _sum_out(operands[0], terms[0], set(out))
        return x.permute(tuple(t.index(ch) for ch in out))
    x, tx = operands[0], terms[0]
    last = len(operands) - 1
    for i in range(1, len(operands)):
        if i == last:
            target = out
        else:
            needed = set(out).union(*(set(t) for t in terms[i + 1:]))
            target = "".join(ch for ch in dict.fromkeys(tx + terms[i]) if ch in needed)
        x = _pair(x, tx, operands[i], terms[i], target, size, bmm)
        tx = target
    return x


def supported(equation: str, operands: Sequence[torch.Tensor]) -> Optional[str]:
    """The reason ``einsum`` would refuse the equation, or None when it plans it
    (reference einsum_ops.py:124-131)."""
    try:
        terms, _ = parse(equation, len(operands))
        _sizes(terms, operands)
    except Unsupported as exc:
        return str(exc)
    return None
