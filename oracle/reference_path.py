"""The reference's own CPU path for the hot ops (TEST INFRASTRUCTURE ONLY -- see oracle/__init__.py).

cmpext3's wrappers route CPU tensors to the stock PyTorch ops they saved at enable() time
(reference cmpext3/__init__.py:609-633 ``_patched_sdpa``: ``_usable`` fails for a CPU tensor, so
``orig(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=..., scale=...)`` runs; :467-479
``_patched_bmm`` -> ``orig(input, mat2)``; :482-501 ``_patched_einsum`` -> ``orig(*args)``; :410-420
``_patched_linear`` -> ``orig(input, weight, bias)``).  The calls
below are those calls, made on CPU tensors with the host's threads.
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

# Captured at import: the oracle must never see a patched op.
_SDPA = F.scaled_dot_product_attention
_BMM = torch.bmm
_EINSUM = torch.einsum
_SOFTMAX = torch.softmax
_LINEAR = F.linear


def set_threads(n: int | None = None) -> int:
    """Use all host cores (or n) for the CPU path; returns the thread count in effect."""
    n = n or os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale=None, is_causal: bool = False):
    """Stock CPU SDPA as the reference's wrapper calls it for a CPU tensor."""
    assert q.device.type == "cpu"
    return _SDPA(q, k, v, attn_mask=None, dropout_p=0.0, is_causal=is_causal, scale=scale)


def bmm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    assert a.device.type == "cpu"
    return _BMM(a, b)


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """Stock CPU F.linear as the reference's ``_patched_linear`` (cmpext3/__init__.py:410-420) calls it
    for a CPU tensor: ``orig(input, weight, bias)``."""
    assert x.device.type == "cpu"
    return _LINEAR(x, w, b)


def einsum(eq: str, *operands: torch.Tensor) -> torch.Tensor:
    assert all(t.device.type == "cpu" for t in operands)
    return _EINSUM(eq, *operands)


def softmax(x: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """Stock CPU softmax: the reference never patches softmax (cmpext3/__init__.py:133-138), so
    its einsum-attention chain always runs this op."""
    assert x.device.type == "cpu"
    return _SOFTMAX(x, dim=dim)


def einsum_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """The einsum-routed attention workload: scores einsum -> softmax (stock) -> values einsum."""
    s = einsum("bhid,bhjd->bhij", q, k)
    p = _SOFTMAX(s, dim=-1)
    return einsum("bhij,bhjd->bhid", p, v)


def sdpa_rows(q_rows: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rows, scale=None,
              is_causal: bool = False) -> torch.Tensor:
    """Stock CPU SDPA for a subset of query rows of one [L, D] slice.

    ``rows`` are the absolute query positions of ``q_rows``; the causal mask (key j visible to query
    i iff j <= i, top-left aligned) is passed explicitly because the row subset no longer starts at 0.
    Inputs are [n, D] / [Lk, D]; returns [n, D].
    """
    rows = torch.as_tensor(rows)
    mask = None
    if is_causal:
        mask = torch.arange(k.shape[0])[None, :] <= rows[:, None]
    out = _SDPA(q_rows[None, None], k[None, None], v[None, None], attn_mask=None if mask is None else mask[None, None],
                dropout_p=0.0, is_causal=False, scale=scale)
    return out[0, 0]
