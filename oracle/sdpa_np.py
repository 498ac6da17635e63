"""Float64 numpy restatement of the hot-path math (TEST INFRASTRUCTURE ONLY -- see oracle/__init__.py).

* ``sdpa``: O = softmax(Q K^T * scale + M) V with M = -inf where key j > query i when causal
  (top-left aligned, as torch's is_causal builds ``tril(ones(Lq, Lk))``); scale defaults to
  1/sqrt(head_dim).  This is the computation every reference attention kernel implements
  (fp16_flash_attention_hfma2.cu:72-243, fp16_attention.cu:135-319, fp32_attention.cu:35-198),
  without their precision shortcuts.
* ``bmm``: C[b] = A[b] @ B[b] (reference custom_bmm_forward, src/main.cpp:363-441).
* ``sdpa_rows``: the same for a subset of query rows, for full-size spot checks.
"""
from __future__ import annotations

import math

import numpy as np


def _softmax_rows(s: np.ndarray) -> np.ndarray:
    m = np.max(s, axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    e = np.exp(s - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale=None, causal: bool = False) -> np.ndarray:
    """q [..., Lq, D], k [..., Lk, D], v [..., Lk, Dv] -> [..., Lq, Dv] in float64."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * scale
    if causal:
        lq, lk = q.shape[-2], k.shape[-2]
        mask = np.arange(lk)[None, :] > np.arange(lq)[:, None]
        s = np.where(mask, -np.inf, s)
    return np.matmul(_softmax_rows(s), v)


def sdpa_rows(q: np.ndarray, k: np.ndarray, v: np.ndarray, rows: np.ndarray, scale=None,
              causal: bool = False) -> np.ndarray:
    """SDPA for the query rows ``rows`` of a single [L, D] slice (rows attend to k/v as in sdpa)."""
    q = np.asarray(q, dtype=np.float64)[rows]
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    s = (q @ k.T) * scale
    if causal:
        mask = np.arange(k.shape[0])[None, :] > np.asarray(rows)[:, None]
        s = np.where(mask, -np.inf, s)
    return _softmax_rows(s) @ v


def bmm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return np.matmul(np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64))


def linear(x: np.ndarray, w: np.ndarray, b: np.ndarray | None = None) -> np.ndarray:
    """y = x W^T + b in float64 (the reference's custom_linear_forward, src/main.cpp:195-346, computes
    this product and then adds the bias row to every output row)."""
    y = np.matmul(np.asarray(x, dtype=np.float64), np.asarray(w, dtype=np.float64).T)
    return y if b is None else y + np.asarray(b, dtype=np.float64)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    x = np.moveaxis(x, axis, -1)
    return np.moveaxis(_softmax_rows(x), -1, axis)


def rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max |got - ref| / max |ref| -- the reference's correctness rule (autoselect.py:242-260)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if ref.size == 0:
        return 0.0
    scale = float(np.max(np.abs(ref)))
    diff = float(np.max(np.abs(got - ref)))
    return diff / scale if scale > 0 else diff


def max_abs(got: np.ndarray, ref: np.ndarray) -> float:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(got - ref))) if ref.size else 0.0


def cosine(got: np.ndarray, ref: np.ndarray) -> float:
    a = np.asarray(got, dtype=np.float64).ravel()
    b = np.asarray(ref, dtype=np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))
