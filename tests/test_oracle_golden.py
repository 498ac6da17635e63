"""Pins the oracle against golden vectors made by the reference package itself (CPU, no GPU).

tests/golden/reference_cpu_path.npz holds the outputs of the reference's patched
F.scaled_dot_product_attention / torch.bmm / F.linear / torch.einsum on seeded CPU tensors (which the
reference routes to stock PyTorch); tests/golden/make_golden.py made it.  Both oracles must
reproduce them: ``oracle.reference_path`` (the same stock calls) bit-for-bit, and the float64
numpy restatement ``oracle.sdpa_np`` within the rounding of the output dtype.
"""
from __future__ import annotations

import ast

import numpy as np
import pytest
import torch

from oracle import reference_path as RP
from oracle import sdpa_np
from tests.golden import load
from tests.golden import cases as C

G = load()


def _as_float(x) -> np.ndarray:
    return x.float().numpy() if isinstance(x, torch.Tensor) else np.asarray(x, dtype=np.float32)


def _golden(key):
    x = G[key]
    return x.float().numpy() if isinstance(x, torch.Tensor) else x


# Output rounding of each dtype relative to the output's peak (plus accumulation differences).
_NP_TOL = {"float32": 2e-6, "float16": 2e-3, "bfloat16": 1e-2}


@pytest.mark.parametrize("i", range(len(C.SDPA_CASES)), ids=[c[0] for c in C.SDPA_CASES])
def test_sdpa_inputs_match_golden_digests(i):
    name = C.SDPA_CASES[i][0]
    q, k, v = C.sdpa_inputs(i)
    for key, t in (("q", q), ("k", k), ("v", v)):
        assert C.digest(t) == str(G[f"sdpa/{name}/{key}_sha256"]), f"{name}/{key} generator drifted"


@pytest.mark.parametrize("i", range(len(C.SDPA_CASES)), ids=[c[0] for c in C.SDPA_CASES])
def test_reference_path_reproduces_golden_sdpa(i):
    name, dtn, B, H, Lq, Lk, D, causal, scale, _ = C.SDPA_CASES[i]
    q, k, v = C.sdpa_inputs(i)
    with torch.no_grad():
        o = RP.sdpa(q, k, v, scale=scale, is_causal=causal)
    assert np.array_equal(C.to_numpy(o), G[f"sdpa/{name}/o"] if not isinstance(G[f"sdpa/{name}/o"], torch.Tensor)
                          else C.to_numpy(G[f"sdpa/{name}/o"]))


@pytest.mark.parametrize("i", range(len(C.SDPA_CASES)), ids=[c[0] for c in C.SDPA_CASES])
def test_numpy_restatement_matches_golden_sdpa(i):
    name, dtn, B, H, Lq, Lk, D, causal, scale, _ = C.SDPA_CASES[i]
    q, k, v = C.sdpa_inputs(i)
    ref = sdpa_np.sdpa(q.float().numpy(), k.float().numpy(), v.float().numpy(), scale=scale, causal=causal)
    gold = _golden(f"sdpa/{name}/o").astype(np.float64)
    assert sdpa_np.rel_err(ref, gold) <= _NP_TOL[dtn], name


@pytest.mark.parametrize("i", range(len(C.LINEAR_CASES)), ids=[c[0] for c in C.LINEAR_CASES])
def test_linear_oracles_match_golden(i):
    name, dtn, shape, n, has_bias = C.LINEAR_CASES[i]
    x, w, b = C.linear_inputs(i)
    for key, t in (("x", x), ("w", w)) + ((("b", b),) if b is not None else ()):
        assert C.digest(t) == str(G[f"linear/{name}/{key}_sha256"]), f"{name}/{key} generator drifted"
    gold = G[f"linear/{name}/y"]
    got = RP.linear(x, w, b)
    assert np.array_equal(C.to_numpy(got), gold if not isinstance(gold, torch.Tensor) else C.to_numpy(gold))
    ref = sdpa_np.linear(x.float().numpy(), w.float().numpy(), None if b is None else b.float().numpy())
    assert sdpa_np.rel_err(ref, _golden(f"linear/{name}/y")) <= _NP_TOL[dtn], name


@pytest.mark.parametrize("i", range(len(C.BMM_CASES)), ids=[c[0] for c in C.BMM_CASES])
def test_bmm_oracles_match_golden(i):
    name, dtn = C.BMM_CASES[i][:2]
    a, b = C.bmm_inputs(i)
    assert C.digest(a) == str(G[f"bmm/{name}/a_sha256"])
    assert C.digest(b) == str(G[f"bmm/{name}/b_sha256"])
    gold = G[f"bmm/{name}/c"]
    got = RP.bmm(a, b)
    assert np.array_equal(C.to_numpy(got), gold if not isinstance(gold, torch.Tensor) else C.to_numpy(gold))
    ref = sdpa_np.bmm(a.float().numpy(), b.float().numpy())
    assert sdpa_np.rel_err(ref, _golden(f"bmm/{name}/c")) <= _NP_TOL[dtn]


def test_einsum_attention_oracles_match_golden():
    q, k, v = C.einsum_attn_inputs()
    for key, t in (("q", q), ("k", k), ("v", v)):
        assert C.digest(t) == str(G[f"einsum_attn/{key}_sha256"])
    o = RP.einsum_attention(q, k, v)
    assert torch.equal(o, G["einsum_attn/o"])
    s = sdpa_np.bmm(q.float().numpy(), np.swapaxes(k.float().numpy(), -1, -2))
    assert sdpa_np.rel_err(s, _golden("einsum_attn/s")) <= 1e-2
    # The stock chain rounds the unscaled scores (|s| up to ~30, bf16 step 0.125 there) and the
    # probabilities to bf16, so against the float64 restatement it sits within the reference's own
    # bf16 rule (autoselect.py:93-97 there: 5e-2 of the peak), not within a single bf16 rounding.
    o_np = sdpa_np.sdpa(q.float().numpy(), k.float().numpy(), v.float().numpy(), scale=1.0)
    assert sdpa_np.rel_err(o_np, _golden("einsum_attn/o")) <= 5e-2


def test_sdpa_rows_restatement_equals_full():
    q, k, v = C.sdpa_inputs(7)  # bf16 causal
    full = sdpa_np.sdpa(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=True)[0, 0]
    rows = np.array([0, 5, 127, 128, 299])
    part = sdpa_np.sdpa_rows(q[0, 0].float().numpy(), k[0, 0].float().numpy(), v[0, 0].float().numpy(),
                             rows, causal=True)
    assert np.allclose(part, full[rows], rtol=0, atol=1e-12)


def test_planted_mistake_in_oracle_is_caught():
    """A deliberately wrong oracle (non-causal where causal is asked) must fail the golden check."""
    name, dtn, B, H, Lq, Lk, D, causal, scale, _ = C.SDPA_CASES[7]
    q, k, v = C.sdpa_inputs(7)
    wrong = sdpa_np.sdpa(q.float().numpy(), k.float().numpy(), v.float().numpy(), causal=False)
    assert sdpa_np.rel_err(wrong, _golden(f"sdpa/{name}/o")) > 0.1
