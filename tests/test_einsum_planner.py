"""The einsum planner (cmpext3.einsum_ops) against the reference planner's own outputs and stock einsum.

Golden: tests/golden/reference_cpu_path.npz ``planner/*`` -- the reference's einsum_ops.einsum run in
float64 on the equations of its planner test (tests/test_einsum.py:24-44 there).  Tolerance 1e-12
relative to the peak, the reference's own CPU float64 bound (tests/test_einsum.py:68 there).
"""
from __future__ import annotations

import ast

import numpy as np
import pytest
import torch

from cmpext3 import einsum_ops
from oracle import sdpa_np
from tests.golden import load
from tests.golden import cases as C

G = load()
N = int(G["planner/count"])
CASES = [(str(G[f"planner/{i}/eq"]), ast.literal_eval(str(G[f"planner/{i}/shapes"]))) for i in range(N)]
INPUTS = C.planner_inputs(CASES)
STOCK = torch.einsum


@pytest.mark.parametrize("i", range(N), ids=[c[0] for c in CASES])
def test_planner_matches_reference_planner(i):
    eq, _ = CASES[i]
    got = einsum_ops.einsum(eq, INPUTS[i])
    gold = G[f"planner/{i}/out"]
    assert tuple(got.shape) == gold.shape
    assert sdpa_np.rel_err(got.numpy(), gold) <= 1e-12


@pytest.mark.parametrize("i", range(N), ids=[c[0] for c in CASES])
def test_planner_matches_stock_einsum(i):
    eq, _ = CASES[i]
    got = einsum_ops.einsum(eq, INPUTS[i])
    want = STOCK(eq, *INPUTS[i])
    assert sdpa_np.rel_err(got.numpy(), want.numpy()) <= 1e-12


@pytest.mark.parametrize("eq,shapes,reason", [
    ("ii->i", [(4, 4)], "repeated index in one operand"),
    ("...ij,...jk->...ik", [(2, 3, 4), (2, 4, 5)], "ellipsis"),
    ("ij,jk->iz", [(2, 3), (3, 4)], "bad output"),
    ("ij,jk->ik", [(2, 3)], "operand count"),
    ("ijk,jk->ik", [(2, 3), (3, 4)], "rank mismatch"),
    ("ij,jk->ik", [(2, 3), (4, 5)], "size mismatch"),
])
def test_unsupported_forms_report_a_reason(eq, shapes, reason):
    ops = [torch.randn(*s) for s in shapes]
    assert einsum_ops.supported(eq, ops) == reason


def test_bmm_receives_views_for_attention_scores():
    seen = []

    def spy(a, b):
        seen.append((a, b))
        return torch.bmm(a, b)

    q = torch.randn(2, 3, 16, 8)
    k = torch.randn(2, 3, 24, 8)
    out = einsum_ops.einsum("bhid,bhjd->bhij", [q, k], bmm=spy)
    (a, b), = seen
    assert a.data_ptr() == q.data_ptr() and b.data_ptr() == k.data_ptr()
    assert b.shape == (6, 8, 24) and b.stride(1) == 1
    assert torch.allclose(out, STOCK("bhid,bhjd->bhij", q, k), atol=1e-5)
