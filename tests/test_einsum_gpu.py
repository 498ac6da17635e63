"""torch.einsum through the patched wrapper on the GPU (needs a B200; marked gpu).

The reference's planner test (tests/test_einsum.py:24-44 there) runs its equations on CUDA and
bounds the error relative to the output's peak at 1e-5 for fp32 and 5e-3 for fp16.  Here:
* the same equations and shapes, fp32 on the GPU, against the golden float64 outputs of the
  reference planner (tests/golden ``planner/*``).  These sizes are below the small-matmul
  threshold, so their pair products take the broadcast-multiply route as in the reference;
* the two-operand equations with every index scaled up past that threshold, so the planner's bmm
  calls reach the 3xTF32 GEMM (fp32) or the 16-bit GEMM (fp16), against float64 einsum on the CPU.
"""
from __future__ import annotations

import ast

import pytest
import torch

import cmpext3
from oracle import sdpa_np
from tests.golden import cases as C
from tests.golden import load

pytestmark = pytest.mark.gpu

G = load()
N = int(G["planner/count"])
CASES = [(str(G[f"planner/{i}/eq"]), ast.literal_eval(str(G[f"planner/{i}/shapes"]))) for i in range(N)]
INPUTS = C.planner_inputs(CASES)
BOUND = {torch.float32: 1e-5, torch.float16: 5e-3}


@pytest.mark.parametrize("i", range(N), ids=[c[0] for c in CASES])
def test_reference_equations_fp32(cuda_device, patched, i):
    eq, _ = CASES[i]
    ops = [t.float().to(cuda_device) for t in INPUTS[i]]
    with torch.no_grad():
        got = torch.einsum(eq, *ops)
    torch.cuda.synchronize()
    gold = G[f"planner/{i}/out"]
    assert tuple(got.shape) == gold.shape
    assert sdpa_np.rel_err(got.double().cpu().numpy(), gold) <= BOUND[torch.float32], eq


def _scaled(eq: str, shapes, factor: int):
    """The operands' shapes with every index size multiplied by `factor` (keeps the equation)."""
    lhs = eq.split("->")[0].split(",")
    size = {}
    for term, shape in zip(lhs, shapes):
        for ch, s in zip(term, shape):
            size[ch] = s * factor
    return [tuple(size[ch] for ch in term) for term in lhs]


PAIR_EQS = ["ij,jk->ik", "bij,bjk->bik", "ij,kj->ik", "ji,jk->ik", "ij,mjc->mic", "mij,mjc->mic",
            "bhqd,bhkd->bhqk", "bhqk,bhkd->bhqd"]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
@pytest.mark.parametrize("eq", PAIR_EQS)
def test_scaled_equations_reach_the_gemm(cuda_device, patched, eq, dtype):
    i = [c[0] for c in CASES].index(eq)
    factor = 4 if eq.startswith(("mij", "ij,mjc", "bh")) else 16
    shapes = _scaled(eq, CASES[i][1], factor)
    g = torch.Generator().manual_seed(i)
    ops = [torch.randn(*s, generator=g, dtype=torch.float64) for s in shapes]
    cmpext3.autoselect.reset()
    with torch.no_grad():
        got = torch.einsum(eq, *[t.to(dtype).to(cuda_device) for t in ops])
    torch.cuda.synchronize()
    want = torch.einsum(eq, *[t.to(dtype).double() for t in ops])
    assert sdpa_np.rel_err(got.double().cpu().numpy(), want.numpy()) <= BOUND[dtype], (eq, shapes)
    if dtype == torch.float32:
        entries = [d.entry for d in cmpext3.autoselect.report() if d.use_native]
        assert any("bmm_x3tf32" in (e or "") for e in entries), (eq, shapes, cmpext3.autoselect_report())
