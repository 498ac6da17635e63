"""The 128x256-tile batched matmul (wide N, K >= 512) against the reference's CPU path -- stock torch
bmm on CPU tensors (needs a B200; marked gpu).  Every operand layout the kernel reads in place, ragged
M / N / K edges, and launches with several tiles per persistent CTA (the single staging slot of each
epilogue warp reused chunk after chunk, tile after tile).  Tolerances as in test_parity_gpu.py."""
from __future__ import annotations

import pytest
import torch

import cmpext3
from cmpext3 import _native as N
from oracle import reference_path as RP
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu

SHAPES = [
    # (batch, m, k, n)
    (1, 300, 600, 520),     # ragged m, k and n edges; one partial n tile
    (2, 256, 1024, 512),
    (3, 130, 768, 1000),
    (8, 1024, 512, 2048),   # 512 tiles: several per CTA
]


def _operand(g, rows, cols, dtype, mn_major, batch):
    """[batch, rows, cols] with the requested contiguous dimension (a transposed view for MN-major)."""
    if mn_major:
        return torch.randn(batch, cols, rows, generator=g).to(dtype).transpose(1, 2)
    return torch.randn(batch, rows, cols, generator=g).to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{s[0]}x{s[1]}x{s[2]}x{s[3]}" for s in SHAPES])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)],
                         ids=["A_k-B_n", "A_k-B_k", "A_m-B_n", "A_m-B_k"])
def test_wide_bmm_matches_reference(cuda_device, dtype, shape, a_t, b_t):
    nb, m, k, n = shape
    g = torch.Generator().manual_seed(nb * 7 + m + 3 * k + 5 * n)
    a = _operand(g, m, k, dtype, a_t, nb)       # A: [nb, m, k]; a_t -> M contiguous
    # B: [nb, k, n]; b_t -> K contiguous (the layout of a linear layer's weight viewed as W^T)
    b = (torch.randn(nb, n, k, generator=g).to(dtype).transpose(1, 2) if b_t
         else torch.randn(nb, k, n, generator=g).to(dtype))
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    plan = N.bmm_plan(ad, bd)
    assert "128x256" in plan, plan
    got = cmpext3.ops.bmm(ad, bd)
    torch.cuda.synchronize()
    check(got, RP.bmm(a, b), dtype, f"wide bmm {shape} A^T={a_t} B^T={b_t}", attention=False)
    assert N.device_status() == 0


def test_short_k_keeps_the_128_wide_tile(cuda_device):
    # the attention-score shape (K = 64) is an output-write stream: it keeps the 128x128 tile
    a = torch.randn(4, 256, 64, dtype=torch.bfloat16, device=cuda_device)
    b = torch.randn(4, 64, 512, dtype=torch.bfloat16, device=cuda_device)
    assert "128x128" in N.bmm_plan(a, b)
