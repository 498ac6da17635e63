"""The small-matrix batched product (cmpx_bmm_small, the route the reference's _small_bmm takes for
M*K*N <= 32768 per item, cmpext3/__init__.py:440-464) against the reference's CPU path -- stock
torch.bmm on CPU tensors -- on a B200 (marked gpu).

Shapes cover both kernel forms (thread per output element for K < 128, warp per element for
K >= 128), the FEM-style case the reference's comment names (20000 x 24x24 @ 24x3), K = 1, a single
long dot product (M = N = 1, K = 32768), strided and transposed operands read in place, a zero
batch and K = 0.  Tolerances as in the parity tests: fp32 rel 1e-4, fp16 / bf16 rel 1e-2.
"""
from __future__ import annotations

import pytest
import torch

import cmpext3
from cmpext3 import _native as N
from oracle import reference_path as RP
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.float16, torch.bfloat16]
IDS = ["f32", "f16", "bf16"]

SHAPES = [
    # (batch, M, K, N)
    (20000, 24, 24, 3),   # FEM element blocks
    (7, 5, 3, 2),
    (64, 32, 32, 32),     # M*K*N = 32768, the default threshold
    (3, 1, 32768, 1),     # one long dot product per item (warp form)
    (5, 16, 128, 16),     # warp form, M*N = 256
    (100, 8, 1, 8),       # K = 1
    (1, 1, 1, 1),
]


def _ab(shape, dtype, seed):
    bsz, m, k, n = shape
    g = torch.Generator().manual_seed(seed)
    return torch.randn(bsz, m, k, generator=g).to(dtype), torch.randn(bsz, k, n, generator=g).to(dtype)


@pytest.mark.parametrize("dtype", DTYPES, ids=IDS)
@pytest.mark.parametrize("shape", SHAPES, ids=["x".join(map(str, s)) for s in SHAPES])
def test_small_bmm_matches_reference(cuda_device, dtype, shape):
    a, b = _ab(shape, dtype, seed=sum(shape))
    plan = N.bmm_small_plan(a.to(cuda_device), b.to(cuda_device))
    assert plan.startswith("bmm_small<") and ("warp" in plan) == (shape[2] >= 128)
    got = N.bmm_small(a.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    check(got, RP.bmm(a, b), dtype, f"bmm_small {shape} {dtype}", attention=False)
    assert got.dtype == dtype and got.shape == (shape[0], shape[1], shape[3])
    assert N.device_status() == 0


@pytest.mark.parametrize("dtype", DTYPES, ids=IDS)
def test_small_bmm_reads_strided_and_transposed_views(cuda_device, dtype):
    g = torch.Generator().manual_seed(3)
    at = torch.randn(50, 12, 9, generator=g).to(dtype)         # a = at^T: column-major A
    b_wide = torch.randn(50, 12, 20, generator=g).to(dtype)    # b = every other column: strided B
    a, b = at.transpose(1, 2), b_wide[:, :, ::2]
    a_dev, b_dev = at.to(cuda_device).transpose(1, 2), b_wide.to(cuda_device)[:, :, ::2]
    assert a_dev.stride() == (108, 1, 9) and b_dev.stride() == (240, 20, 2)  # views, not copies
    got = N.bmm_small(a_dev, b_dev)
    torch.cuda.synchronize()
    check(got, RP.bmm(a.contiguous(), b.contiguous()), dtype, "strided views", attention=False)


def test_small_bmm_empty_and_zero_k(cuda_device):
    a = torch.randn(0, 3, 4, device=cuda_device)
    b = torch.randn(0, 4, 5, device=cuda_device)
    assert N.bmm_small(a, b).shape == (0, 3, 5)
    a = torch.randn(4, 3, 0, device=cuda_device)
    b = torch.randn(4, 0, 5, device=cuda_device)
    got = N.bmm_small(a, b)
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), torch.zeros(4, 3, 5))


@pytest.mark.parametrize("op", ["bmm", "matmul"])
def test_patched_ops_route_small_products_to_the_kernel(cuda_device, patched, op):
    a, b = _ab((20000, 24, 24, 3), torch.float32, seed=5)
    fn = torch.bmm if op == "bmm" else torch.matmul
    got = fn(a.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    check(got, RP.bmm(a, b), torch.float32, f"patched {op}", attention=False)
    report = cmpext3.autoselect_report()
    assert "bmm_small" in report and "bmm_small<f32,thread-per-element>" in report
