"""The row-softmax kernel (cmpx_softmax_rows, the einsum-attention chain's middle step) against
the reference's CPU path -- stock torch.softmax on CPU tensors -- on a B200 (marked gpu).

Both kernel forms are covered: rows held in registers (16-byte aligned, up to 2048 16-bit / 1024
fp32 values) and the two-pass form (longer or unaligned rows).  Tolerances as in the parity tests:
fp16 max-abs 2e-3 and rel 1e-2, bf16 rel 1e-2, fp32 rel 1e-4 (max |got - ref| / max |ref|).
"""
from __future__ import annotations

import math

import pytest
import torch

import cmpext3
from cmpext3 import _native as N
from oracle import reference_path as RP
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1), (3, 7), (5, 8), (4, 77), (64, 2048), (2, 16, 64, 2048), (3, 1000), (6, 2056),
          (3, 4097), (2, 3, 257)]


def _x(shape, dtype, seed, scale=3.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32], ids=["f16", "bf16", "f32"])
@pytest.mark.parametrize("shape", SHAPES, ids=["x".join(map(str, s)) for s in SHAPES])
def test_softmax_matches_reference(cuda_device, dtype, shape):
    x = _x(shape, dtype, seed=sum(shape))
    got = N.softmax(x.to(cuda_device), -1)
    torch.cuda.synchronize()
    ref = RP.softmax(x, -1)
    check(got, ref, dtype, f"softmax {shape} {dtype}")
    assert got.dtype == dtype and got.shape == x.shape
    # rows sum to one (within output rounding)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert (got.float().sum(-1) - 1).abs().max().item() <= tol


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32], ids=["f16", "bf16", "f32"])
def test_softmax_masked_and_extreme_rows(cuda_device, dtype):
    x = _x((8, 2048), torch.float32, seed=5)
    x[0, 100:] = -math.inf            # masked tail
    x[1, ::2] = -math.inf             # every other key masked
    x[2, 0] = -math.inf               # first key masked (the two-pass form's first element)
    x[3] *= 40                        # large logits (fp16 would overflow exp without the max)
    x[4] = 0.0                        # uniform row
    x = x.to(dtype)
    for xx in (x, x[:, :2047]):       # registers form, and an unaligned row for the two-pass form
        got = N.softmax(xx.contiguous().to(cuda_device), -1)
        torch.cuda.synchronize()
        check(got, RP.softmax(xx.contiguous(), -1), dtype, f"extreme rows {xx.shape} {dtype}")


@pytest.mark.parametrize("cols", [1024, 1023], ids=["registers", "two-pass"])
def test_softmax_fp32_large_magnitude_rows(cuda_device, cols):
    """fp32 rows whose scores sit near +-1e3 with spreads of a few units: the exponent must come
    from the exact difference x - max (an fma with a separately rounded max * log2(e) would carry
    |max| * 2^-24 into every exponent), so the result stays within the fp32 1e-4 bound."""
    g = torch.Generator().manual_seed(17)
    x = torch.randn(6, cols, generator=g) * 3.0
    x[0] += 1000.0
    x[1] -= 1000.0
    x[2] += 3000.0
    x[3] = x[3] * 200.0 + 1500.0
    got = N.softmax(x.to(cuda_device), -1)
    torch.cuda.synchronize()
    ref = RP.softmax(x, -1)
    check(got, ref, torch.float32, f"large-magnitude fp32 rows ({cols})")
    rel = ((got.cpu() - ref).abs().amax(-1) / ref.abs().amax(-1)).max().item()
    assert rel <= 2e-5, rel


def test_fully_masked_row_is_nan_like_torch(cuda_device):
    x = torch.zeros(2, 512)
    x[1] = -math.inf
    got = N.softmax(x.to(cuda_device), -1).cpu()
    ref = RP.softmax(x, -1)
    assert torch.isnan(ref[1]).all() and torch.isnan(got[1]).all()
    assert torch.allclose(got[0], ref[0])


def test_noncontiguous_input_is_copied_then_computed(cuda_device):
    x = _x((64, 96), torch.bfloat16, seed=9).t()  # last dim strided
    got = N.softmax(x.to(cuda_device), -1)
    check(got, RP.softmax(x.contiguous(), -1), torch.bfloat16, "transposed")


def test_patched_einsum_chain_runs_the_native_softmax(cuda_device, patched):
    from cmpext3 import autoselect
    g = torch.Generator().manual_seed(21)
    q, k, v = (torch.randn(2, 4, 256, 64, generator=g).to(torch.bfloat16) for _ in range(3))
    qd, kd, vd = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    with torch.no_grad():
        s = torch.einsum("bhid,bhjd->bhij", qd, kd)
        o = torch.einsum("bhij,bhjd->bhid", torch.softmax(s, dim=-1), vd)
    torch.cuda.synchronize()
    check(o, RP.einsum_attention(q, k, v), torch.bfloat16, "einsum chain")
    report = autoselect.format_report()
    assert any(line.strip().startswith("cmpext3") and "softmax" in line
               for line in report.splitlines()), report
