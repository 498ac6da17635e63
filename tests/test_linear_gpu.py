"""F.linear on the sm_100a GEMM (bias added in the epilogue) against the reference's CPU path --
the reference's patched F.linear routes CPU tensors to stock F.linear (needs a B200; marked gpu).
Golden vectors from the reference package, then sweeps: 2-D and 3-D inputs, with and without
bias, ragged m / n / k, strided inputs, the projection shapes of the configs' models, nn.Linear
through the patched F.linear.  Tolerances as in test_parity_gpu.py (relative to the output's peak)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import cmpext3
from cmpext3 import _native as N
from oracle import reference_path as RP
from tests.golden import cases as C
from tests.golden import load
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("i", range(len(C.LINEAR_CASES)), ids=[c[0] for c in C.LINEAR_CASES])
def test_linear_matches_reference_golden(cuda_device, i):
    name, dtn, shape, n, has_bias = C.LINEAR_CASES[i]
    x, w, b = C.linear_inputs(i)
    gold = load()[f"linear/{name}/y"]
    got = cmpext3.ops.linear(x.to(cuda_device), w.to(cuda_device), None if b is None else b.to(cuda_device))
    torch.cuda.synchronize()
    assert got.shape == x.shape[:-1] + (n,) and got.dtype == x.dtype
    check(got, gold, x.dtype, name, attention=False)


SHAPES = [
    # (input shape, out_features)
    ((1, 8), 8),                  # one row, one k block
    ((3, 77, 768), 320),          # SD1.5 cross-attention K/V projection of the text states
    ((2, 4096, 320), 1280),       # SD1.5 feed-forward up-projection (GEGLU in)
    ((2, 1024, 640), 640),        # SD1.5 attention output projection, level 2
    ((1, 1000, 1024), 2056),      # ragged m and n
    ((4, 64, 1000), 512),         # ragged k
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32], ids=["bf16", "f16", "f32"])
@pytest.mark.parametrize("bias", [False, True], ids=["nobias", "bias"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{'x'.join(map(str, s[0]))}->{s[1]}" for s in SHAPES])
def test_linear_sweep(cuda_device, dtype, bias, shape):
    in_shape, n = shape
    k = in_shape[-1]
    g = torch.Generator().manual_seed(sum(in_shape) * 31 + n)
    x = torch.randn(*in_shape, generator=g).to(dtype)
    w = (torch.randn(n, k, generator=g) / k ** 0.5).to(dtype)
    b = torch.randn(n, generator=g).to(dtype) if bias else None
    got = cmpext3.ops.linear(x.to(cuda_device), w.to(cuda_device), None if b is None else b.to(cuda_device))
    torch.cuda.synchronize()
    check(got, RP.linear(x, w, b), dtype, f"linear {shape} bias={bias}", attention=False)
    assert N.device_status() == 0


def test_linear_strided_input_rows(cuda_device):
    # x is every other row of a wider buffer (row stride 2k): read in place through the TMA map
    g = torch.Generator().manual_seed(5)
    buf = torch.randn(300, 2 * 256, generator=g).to(torch.bfloat16)
    x = buf[:, :256]
    w = (torch.randn(384, 256, generator=g) / 16).to(torch.bfloat16)
    b = torch.randn(384, generator=g).to(torch.bfloat16)
    got = cmpext3.ops.linear(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    check(got, RP.linear(x, w, b), torch.bfloat16, "strided rows", attention=False)


def test_bias_is_added_once_in_fp32(cuda_device):
    # with x = 0 the output is exactly the bias (one rounding of an already 16-bit value)
    x = torch.zeros(130, 512, dtype=torch.float16, device=cuda_device)
    w = torch.randn(264, 512, dtype=torch.float16, device=cuda_device)
    b = torch.randn(264, dtype=torch.float16, device=cuda_device)
    got = cmpext3.ops.linear(x, w, b)
    torch.cuda.synchronize()
    assert torch.equal(got, b.expand(130, 264))


def test_nn_linear_through_the_patched_f_linear(cuda_device, patched):
    torch.manual_seed(0)
    layer = torch.nn.Linear(640, 1280).to(device=cuda_device, dtype=torch.bfloat16)
    x = torch.randn(2, 1024, 640, device=cuda_device, dtype=torch.bfloat16)
    with torch.no_grad():
        got = layer(x)
    torch.cuda.synchronize()
    ref = RP.linear(x.cpu(), layer.weight.detach().cpu(), layer.bias.detach().cpu())
    check(got, ref, torch.bfloat16, "nn.Linear", attention=False)
    entries = [d.entry for d in cmpext3.autoselect.report() if d.use_native]
    assert any("bmm_sm100" in (e or "") for e in entries), cmpext3.autoselect_report()
