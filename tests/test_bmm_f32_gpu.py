"""fp32 bmm / matmul / einsum / linear on the 3xTF32 tensor-core GEMM (needs a B200; marked gpu).

The reference runs fp32 bmm on its CUDA-core GEMM (gemm_fp32_ga100_kernel,
src/cuda/fp32_matmul.cu:31-184) and checks fp32 results at 1e-5 relative to the peak
(tests/test_einsum.py:24-44).  Every case here is checked against the reference's CPU path (stock
torch on CPU tensors) within the fp32 contract (1e-4 of the peak, `check`), and against a float64
product within 5e-5 of the peak.  A single TF32 product (10-bit mantissa) lands near 2e-4 of the
peak on these sizes, so this bound shows the hi / lo split at work; what remains at long K is the
tensor core's fp32 accumulation (3e-5 at K = 4097).  Layouts: row-major, transposed views (copied to a
K-major buffer by the binding), ragged m / n / k (rows padded to 16 bytes), batch items of one row
or column.  Special values: a NaN operand makes NaN outputs."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import cmpext3
from cmpext3 import _native as N
from oracle import reference_path as RP
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu

X3 = "bmm_x3tf32_sm100"


def _rel64(got: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> float:
    ref = torch.bmm(a.double(), b.double())
    return ((got.double().cpu() - ref).abs().max() / ref.abs().max().clamp_min(1e-300)).item()


SHAPES = [(1, 1, 1, 1), (3, 1, 64, 1), (2, 64, 32, 64), (4, 130, 72, 200), (2, 257, 129, 300),
          (1, 1000, 64, 136), (2, 333, 257, 129), (1, 128, 4097, 128), (5, 17, 3, 5),
          (64, 128, 64, 128)]


@pytest.mark.parametrize("a_t", [False, True], ids=["A_rowmajor", "A_transposed"])
@pytest.mark.parametrize("b_t", [False, True], ids=["B_rowmajor", "B_transposed"])
@pytest.mark.parametrize("shape", SHAPES, ids=["x".join(map(str, s)) for s in SHAPES])
def test_fp32_bmm_sweep(cuda_device, shape, a_t, b_t):
    nb, m, k, n = shape
    g = torch.Generator().manual_seed(nb * 7919 + m * 31 + k * 7 + n)
    a = torch.randn(nb, k, m, generator=g).transpose(1, 2) if a_t else torch.randn(nb, m, k, generator=g)
    b = torch.randn(nb, n, k, generator=g).transpose(1, 2) if b_t else torch.randn(nb, k, n, generator=g)
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    assert N.bmm_plan(ad, bd).startswith(X3)
    got = cmpext3.ops.bmm(ad, bd)
    torch.cuda.synchronize()
    assert got.shape == (nb, m, n) and got.dtype == torch.float32 and got.is_contiguous()
    check(got, RP.bmm(a, b), torch.float32, f"fp32 bmm {shape}", attention=False)
    assert _rel64(got, a, b) <= 5e-5, shape
    assert N.device_status() == 0


def test_fp32_bmm_large_k_accuracy(cuda_device):
    # K = 8192: 256 K blocks accumulated in the tensor core's fp32
    g = torch.Generator().manual_seed(3)
    a = torch.randn(2, 256, 8192, generator=g)
    b = torch.randn(2, 8192, 384, generator=g)
    got = cmpext3.ops.bmm(a.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    assert _rel64(got, a, b) <= 5e-5


@pytest.mark.parametrize("k", [8200, 16384, 40000])
def test_fp32_bmm_long_k_runs_in_chunks(cuda_device, patched, k):
    # K > 8192: the product runs over K chunks of at most 8192, each accumulated in the tensor
    # core's fp32 and added into C in fp32, so the error stays that of one chunk (the fp32 contract
    # 1e-4, measured against float64); the patched torch.bmm takes the same kernel
    g = torch.Generator().manual_seed(9)
    a, b = torch.randn(2, 96, k, generator=g), torch.randn(2, k, 80, generator=g)
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    assert cmpext3.ops.bmm_plan(ad, bd).endswith("+k-chunks>")
    got = cmpext3.ops.bmm(ad, bd)
    torch.cuda.synchronize()
    assert _rel64(got, a, b) <= 5e-5
    with torch.no_grad():
        got2 = torch.bmm(ad, bd)
    torch.cuda.synchronize()
    check(got2, RP.bmm(a, b), torch.float32, f"K {k}", attention=False)
    assert "k-chunks" in cmpext3.autoselect_report()


def test_fp32_bmm_inf_operand(cuda_device):
    # An inf operand: its row of C is +-inf or NaN (the 3xTF32 cross terms multiply the inf by
    # exactly-zero remainders), never finite; the other rows are unaffected.
    a = torch.randn(1, 32, 64)
    b = torch.randn(1, 64, 32)
    a[0, 5, 7] = float("inf")
    got = cmpext3.ops.bmm(a.to(cuda_device), b.to(cuda_device)).cpu()
    assert not torch.isfinite(got[0, 5]).any()
    rows = [r for r in range(32) if r != 5]
    check(got[:, rows], RP.bmm(a[:, rows], b), torch.float32, "rows without inf", attention=False)


def test_fp32_bmm_strided_operands_in_place(cuda_device):
    # every other row of a wider buffer: K-major with a 16-byte-multiple row stride -> no copy
    g = torch.Generator().manual_seed(4)
    buf = torch.randn(3, 200, 256, generator=g).to(cuda_device)
    a = buf[:, :, :128]
    bt = torch.randn(3, 96, 128, generator=g).to(cuda_device)
    got = cmpext3.ops.bmm(a, bt.transpose(1, 2))
    torch.cuda.synchronize()
    check(got, RP.bmm(a.cpu(), bt.transpose(1, 2).cpu()), torch.float32, "strided", attention=False)


def test_fp32_bmm_nan_propagates(cuda_device):
    g = torch.Generator().manual_seed(5)
    a = torch.randn(1, 64, 64, generator=g)
    b = torch.randn(1, 64, 64, generator=g)
    a[0, 3, 10] = float("nan")
    # a NaN whose payload is only in the mantissa bits TF32 drops: still a NaN
    a[0, 7, 20] = torch.tensor([0x7F800001], dtype=torch.int32).view(torch.float32)[0]
    got = cmpext3.ops.bmm(a.to(cuda_device), b.to(cuda_device)).cpu()
    assert torch.isnan(got[0, 3]).all() and torch.isnan(got[0, 7]).all()
    rows = [r for r in range(64) if r not in (3, 7)]
    check(got[:, rows], RP.bmm(a[:, rows], b), torch.float32, "rows without NaN", attention=False)


def test_fp32_einsum_attention_chain_runs_native(cuda_device, patched):
    g = torch.Generator().manual_seed(6)
    q, k, v = (torch.randn(2, 4, 256, 64, generator=g) for _ in range(3))
    qd, kd, vd = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    cmpext3.autoselect.reset()
    with torch.no_grad():
        s = torch.einsum("bhid,bhjd->bhij", qd, kd)
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("bhij,bhjd->bhid", p, vd)
    torch.cuda.synchronize()
    s_ref = torch.einsum("bhid,bhjd->bhij", q, k)
    o_ref = torch.einsum("bhij,bhjd->bhid", torch.softmax(s_ref, dim=-1), v)
    check(s, s_ref, torch.float32, "fp32 scores", attention=False)
    check(o, o_ref, torch.float32, "fp32 values", attention=False)
    entries = [d.entry for d in cmpext3.autoselect.report() if d.use_native]
    assert sum(X3 in (e or "") for e in entries) >= 2, cmpext3.autoselect_report()


def test_fp32_matmul_2d_runs_native(cuda_device, patched):
    g = torch.Generator().manual_seed(7)
    a, b = torch.randn(300, 520, generator=g), torch.randn(520, 260, generator=g)
    cmpext3.autoselect.reset()
    with torch.no_grad():
        got = torch.matmul(a.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    check(got, a @ b, torch.float32, "fp32 matmul", attention=False)
    entries = [d.entry for d in cmpext3.autoselect.report() if d.use_native]
    assert any(X3 in (e or "") for e in entries), cmpext3.autoselect_report()


@pytest.mark.parametrize("shape", [((3, 77, 768), 320), ((1, 1000, 1024), 2056), ((4, 64, 1001), 510)],
                         ids=["sd15-text-kv", "ragged-mn", "ragged-k-odd-n"])
@pytest.mark.parametrize("bias", [False, True], ids=["nobias", "bias"])
def test_fp32_linear(cuda_device, shape, bias):
    in_shape, n = shape
    k = in_shape[-1]
    g = torch.Generator().manual_seed(k + n)
    x = torch.randn(*in_shape, generator=g)
    w = torch.randn(n, k, generator=g) / k ** 0.5
    b = torch.randn(n, generator=g) if bias else None
    xd, wd, bd = x.to(cuda_device), w.to(cuda_device), None if b is None else b.to(cuda_device)
    assert N.linear_plan(xd, wd, bd).startswith(X3)
    got = cmpext3.ops.linear(xd, wd, bd)
    torch.cuda.synchronize()
    assert got.shape == x.shape[:-1] + (n,) and got.is_contiguous()
    check(got, RP.linear(x, w, b), torch.float32, f"fp32 linear {shape}", attention=False)


def test_fp32_nn_linear_through_the_patched_f_linear(cuda_device, patched):
    torch.manual_seed(0)
    layer = torch.nn.Linear(640, 1280).to(cuda_device)
    x = torch.randn(2, 1024, 640, device=cuda_device)
    cmpext3.autoselect.reset()
    with torch.no_grad():
        got = layer(x)
    torch.cuda.synchronize()
    ref = RP.linear(x.cpu(), layer.weight.detach().cpu(), layer.bias.detach().cpu())
    check(got, ref, torch.float32, "fp32 nn.Linear", attention=False)
    entries = [d.entry for d in cmpext3.autoselect.report() if d.use_native]
    assert any(X3 in (e or "") for e in entries), cmpext3.autoselect_report()


def test_fp32_bmm_in_a_graph(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(8)
    a = torch.randn(4, 200, 96, device=cuda_device, generator=g)
    b = torch.randn(4, 96, 136, device=cuda_device, generator=g)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        cmpext3.ops.bmm(a, b)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = cmpext3.ops.bmm(a, b)
    for trial in range(2):
        a.copy_(torch.randn(a.shape, device=cuda_device, generator=g))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, cmpext3.ops.bmm(a, b)), trial
    del graph
