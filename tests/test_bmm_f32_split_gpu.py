"""fp32 bmm / linear with split operands (needs a B200; marked gpu).

For products large enough to pay (m n / (m + n) >= 512 per batch item, k >= 512) the binding passes a
workspace to cmpx_bmm_ws / cmpx_linear_ws: a pass writes the low TF32 parts of A and B once per call
and the GEMM loads them beside the operands.  Checked here: the result bit for bit against the same
product without a workspace (the converter path, which splits every shared-memory tile), against
the reference's CPU path within the fp32 contract and against float64; operands with inf, NaN and a
NaN whose payload sits only in the bits TF32 drops (the pass flags it and the GEMM falls back to the
converter path, which rewrites it); K chunks; and the workspace's first 256 bytes left as they were.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import cmpext3
from cmpext3 import _native as N
from oracle import reference_path as RP
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu


def _no_workspace(a, b):
    """The same product through cmpx_bmm (no workspace): the converter path."""
    a2, b2, c = N._prepare_bmm(a, b)
    desc = N._bmm_desc(a2, b2, c)
    st = N.lib.cmpx_bmm(ctypes.byref(desc), N._stream_handle(a.device))
    assert st == 0, N.lib.cmpx_status_str(st)
    return c


def _ws_size(a, b):
    a2, b2, c = N._prepare_bmm(a, b)
    return N.lib.cmpx_bmm_workspace_size(ctypes.byref(N._bmm_desc(a2, b2, c)))


def _rel64(got, a, b):
    ref = torch.bmm(a.double().cpu(), b.double().cpu())
    return ((got.double().cpu() - ref).abs().max() / ref.abs().max()).item()


# (nb, m, k, n, B transposed)
SHAPES = [(1, 1024, 512, 1024, True), (2, 1536, 520, 1100, False), (1, 1024, 9000, 1024, True),
          (3, 768, 600, 2000, True), (1, 2048, 516, 2048, False)]


@pytest.mark.parametrize("shape", SHAPES, ids=["x".join(map(str, s[:4])) + ("t" if s[4] else "") for s in SHAPES])
def test_split_operands_match_the_converter_path(cuda_device, shape):
    nb, m, k, n, bt = shape
    g = torch.Generator().manual_seed(m + k + n)
    a = torch.randn(nb, m, k, generator=g)
    b = torch.randn(nb, n, k, generator=g).transpose(1, 2) if bt else torch.randn(nb, k, n, generator=g)
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    assert _ws_size(ad, bd) > 0
    got = cmpext3.ops.bmm(ad, bd)
    plain = _no_workspace(ad, bd)
    torch.cuda.synchronize()
    assert torch.equal(got, plain)
    check(got, RP.bmm(a, b), torch.float32, f"split fp32 bmm {shape}", attention=False)
    assert _rel64(got, a, b) <= 5e-5
    assert N.device_status() == 0


@pytest.mark.parametrize("where", ["A", "B"])
def test_special_values_with_split_operands(cuda_device, where):
    g = torch.Generator().manual_seed(11)
    a = torch.randn(1, 1024, 512, generator=g)
    b = torch.randn(1, 512, 1024, generator=g)
    low_nan = torch.tensor([0x7F800001], dtype=torch.int32).view(torch.float32)[0]
    if where == "A":
        a[0, 3, 10] = float("inf")
        a[0, 5, 11] = float("nan")
        a[0, 7, 20] = low_nan  # read as inf through TF32: the GEMM must fall back and rewrite it
    else:
        b[0, 10, 3] = float("inf")
        b[0, 11, 5] = float("nan")
        b[0, 20, 7] = low_nan
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    got = cmpext3.ops.bmm(ad, bd)
    plain = _no_workspace(ad, bd)
    torch.cuda.synchronize()
    assert torch.equal(got.isnan(), plain.isnan())
    assert torch.equal(torch.nan_to_num(got), torch.nan_to_num(plain))
    nan_line = got[0, 7] if where == "A" else got[0, :, 7]
    assert torch.isnan(nan_line).all()
    # without the low-payload NaN the split path runs, with the same results
    if where == "A":
        a[0, 7, 20] = 0.0
    else:
        b[0, 20, 7] = 0.0
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    got = cmpext3.ops.bmm(ad, bd)
    plain = _no_workspace(ad, bd)
    torch.cuda.synchronize()
    assert torch.equal(torch.nan_to_num(got), torch.nan_to_num(plain))
    assert torch.equal(got.isnan(), plain.isnan()) and torch.equal(got.isinf(), plain.isinf())


def test_split_leaves_the_first_256_workspace_bytes_alone(cuda_device):
    g = torch.Generator().manual_seed(12)
    a = torch.randn(1, 1024, 512, generator=g).to(cuda_device)
    b = torch.randn(1, 512, 1024, generator=g).to(cuda_device)
    a2, b2, c = N._prepare_bmm(a, b)
    desc = N._bmm_desc(a2, b2, c)
    need = N.lib.cmpx_bmm_workspace_size(ctypes.byref(desc))
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda_device)
    ws[:256] = torch.arange(256, dtype=torch.uint8, device=cuda_device)
    st = N.lib.cmpx_bmm_ws(ctypes.byref(desc), ws.data_ptr(), ws.numel(), N._stream_handle(a.device))
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(ws[:256].cpu(), torch.arange(256, dtype=torch.uint8))
    assert torch.equal(c, _no_workspace(a, b))
    # a workspace one byte short runs the converter path: same result
    c2 = torch.empty_like(c)
    desc2 = N._bmm_desc(a2, b2, c2)
    st = N.lib.cmpx_bmm_ws(ctypes.byref(desc2), ws.data_ptr(), need - 1, N._stream_handle(a.device))
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(c2, c)


@pytest.mark.parametrize("bias", [True, False], ids=["bias", "nobias"])
def test_fp32_linear_split_operands(cuda_device, bias):
    g = torch.Generator().manual_seed(13)
    x = torch.randn(2048, 1024, generator=g)
    w = torch.randn(1536, 1024, generator=g)
    bb = torch.randn(1536, generator=g) if bias else None
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    bd = bb.to(cuda_device) if bias else None
    x2, w2, b2, y = N._prepare_linear(xd, wd, bd)
    desc = N._linear_desc(x2, w2, b2, y)
    assert N.lib.cmpx_linear_workspace_size(ctypes.byref(desc)) > 0
    got = cmpext3.ops.linear(xd, wd, bd)
    st = N.lib.cmpx_linear(ctypes.byref(desc), N._stream_handle(xd.device))  # no workspace, into y
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(got, y)
    ref = torch.nn.functional.linear(x.double(), w.double(), bb.double() if bias else None)
    assert ((got.double().cpu() - ref).abs().max() / ref.abs().max()).item() <= 5e-5


def test_released_workspaces_are_allocated_again(cuda_device):
    a = torch.randn(1, 1024, 512, device=cuda_device)
    b = torch.randn(1, 512, 1024, device=cuda_device)
    first = cmpext3.ops.bmm(a, b)
    N.release_workspaces()
    assert not N._WORKSPACES
    again = cmpext3.ops.bmm(a, b)
    torch.cuda.synchronize()
    assert torch.equal(first, again) and N._WORKSPACES


def test_split_operands_in_a_graph(cuda_device):
    # the pass, the flag's memset and the GEMM are all captured; the workspace of the capture
    # stream is allocated by the warm-up call on that stream, before the capture
    g = torch.Generator(device=cuda_device).manual_seed(14)
    a = torch.randn(2, 1024, 512, device=cuda_device, generator=g)
    b = torch.randn(2, 512, 1024, device=cuda_device, generator=g)
    assert _ws_size(a, b) > 0
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        cmpext3.ops.bmm(a, b)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        out = cmpext3.ops.bmm(a, b)
    for trial in range(2):
        a.copy_(torch.randn(a.shape, device=cuda_device, generator=g))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, _no_workspace(a, b)), trial
    del graph


def test_mn_major_b_through_the_workspace(cuda_device):
    # a row-major [k, n] B goes to cmpx_bmm_ws as it is: the pass transposes it into the workspace
    g = torch.Generator().manual_seed(15)
    a = torch.randn(2, 1024, 1000, generator=g).to(cuda_device)
    b = torch.randn(2, 1000, 1028, generator=g).to(cuda_device)
    a2, b2, c = N._prepare_bmm(a, b, keep_mn_b=True)
    assert b2.data_ptr() == b.data_ptr() and b2.stride(2) == 1  # not copied
    desc = N._bmm_desc(a2, b2, c)
    need = N.lib.cmpx_bmm_workspace_size(ctypes.byref(desc))
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device=cuda_device)
    st = N.lib.cmpx_bmm_ws(ctypes.byref(desc), ws.data_ptr(), ws.numel(), N._stream_handle(a.device))
    assert st == 0, N.lib.cmpx_status_str(st)
    plain = _no_workspace(a, b)
    torch.cuda.synchronize()
    assert torch.equal(c, plain)
    assert torch.equal(cmpext3.ops.bmm(a, b), plain)
    # a low-payload NaN in B: the flag sends the GEMM to the converter path over the copy of B
    b[1, 7, 3] = torch.tensor([0x7F800001], dtype=torch.int32, device=cuda_device).view(torch.float32)[0]
    got = cmpext3.ops.bmm(a, b)
    plain = _no_workspace(a, b)
    torch.cuda.synchronize()
    assert torch.isnan(got[1, :, 3]).all()
    assert torch.equal(torch.nan_to_num(got), torch.nan_to_num(plain))


def test_mn_major_b_with_k_chunks(cuda_device):
    # K > 8192 runs as K chunks; B row-major goes through the transposing pass, every chunk reading
    # its slice of the workspace copy
    g = torch.Generator().manual_seed(16)
    a = torch.randn(1, 1024, 8200, generator=g)
    b = torch.randn(1, 8200, 1024, generator=g)
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    assert N.bmm_plan(ad, bd).endswith("+k-chunks>")
    got = cmpext3.ops.bmm(ad, bd)
    plain = _no_workspace(ad, bd)
    torch.cuda.synchronize()
    assert torch.equal(got, plain)
    check(got, RP.bmm(a, b), torch.float32, "split fp32 bmm, row-major B, K chunks", attention=False)


def test_patched_fp32_matmul_and_linear_take_the_split_schedule(cuda_device, patched):
    # torch.matmul of two row-major fp32 matrices (a row-major B: the transposing pass) and
    # nn.Linear (the weight read as the K-major operand), both through the patched ops
    g = torch.Generator().manual_seed(17)
    x = torch.randn(2048, 1024, generator=g)
    w = torch.randn(1024, 2048, generator=g)
    lin = torch.nn.Linear(1024, 1536).to(cuda_device)
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    cmpext3.autoselect.reset()
    with torch.no_grad():
        got = torch.matmul(xd, wd)
        got_lin = lin(xd)
    torch.cuda.synchronize()
    check(got, RP.bmm(x[None], w[None])[0], torch.float32, "patched fp32 matmul", attention=False)
    ref_lin = torch.nn.functional.linear(x.double(), lin.weight.detach().double().cpu(), lin.bias.detach().double().cpu())
    assert ((got_lin.double().cpu() - ref_lin).abs().max() / ref_lin.abs().max()).item() <= 5e-5
    report = cmpext3.autoselect_report()
    assert "bmm_x3tf32_sm100" in report
