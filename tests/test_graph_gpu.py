"""The ops inside CUDA graphs (needs a B200; marked gpu).  Serving stacks capture their forward pass
to take the host off the critical path; every op here must capture and replay: its kernels take the
capture stream, the persistent attention kernel leaves its work counters zeroed for the next replay,
the tail split's merge kernel and the mask packing kernel are captured with it.  Replays with new
inputs copied into the captured tensors must equal eager calls bit for bit (the kernels are
deterministic)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import cmpext3

pytestmark = pytest.mark.gpu


def _capture(fn):
    """Warm fn up on a side stream (torch's recipe), capture one call, return (graph, output)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out


def _replay_matches_eager(fn, inputs, make_new):
    g, out = _capture(fn)
    for trial in range(3):
        for t, new in zip(inputs, make_new(trial)):
            t.copy_(new)
        g.replay()
        torch.cuda.synchronize()
        want = fn()
        torch.cuda.synchronize()
        assert torch.equal(out, want), f"replay {trial} differs from the eager call"
    del g


def _randn(shape, dtype, dev, seed):
    gen = torch.Generator(device=dev).manual_seed(seed)
    return torch.randn(*shape, generator=gen, device=dev, dtype=dtype)


@pytest.mark.parametrize("case", ["causal", "split", "mask", "short_keys", "fp32"])
def test_attention_in_a_graph(cuda_device, case):
    dev = cuda_device
    if case == "causal":
        shape_q, shape_k, dtype, causal = (2, 4, 700, 128), (2, 4, 700, 128), torch.bfloat16, True
    elif case == "split":   # 2 items: tail split into 4 key ranges + merge kernel
        shape_q, shape_k, dtype, causal = (1, 1, 512, 64), (1, 1, 4096, 64), torch.float16, False
    elif case == "mask":
        shape_q, shape_k, dtype, causal = (2, 4, 300, 64), (2, 4, 500, 64), torch.bfloat16, False
    elif case == "short_keys":
        shape_q, shape_k, dtype, causal = (2, 10, 1024, 64), (2, 10, 77, 64), torch.float16, False
    else:
        shape_q, shape_k, dtype, causal = (1, 4, 256, 40), (1, 4, 256, 40), torch.float32, False
    q, k, v = _randn(shape_q, dtype, dev, 1), _randn(shape_k, dtype, dev, 2), _randn(shape_k, dtype, dev, 3)
    mask = (torch.rand(shape_q[2], shape_k[2], device=dev) > 0.3) if case == "mask" else None

    def fn():
        return cmpext3.ops.attention(q, k, v, None, causal, mask)

    _replay_matches_eager(fn, [q, k, v], lambda i: [_randn(t.shape, dtype, dev, 10 * i + j)
                                                   for j, t in enumerate((q, k, v))])


def test_bmm_linear_softmax_in_a_graph(cuda_device):
    dev = cuda_device
    a = _randn((4, 256, 512), torch.bfloat16, dev, 1)
    b = _randn((4, 512, 384), torch.bfloat16, dev, 2)
    x = _randn((300, 640), torch.bfloat16, dev, 3)
    w = _randn((1280, 640), torch.bfloat16, dev, 4)
    bias = _randn((1280,), torch.bfloat16, dev, 5)

    def fn():
        c = cmpext3.ops.bmm(a, b)
        return torch.cat([cmpext3.ops.softmax(c, -1).flatten(), cmpext3.ops.linear(x, w, bias).flatten()])

    _replay_matches_eager(fn, [a, b, x], lambda i: [_randn(t.shape, t.dtype, dev, 20 + 3 * i + j)
                                                   for j, t in enumerate((a, b, x))])


def test_patched_sdpa_in_a_graph(cuda_device, patched):
    dev = cuda_device
    q, k, v = (_randn((1, 8, 512, 128), torch.bfloat16, dev, s) for s in (7, 8, 9))

    def fn():
        with torch.no_grad():
            return F.scaled_dot_product_attention(q, k, v, is_causal=True)

    _replay_matches_eager(fn, [q, k, v], lambda i: [_randn(t.shape, t.dtype, dev, 30 + 3 * i + j)
                                                   for j, t in enumerate((q, k, v))])
    entries = [d.entry for d in cmpext3.autoselect.report() if d.use_native]
    assert any("fmha_sm100" in (e or "") for e in entries), cmpext3.autoselect_report()
