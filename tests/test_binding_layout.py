"""Host-side layout preparation of the ctypes binding (CPU tensors; no kernel runs).

The fp32 GEMM reads K-major operands whose rows and batch items start on 16-byte boundaries
(include/cmpx_b200.h, cmpx_bmm); the fp32 attention kernel reads mask rows with 16-byte loads.  The
binding copies or pads what does not fit and passes everything else through untouched -- these
tests pin both halves: the values are unchanged, the layout meets the kernels' rules, and nothing
is copied when nothing needs to be."""
from __future__ import annotations

import pytest
import torch

from cmpext3 import _native as N


def _meets_x3_rules(t: torch.Tensor) -> bool:
    nb, r, _ = t.shape
    s0, s1, s2 = t.stride()
    return (t.data_ptr() % 16 == 0 and s2 == 1 and (r == 1 or s1 % 4 == 0)
            and (nb == 1 or s0 % 4 == 0))


@pytest.mark.parametrize("shape", [(2, 5, 7), (1, 1, 3), (3, 4, 8), (1, 300, 1001)])
@pytest.mark.parametrize("transposed", [False, True])
def test_kmajor_copy_keeps_values_and_meets_the_layout(shape, transposed):
    g = torch.Generator().manual_seed(sum(shape))
    nb, r, k = shape
    t = torch.randn(nb, k, r, generator=g).transpose(1, 2) if transposed else torch.randn(nb, r, k, generator=g)
    out = N._kmajor_f32(t)
    assert torch.equal(out, t) and _meets_x3_rules(out)


def test_kmajor_passes_an_aligned_operand_through():
    t = torch.randn(3, 16, 64)
    assert N._kmajor_f32(t).data_ptr() == t.data_ptr()
    # a B operand given as the transpose of a k-contiguous buffer: no copy either
    bt = torch.randn(3, 48, 64)
    b = bt.transpose(1, 2)
    out = N._kmajor_f32(b.transpose(1, 2)).transpose(1, 2)
    assert out.data_ptr() == bt.data_ptr() and torch.equal(out, b)


@pytest.mark.parametrize("nb,m,n", [(2, 5, 7), (1, 1, 3), (4, 1, 1), (1, 8, 12), (3, 9, 16)])
def test_fp32_output_rows_are_16_byte_aligned(nb, m, n):
    c = N._out_rows(nb, m, n, torch.float32, torch.device("cpu"))
    assert c.shape == (nb, m, n)
    assert m == 1 or c.stride(1) % 4 == 0
    assert nb == 1 or c.stride(0) % 4 == 0
    if n % 4 == 0 or (m == 1 and nb == 1):
        assert c.is_contiguous()


def test_16bit_output_rows_are_never_padded():
    assert N._out_rows(2, 5, 7, torch.bfloat16, torch.device("cpu")).is_contiguous()


@pytest.mark.parametrize("dtype,unit", [(torch.bool, 16), (torch.float32, 4)])
@pytest.mark.parametrize("shape", [(7, 77), (2, 1, 7, 77), (1, 200), (2, 3, 7, 1)])
def test_fp32_call_masks_are_padded_to_16_byte_rows(dtype, unit, shape):
    q = torch.randn(2, 3, 7, 40)
    k = torch.randn(2, 3, 77 if shape[-1] != 200 else 200, 40)
    if shape == (1, 200):
        q = torch.randn(2, 3, 1, 40)
    g = torch.Generator().manual_seed(len(shape))
    mask = (torch.rand(*shape, generator=g) > 0.5) if dtype == torch.bool else torch.randn(*shape, generator=g)
    m = N._prepare_mask(mask, q, k)
    assert m.shape == (q.shape[0], q.shape[1], q.shape[2], k.shape[2])
    assert torch.equal(m, mask.expand_as(m))
    assert m.stride(3) == 1 and m.data_ptr() % 16 == 0
    for i in range(3):   # every dimension that is stepped
        assert m.size(i) == 1 or m.stride(i) % unit == 0


def test_16bit_call_boolean_masks_are_not_padded():
    # the 16-bit kernels pack boolean masks (any layout): the view is passed through
    q, k = torch.randn(1, 2, 7, 64).to(torch.bfloat16), torch.randn(1, 2, 77, 64).to(torch.bfloat16)
    mask = torch.rand(7, 77) > 0.5
    m = N._prepare_mask(mask, q, k)
    assert m.data_ptr() == mask.data_ptr()


def test_additive_mask_of_another_dtype_is_refused():
    q, k = torch.randn(1, 2, 7, 64), torch.randn(1, 2, 9, 64)
    with pytest.raises(RuntimeError):
        N._prepare_mask(torch.zeros(7, 9, dtype=torch.float16), q, k)


def test_nvtx_ranges_wrap_the_ops_when_enabled():
    # CMPEXT3_NVTX is read at import: check in a fresh interpreter that the public ops are wrapped
    # and that a call pushes and pops a range (the op itself then refuses the CPU tensors)
    import os
    import subprocess
    import sys
    code = (
        "import sys; sys.path[:0] = ['torch-cmp-patch_b200', '.']\n"
        "import torch\n"
        "pushed = []\n"
        "torch.cuda.nvtx.range_push = lambda name: pushed.append(name) or 0\n"
        "torch.cuda.nvtx.range_pop = lambda: pushed.append('pop') or 0\n"
        "from cmpext3 import _native as N\n"
        "assert all(hasattr(f, '__wrapped__') for f in (N.attention, N.bmm, N.linear, N.softmax))\n"
        "try:\n"
        "    N.bmm(torch.randn(1, 2, 2), torch.randn(1, 2, 2))\n"
        "except RuntimeError:\n"
        "    pass\n"
        "assert pushed == ['cmpx.bmm', 'pop'], pushed\n"
        "print('ok')\n")
    env = dict(os.environ, CMPEXT3_NVTX="1", CMPEXT3_AUTOPATCH="0")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stderr[-2000:]


def test_ops_are_unwrapped_by_default():
    assert not hasattr(N.attention, "__wrapped__") and not hasattr(N.bmm, "__wrapped__")
