"""fp32 attention's tail split on a B200 (marked gpu).

When the last wave of 128-row items is at most half a wave, the fp32 (3xTF32) kernel cuts those
items into key ranges, parks each range's (O, m, l) rows in the workspace and merges them in the CTA
of the item's last range to finish.  Checked here: the result against the reference's CPU path
(stock torch SDPA on CPU) within the fp32 contract, against the same kernel run unsplit (no
workspace) within fp32 summation-order differences, a second call bit-identical to the first (the
arrival counters are left at zero), the workspace's first 256 bytes zero afterwards, and masks.
"""
from __future__ import annotations

import ctypes

import pytest
import torch
import torch.nn.functional as F

from cmpext3 import _native as N
from oracle import reference_path as RP
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu

# (B, H, Lq, Lk, D): the number of 128-row items against the 148 SMs sets the split
SPLIT_SHAPES = [
    (1, 218, 128, 640, 40),    # 218 items: 70 tail items cut in 2 key ranges
    (1, 150, 128, 4096, 64),   # 2 tail items cut in 8
    (1, 75, 512, 1024, 128),   # D = 128 (32-key tiles): 4 tail items cut in 8
    (2, 3, 4500, 556, 24),     # 216 items, a ragged last row tile (4500 rows) and key tile (556 keys)
    (2, 8, 128, 8192, 64),     # 16 items, fewer than SMs: every item cut into 8 key ranges
    (1, 8, 256, 4096, 100),    # 16 items, D = 100 (32-key tiles), every item cut 8 ways
]


def _qkv(shape, seed):
    B, H, Lq, Lk, D = shape
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, H, Lq, D, generator=g), torch.randn(B, H, Lk, D, generator=g),
            torch.randn(B, H, Lk, D, generator=g))


def _unsplit(qd, kd, vd, scale):
    """The same kernel through the C ABI with no workspace: it then runs without the split."""
    q, k, v, out, scale = N._prepare_attention(qd, kd, vd, scale, False)
    desc = N._attn_desc(q, k, v, out, scale, False)
    assert desc.workspace is None or desc.workspace == 0
    st = N.lib.cmpx_attn_fwd(ctypes.byref(desc), N._stream_handle(qd.device))
    assert st == 0, N.lib.cmpx_status_str(st)
    return out


@pytest.mark.parametrize("shape", SPLIT_SHAPES, ids=["x".join(map(str, s)) for s in SPLIT_SHAPES])
def test_split_matches_reference_and_unsplit_run(cuda_device, shape):
    q, k, v = _qkv(shape, seed=sum(shape))
    qd, kd, vd = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    assert N.attention_plan(qd, kd, vd, None, False).endswith("+tail-split>")
    got = N.attention(qd, kd, vd)
    again = N.attention(qd, kd, vd)
    plain = _unsplit(qd, kd, vd, None)
    torch.cuda.synchronize()
    with torch.no_grad():
        ref = RP.sdpa(q, k, v)
    check(got, ref, torch.float32, f"split {shape}")
    assert torch.equal(got, again)  # the counters were left at zero: the second call merges the same way
    assert (got - plain).abs().max().item() <= 1e-5 * max(1.0, plain.abs().max().item())
    ws = [w for (dev, _), w in N._WORKSPACES.items() if dev == qd.device.index]
    assert ws and all(int(w[:256].count_nonzero()) == 0 for w in ws)
    assert N.device_status() == 0


@pytest.mark.parametrize("kind", ["bool", "additive"])
def test_split_with_masks(cuda_device, kind):
    shape = (1, 150, 128, 1024, 64)
    q, k, v = _qkv(shape, seed=9)
    g = torch.Generator().manual_seed(10)
    if kind == "bool":
        mask = torch.rand(1, 1, 128, 1024, generator=g) > 0.3
        mask[..., 5, :] = False  # a row with no key left: output 0, as torch
    else:
        mask = torch.randn(1, 1, 128, 1024, generator=g)
    qd, kd, vd, md = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), mask.to(cuda_device)
    got = N.attention(qd, kd, vd, attn_mask=md)
    torch.cuda.synchronize()
    with torch.no_grad():
        ref = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    if kind == "bool":
        ref = torch.nan_to_num(ref, nan=0.0)  # stock CPU gives NaN for a row with no key; torch CUDA and this kernel 0
        assert got[0, :, 5].abs().max().item() == 0
    check(got, ref, torch.float32, f"split with {kind} mask")
