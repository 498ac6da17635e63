"""Tail split of non-causal 16-bit attention (needs a B200; marked gpu).

When the persistent kernel's last wave of (row pair, head) items is partial, each of those items is
cut into key ranges whose partial results a second kernel merges.  These tests check that path
against the reference's CPU path (stock torch SDPA), against the same call run unsplit (a
workspace of only the 256-byte minimum), for determinism, and that the workspace's counters come
back zeroed.  Tolerances as in test_parity_gpu.py."""
from __future__ import annotations

import ctypes
import math

import pytest
import torch

from cmpext3 import _native as N
from oracle import reference_path as RP
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu

NUM_SMS = 148

CASES = [
    # (dtype, B, H, Hkv, Lq, Lk, D)  -- every one splits on a 148-SM B200
    (torch.float16, 1, 1, 1, 512, 4096, 64),     # 2 items, 4 ranges of 8 key tiles each
    (torch.bfloat16, 1, 2, 2, 1024, 2048, 128),  # 8 items, 2 ranges each
    (torch.bfloat16, 2, 3, 3, 300, 4000, 64),    # ragged rows and last key tile, 4 ranges
    (torch.float16, 1, 4, 2, 512, 2048, 128),    # grouped-query heads, 2 ranges
    (torch.bfloat16, 2, 10, 10, 4096, 4096, 64),  # the SD1.5 self-attention shape: 24 of 320 items split 6 ways
]


def _split_of(B, H, Lq, Lk):
    items = ((Lq + 255) // 256) * H * B
    rem = items % NUM_SMS
    if rem == 0:
        return 1, items
    per_range = 8 if items < NUM_SMS else 4  # every item cut: at least 8 key tiles a range
    n_kv = (Lk + 127) // 128
    return (min(NUM_SMS // rem, n_kv // per_range, 8) if n_kv >= 16 else 1), rem


def _inputs(case, seed):
    dtype, B, H, Hkv, Lq, Lk, D = case
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, Lq, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, Lk, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, Lk, D, generator=g).to(dtype)
    return q, k, v


def _call(dev, q, k, v, ws_bytes=None):
    """cmpx_attn_fwd into a NaN-poisoned output; returns (output, workspace)."""
    B, H, Lq, D = q.shape
    out = torch.full((B, Lq, H, D), float("nan"), dtype=q.dtype, device=dev).transpose(1, 2)
    desc = N._attn_desc(q, k, v, out, 1 / math.sqrt(D), False)
    need = N.lib.cmpx_attn_workspace_size(ctypes.byref(desc))
    ws = torch.zeros(need if ws_bytes is None else ws_bytes, dtype=torch.uint8, device=dev)
    desc.workspace, desc.workspace_bytes = ws.data_ptr(), ws.numel()
    assert N.lib.cmpx_attn_fwd(ctypes.byref(desc), N._stream_handle(dev)) == 0
    torch.cuda.synchronize()
    assert N.device_status() == 0
    return out, ws, need


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-{c[1]}x{c[2]}-{c[4]}x{c[5]}-D{c[6]}" for c in CASES])
def test_split_matches_reference_and_unsplit(cuda_device, case):
    dtype, B, H, Hkv, Lq, Lk, D = case
    split, rem = _split_of(B, H, Lq, Lk)
    assert split >= 2, "the case must exercise the split path"
    q, k, v = _inputs(case, seed=B * 1000 + H * 10 + D)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    got, ws, need = _call(cuda_device, qd, kd, vd)
    assert need > 256
    # the work counters are back at zero (the rest of the workspace is the ranges' scratch)
    assert int(ws[:256].count_nonzero()) == 0, "the work counters must be left zeroed"
    assert torch.isfinite(got.float()).all(), "every output element must be written"
    with torch.no_grad():
        ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                                               enable_gqa=H != Hkv).to(dtype)
    check(got, ref, dtype, f"split {case}")
    # the same call with the minimum workspace runs unsplit: same fp32 result up to summation
    # order, so the 16-bit outputs differ by at most a rounding step or two
    plain, _, _ = _call(cuda_device, qd, kd, vd, ws_bytes=256)
    diff = (got.float() - plain.float()).abs().max().item()
    ulps = 2 * torch.finfo(dtype).eps * plain.float().abs().max().item()
    assert diff <= ulps, f"split vs unsplit differ by {diff} (> 2 ulp = {ulps})"


def test_split_is_deterministic(cuda_device):
    case = CASES[0]
    q, k, v = (t.to(cuda_device) for t in _inputs(case, seed=7))
    a, _, _ = _call(cuda_device, q, k, v)
    b, _, _ = _call(cuda_device, q, k, v)
    assert torch.equal(a, b), "the merge order is fixed: repeated calls must agree bit for bit"


def test_split_workspace_reused_across_calls(cuda_device):
    # one workspace, several calls of different split shapes in a row (the binding's reuse pattern):
    # one call's scratch must never be read as another's counters or partial results
    import cmpext3
    for i, case in enumerate(CASES[:4] + CASES[:4][::-1]):
        q, k, v = _inputs(case, seed=50 + i)
        got = cmpext3.ops.attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), None, False)
        torch.cuda.synchronize()
        ref = RP.sdpa(q, k.repeat_interleave(case[2] // case[3], 1), v.repeat_interleave(case[2] // case[3], 1))
        check(got, ref, case[0], f"reuse {case}")
    assert N.device_status() == 0


def test_noalloc_runs_split_shapes_unsplit(cuda_device):
    case = CASES[0]
    q, k, v = (t.to(cuda_device) for t in _inputs(case, seed=3))
    out = torch.empty(1, 512, 1, 64, dtype=q.dtype, device=cuda_device).transpose(1, 2)
    desc = N._attn_desc(q, k, v, out, 1 / 8, False)
    assert N.lib.cmpx_attn_fwd_noalloc(ctypes.byref(desc), N._stream_handle(cuda_device)) == 0
    torch.cuda.synchronize()
    split, _, _ = _call(cuda_device, q, k, v)
    diff = (out.float() - split.float()).abs().max().item()
    assert diff <= 2 * torch.finfo(q.dtype).eps * split.float().abs().max().item()
