"""The attention entry point that allocates nothing (cmpx_attn_fwd_noalloc), checked on the GPU.

Some callers cannot allocate device memory when they call attention -- for example a serving
process whose memory pool already owns the whole GPU, or code that runs inside an allocator
callback -- so they cannot hand the kernel a workspace for its work counters.  The no-alloc entry
point uses a fixed scratch array inside the library instead.  This test calls it through the C ABI
twice in a row (the second call sees the scratch the first call left behind) and compares each
result with the ordinary entry point's, within the tolerance the parity tests use.

This file is named so that pytest collects it last; it passes on its own in a fresh process too
(the first call on the device resolves the scratch array's address).
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch

import cmpext3
from cmpext3 import _native as N
from oracle import sdpa_np

pytestmark = pytest.mark.gpu

_fn = N.lib.cmpx_attn_fwd_noalloc
_fn.argtypes = [ctypes.POINTER(N.AttnDesc), ctypes.c_void_p]
_fn.restype = ctypes.c_int


def _noalloc_attention(q, k, v, scale, causal, mask=None):
    """Run the no-alloc entry point into a fresh [B, Lq, H, D]-memory output (no workspace given)."""
    B, H, Lq, D = q.shape
    out = torch.full((B, Lq, H, D), float("nan"), dtype=q.dtype, device=q.device).transpose(1, 2)
    desc = N._attn_desc(q, k, v, out, scale, causal, mask=mask)
    assert desc.workspace is None and desc.workspace_bytes == 0
    st = _fn(ctypes.byref(desc), N._stream_handle(q.device))
    assert st == N.OK, N.lib.cmpx_status_str(st).decode()
    return out


def _workspace_size(q, k, v, scale, causal, mask=None):
    out = torch.empty_like(q)
    desc = N._attn_desc(q, k, v, out, scale, causal, mask=mask)
    return N.lib.cmpx_attn_workspace_size(ctypes.byref(desc))


@pytest.mark.parametrize("dtype,B,H,Lq,Lk,D,causal,additive", [
    (torch.bfloat16, 2, 4, 1000, 1000, 128, True, False),
    (torch.float16, 1, 3, 700, 77, 64, False, False),
    # non-causal with a partial last wave: the allocating entry point splits it (workspace > 256
    # bytes), the no-alloc one runs it unsplit
    (torch.float16, 1, 10, 4096, 4096, 64, False, False),
    # an additive mask needs no workspace beyond the work counters
    (torch.bfloat16, 1, 4, 640, 640, 128, True, True),
])
def test_noalloc_matches_allocating_entry_point_twice(cuda_device, dtype, B, H, Lq, Lk, D, causal, additive):
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(B, H, L, D, generator=g).to(dtype).to(cuda_device) for L in (Lq, Lk, Lk))
    scale = 1.0 / math.sqrt(D)
    mask = None
    if additive:
        mask = (torch.randn(1, 1, Lq, Lk, generator=g) * 2).to(dtype).to(cuda_device)
        mask[..., : Lk // 3] = float("-inf")
    if (B, H, Lq) == (1, 10, 4096):
        assert _workspace_size(q, k, v, scale, causal) > 256  # the split schedule is the fast one here
    # cmpx_attn_fwd with its own workspace
    ref = cmpext3.ops.attention(q, k, v, scale, causal, mask) if mask is not None else \
        cmpext3.ops.attention(q, k, v, scale, causal)
    torch.cuda.synchronize()
    r = ref.float().cpu().numpy()
    m = N._prepare_mask(mask, q, k) if mask is not None else None
    for _ in range(2):
        got = _noalloc_attention(q, k, v, scale, causal, m)
        torch.cuda.synchronize()
        gn = got.float().cpu().numpy()
        assert np.isfinite(gn).all()
        rel = sdpa_np.rel_err(gn, r)
        assert rel <= 1e-2, rel
        if dtype == torch.float16:
            assert sdpa_np.max_abs(gn, r) <= 2e-3
    assert N.device_status() == 0


def test_noalloc_rejects_bad_calls_without_device_work(cuda_device):
    q = torch.randn(1, 1, 64, 256, device=cuda_device, dtype=torch.bfloat16)  # head_dim 256: no kernel
    out = torch.empty_like(q)
    desc = N._attn_desc(q, q, q, out, 1.0, False)
    assert _fn(ctypes.byref(desc), N._stream_handle(cuda_device)) == N.ERR_UNSUPPORTED_SHAPE
    assert _fn(None, None) == N.ERR_INVALID_ARGUMENT


def test_noalloc_declines_boolean_masks(cuda_device):
    """A boolean mask is packed to bits in the workspace, which the fixed scratch cannot hold."""
    q = torch.randn(1, 2, 256, 64, device=cuda_device, dtype=torch.float16)
    mask = torch.ones(1, 1, 256, 256, dtype=torch.bool, device=cuda_device)
    out = torch.empty_like(q)
    desc = N._attn_desc(q, q, q, out, 0.125, False, mask=N._prepare_mask(mask, q, q))
    assert _fn(ctypes.byref(desc), N._stream_handle(cuda_device)) == N.ERR_WORKSPACE
