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


def _noalloc_attention(q, k, v, scale, causal):
    """Run the no-alloc entry point into a fresh [B, Lq, H, D]-memory output (no workspace given)."""
    B, H, Lq, D = q.shape
    out = torch.full((B, Lq, H, D), float("nan"), dtype=q.dtype, device=q.device).transpose(1, 2)
    desc = N._attn_desc(q, k, v, out, scale, causal)
    assert desc.workspace is None and desc.workspace_bytes == 0
    st = _fn(ctypes.byref(desc), N._stream_handle(q.device))
    assert st == N.OK, N.lib.cmpx_status_str(st).decode()
    return out


@pytest.mark.parametrize("dtype,B,H,Lq,Lk,D,causal", [
    (torch.bfloat16, 2, 4, 1000, 1000, 128, True),
    (torch.float16, 1, 3, 700, 77, 64, False),
])
def test_noalloc_matches_allocating_entry_point_twice(cuda_device, dtype, B, H, Lq, Lk, D, causal):
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(B, H, L, D, generator=g).to(dtype).to(cuda_device) for L in (Lq, Lk, Lk))
    scale = 1.0 / math.sqrt(D)
    ref = cmpext3.ops.attention(q, k, v, scale, causal)  # cmpx_attn_fwd with its own workspace
    torch.cuda.synchronize()
    r = ref.float().cpu().numpy()
    for _ in range(2):
        got = _noalloc_attention(q, k, v, scale, causal)
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
