"""Failure detection without a GPU fault (marked gpu).

Every in-kernel wait of this library is bounded: a wait that runs out raises the CTA's abort word
and the device status word, drains its in-flight copies, frees TMEM and returns.  Here the bounded
wait is made to run out on purpose in the self-test kernel (an mbarrier that nothing arrives on,
20 ms limit); the host must see CMPX_DEVFLAG_WAIT_TIMEOUT, and the context must stay usable.
"""
from __future__ import annotations

import time

import pytest
import torch

import cmpext3
from cmpext3 import _native as N

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda_device):
    assert N.device_status() == 0
    t0 = time.perf_counter()
    N.selftest_wait_timeout(20_000_000, cuda_device)
    flags = N.device_status()
    elapsed = time.perf_counter() - t0
    assert flags & N.DEVFLAG_WAIT_TIMEOUT
    assert elapsed < 5.0
    # the status word was cleared by the read, and the device still runs real work
    assert N.device_status() == 0
    q = torch.randn(1, 2, 256, 128, device=cuda_device, dtype=torch.bfloat16)
    out = cmpext3.ops.attention(q, q, q, None, True)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert N.device_status() == 0


def test_selftest_rejects_unbounded_request(cuda_device):
    with pytest.raises(RuntimeError):
        N.selftest_wait_timeout(0, cuda_device)
    with pytest.raises(RuntimeError):
        N.selftest_wait_timeout(60 * 1_000_000_000, cuda_device)
