"""Shared pytest setup.

* registers the ``gpu`` marker (tests that need a B200; ``-m "not gpu"`` runs everything else);
* puts the package directory on sys.path and imports ``cmpext3`` with the import-time patch OFF
  (CMPEXT3_AUTOPATCH=0, as the reference's own conftest does, tests/conftest.py:40 there), so tests
  opt in through the ``patched`` fixture;
* builds the C-ABI library first if it is missing (nvcc cross-compiles without a GPU);
* ``native`` swaps the native ops for MagicMocks (the reference's fake-native pattern,
  tests/conftest.py:42-46 there) so the dispatch logic can be tested on CPU tensors, and
  ``force_eligible`` lets CPU tensors through the CUDA gate (reference tests/conftest.py:145-154).
"""
from __future__ import annotations

import os
import sys
import types
from pathlib import Path
from unittest.mock import MagicMock

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "torch-cmp-patch_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

os.environ.setdefault("CMPEXT3_AUTOPATCH", "0")


def _ensure_library() -> None:
    lib = PKG / "cmpext3" / "libcmpx_b200.so"
    if not lib.exists():
        sys.path.insert(0, str(PKG))
        import build  # torch-cmp-patch_b200/build.py
        build.build()


_ensure_library()

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

import cmpext3  # noqa: E402

# Ops this package leaves alone (the reference's other patches -- conv, norms, activations -- are out
# of this hot path's scope).  softmax is patched, but diverts only the attention chain's softmax.
STOCK_UNPATCHED = {(torch, "baddbmm"): torch.baddbmm, (F, "layer_norm"): F.layer_norm,
                   (F, "conv2d"): F.conv2d, (F, "gelu"): F.gelu}
STOCK_SOFTMAX = {"torch": torch.softmax, "F": F.softmax, "Tensor": torch.Tensor.softmax}

NATIVE_OPS = ["attention", "bmm", "attention_plan", "bmm_plan", "softmax", "linear", "linear_plan",
              "bmm_small", "bmm_small_plan", "bmm_rowstats", "bmm_rowstats_plan", "softmax_product",
              "softmax_product_plan"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100) device")


def has_b200() -> bool:
    return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10


@pytest.fixture(autouse=True)
def _fresh_record():
    """Every test starts with an empty dispatch record and the record switched on."""
    from cmpext3 import autoselect
    previous = autoselect._ENABLED
    autoselect._ENABLED = True
    autoselect.reset()
    try:
        yield
    finally:
        autoselect._ENABLED = previous
        autoselect.reset()


@pytest.fixture
def native(monkeypatch):
    """Fake native module (one MagicMock per op) installed as cmpext3._C / cmpext3.ops."""
    fake = types.ModuleType("cmpext3._native_fake")
    for name in NATIVE_OPS:
        setattr(fake, name, MagicMock(name=name))
    fake.attention_plan.return_value = "fake-attention-entry"
    fake.bmm_plan.return_value = "fake-bmm-entry"
    fake.linear_plan.return_value = "fake-linear-entry"
    fake.bmm_small_plan.return_value = "fake-bmm-small-entry"
    fake.bmm_rowstats_plan.return_value = "fake-bmm-rowstats-entry"
    fake.softmax_product_plan.return_value = "fake-softmax-product-entry"
    monkeypatch.setattr(cmpext3, "_C", fake)
    monkeypatch.setattr(cmpext3, "ops", fake)
    return fake


@pytest.fixture
def patched():
    """cmpext3.enable() for the test, always reverted."""
    assert not cmpext3.is_enabled(), "a previous test left cmpext3 enabled"
    cmpext3.enable()
    try:
        yield cmpext3
    finally:
        cmpext3.disable()


def force_eligible(monkeypatch):
    """Let CPU tensors through the wrappers' CUDA / grad gates."""
    monkeypatch.setattr(cmpext3, "_usable", lambda *a, **k: True)
    monkeypatch.setattr(cmpext3, "_grad_safe", lambda *a, **k: True)


@pytest.fixture
def cuda_device():
    """cuda:0, which must be a B200: a GPU test never passes by skipping on a CUDA machine."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device in this process (run the gpu-marked tests on a B200)")
    cap = torch.cuda.get_device_capability(0)
    assert cap[0] == 10, f"gpu tests need an sm_100 device, got sm_{cap[0]}{cap[1]}"
    return torch.device("cuda", 0)
