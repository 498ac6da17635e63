"""The reference's own attention kernels, compiled from its sources for sm_100a, as a second checker
on a B200 (marked gpu).

oracle/build_ref.sh compiles src/cuda/fp16_flash_attention_hfma2.cu, fp16_attention.cu and
fp32_attention.cu of the reference (with a C-linkage shim) into oracle/_ref/; the tests skip when
that library is absent.  Each case runs the same inputs through this library, through the
reference's kernel and through the reference's CPU path (stock torch on CPU), and checks that
(1) this library meets the contract against the CPU path, (2) the reference's kernel agrees with
the CPU path by the reference's own criterion (cosine similarity > 0.99,
tests_hardware/test_attention_causal.py:103-110), and (3) this library is at least as close to the
CPU path as the reference's kernel (it accumulates in fp32 where the reference accumulates scores in
half precision).
"""
from __future__ import annotations

import ctypes
import math
from pathlib import Path

import pytest
import torch

from cmpext3 import _native as N
from oracle import reference_path as RP
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libcmpext3_ref_kernels.so"


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("the reference's kernels were not compiled (oracle/build_ref.sh)")
    L = ctypes.CDLL(str(LIB))
    i64p = ctypes.POINTER(ctypes.c_int64)
    L.ref_flash_hfma2.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [i64p] * 4 + [ctypes.c_float,
                                                                                          ctypes.c_void_p]
    L.ref_flash_hfma2.restype = ctypes.c_int
    L.ref_attention_fp16.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_int]
    L.ref_attention_fp32.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_float]
    return L


def _qkv(B, H, Lq, Lk, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, H, Lq, D, generator=g).to(dtype), torch.randn(B, H, Lk, D, generator=g).to(dtype),
            torch.randn(B, H, Lk, D, generator=g).to(dtype))


def _cos(a: torch.Tensor, b: torch.Tensor) -> float:
    return torch.nn.functional.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0).item()


def _strides(t: torch.Tensor):
    s = (ctypes.c_int64 * 3)(*t.stride()[:3])
    return ctypes.cast(s, ctypes.POINTER(ctypes.c_int64)), s


def _compare(ours, theirs, ref, dtype, what):
    check(ours, ref, dtype, f"{what}: this library")
    assert _cos(theirs.cpu(), ref) > 0.99, f"{what}: the reference's kernel disagrees with its CPU path"
    e_ours = (ours.float().cpu() - ref.float()).abs().max().item()
    e_theirs = (theirs.float().cpu() - ref.float()).abs().max().item()
    assert e_ours <= e_theirs * 1.01 + 1e-6, (what, e_ours, e_theirs)


@pytest.mark.parametrize("Lk", [1024, 77], ids=["self", "cross"])
def test_flash_hfma2_fp16(cuda_device, ref, Lk):
    q, k, v = _qkv(1, 4, 1024, Lk, 64, torch.float16, seed=Lk)
    qd, kd, vd = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    theirs = torch.empty_like(qd)
    sp = [_strides(t) for t in (qd, kd, vd, theirs)]
    st = ref.ref_flash_hfma2(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), theirs.data_ptr(), 1, 4, 1024, Lk, 64,
                             sp[0][0], sp[1][0], sp[2][0], sp[3][0], 1 / math.sqrt(64), N._stream_handle(qd.device))
    assert st == 0
    ours = N.attention(qd, kd, vd)
    torch.cuda.synchronize()
    _compare(ours, theirs, RP.sdpa(q, k, v), torch.float16, f"hfma2 Lk={Lk}")


def test_attention_fp16_causal_d128(cuda_device, ref):
    q, k, v = _qkv(1, 4, 512, 512, 128, torch.float16, seed=3)
    qd, kd, vd = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    theirs = torch.empty_like(qd)
    torch.cuda.synchronize()
    ref.ref_attention_fp16(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), theirs.data_ptr(), 1, 4, 512, 128,
                           1 / math.sqrt(128), 1)  # the legacy default stream
    torch.cuda.synchronize()
    ours = N.attention(qd, kd, vd, None, True)
    torch.cuda.synchronize()
    _compare(ours, theirs, RP.sdpa(q, k, v, is_causal=True), torch.float16, "fp16 causal D=128")


def test_attention_fp32_d40(cuda_device, ref):
    q, k, v = _qkv(1, 4, 512, 512, 40, torch.float32, seed=4)
    qd, kd, vd = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    theirs = torch.empty_like(qd)
    torch.cuda.synchronize()
    ref.ref_attention_fp32(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), theirs.data_ptr(), 1, 4, 512, 40,
                           1 / math.sqrt(40))
    torch.cuda.synchronize()
    ours = N.attention(qd, kd, vd)
    torch.cuda.synchronize()
    _compare(ours, theirs, RP.sdpa(q, k, v), torch.float32, "fp32 D=40")
