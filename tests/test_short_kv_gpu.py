"""The streamed short-key kernel (fmha_sm100_short: non-causal, 1 <= Lk <= 128) against the
reference's CPU path (needs a B200; marked gpu).

The kernel splits the flattened (batch, head, 128-row Q tile) range evenly over the CTAs, loads
K/V of every head it meets into one of two buffers (one for D = 128), and keeps 2-4 tiles in
flight depending on Lk and D, so these cases vary how many tiles and heads land on one CTA: fewer
tiles than SMs, ranges that straddle head boundaries, one tile per head with several heads per CTA
(buffer reuse), many tiles per CTA, ragged Lq, every Lk edge (1, one K=16 step, 16/17, 64/65, 77,
96/97, 127, 128), padded and full head dims, a negative scale and strided [B, L, H, D] views.
Tolerances as in test_parity_gpu.py.
"""
from __future__ import annotations

import math

import pytest
import torch

import cmpext3
from cmpext3 import _native as N
from oracle import reference_path as RP
from tests.test_parity_gpu import _rand_qkv, check

pytestmark = pytest.mark.gpu

CASES = [
    # (B, H, Lq, Lk, D)
    (1, 1, 1, 1, 64),          # one row, one key
    (1, 3, 100, 16, 64),       # one PV step
    (2, 5, 300, 17, 64),       # ragged Lq, two PV steps
    (3, 7, 1000, 77, 64),      # 168 tiles over 148 CTAs: ranges straddle head boundaries
    (2, 10, 4096, 77, 64),     # C2-cross shape: several tiles and heads per CTA
    (1, 2, 700, 127, 128),     # D = 128: three Q stages
    (4, 9, 257, 128, 128),     # full key tile, head changes inside ranges
    (2, 3, 640, 50, 40),       # padded head dim
    (8, 100, 100, 65, 64),     # one tile per head, 5-6 heads per CTA: both K/V buffers reused
    (6, 100, 64, 128, 128),    # D = 128, one K/V buffer, reloaded for every tile of a CTA
    (2, 6, 1000, 64, 64),      # Lk = 64: four tiles in flight per CTA
    (2, 6, 1000, 96, 64),      # Lk = 96: three in flight, no masked key
    (2, 6, 1000, 97, 64),      # Lk = 97: two in flight (128-wide S)
    (1, 1, 2000, 33, 64),      # fewer tiles than SMs, 1-2 tiles per CTA
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("case", CASES, ids=[f"{b}x{h}x{lq}x{lk}_D{d}" for b, h, lq, lk, d in CASES])
def test_short_kv_matches_reference(cuda_device, dtype, case):
    B, H, Lq, Lk, D = case
    q, k, v = _rand_qkv(B, H, Lq, Lk, D, dtype, seed=B * 1000 + H * 100 + Lk + D)
    assert N.attention_plan(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)).startswith(
        "fmha_sm100_short")
    got = cmpext3.ops.attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), None, False)
    torch.cuda.synchronize()
    with torch.no_grad():
        ref = RP.sdpa(q, k, v, scale=1.0 / math.sqrt(D), is_causal=False)
    check(got, ref, dtype, f"short {case} {dtype}")
    assert N.device_status() == 0


@pytest.mark.parametrize("scale", [-0.3, 0.05, 2.0])
def test_short_kv_scales(cuda_device, scale):
    q, k, v = _rand_qkv(2, 4, 333, 77, 64, torch.bfloat16, seed=7)
    got = cmpext3.ops.attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), scale, False)
    torch.cuda.synchronize()
    with torch.no_grad():
        ref = RP.sdpa(q, k, v, scale=scale, is_causal=False)
    check(got, ref, torch.bfloat16, f"short scale {scale}")


def test_short_kv_strided_blhd_views(cuda_device):
    q, k, v = _rand_qkv(2, 10, 500, 77, 64, torch.float16, seed=11, layout="blhd")
    got = cmpext3.ops.attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), None, False)
    torch.cuda.synchronize()
    with torch.no_grad():
        ref = RP.sdpa(q.contiguous(), k.contiguous(), v.contiguous(), scale=0.125, is_causal=False)
    check(got, ref, torch.float16, "short blhd")


def test_short_kv_repeated_calls_are_identical(cuda_device):
    q, k, v = (t.to(cuda_device) for t in _rand_qkv(3, 7, 1000, 77, 64, torch.float16, seed=3))
    a = cmpext3.ops.attention(q, k, v, None, False)
    b = cmpext3.ops.attention(q, k, v, None, False)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
