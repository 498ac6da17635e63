"""Grouped-query attention (k / v with fewer heads than q; query head h reads key/value head
h // (H // Hkv)) on every attention kernel, against the reference's CPU path -- stock torch SDPA on
CPU tensors with enable_gqa=True (needs a B200; marked gpu).  Tolerances as in test_parity_gpu.py."""
from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

import cmpext3
from cmpext3 import _native as N
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu

CASES = [
    # (dtype, B, H, Hkv, Lq, Lk, D, causal, kernel prefix)
    (torch.bfloat16, 2, 8, 2, 600, 600, 128, True, "fmha_sm100<"),      # general 16-bit kernel
    (torch.float16, 1, 6, 3, 300, 700, 64, False, "fmha_sm100<"),
    (torch.bfloat16, 1, 8, 1, 257, 257, 64, True, "fmha_sm100<"),       # multi-query
    (torch.float16, 2, 10, 5, 500, 77, 64, False, "fmha_sm100_short"),  # short key sequences
    (torch.float32, 1, 8, 2, 300, 300, 40, False, "attn_tf32x3"),        # fp32 tensor cores
    # one query row (decode): the group's query heads folded into one head of `group` rows
    (torch.bfloat16, 8, 32, 8, 1, 4096, 128, False, "fmha_sm100<"),
    (torch.float16, 2, 12, 4, 1, 1000, 64, False, "fmha_sm100<"),
    (torch.bfloat16, 3, 16, 2, 1, 77, 128, False, "fmha_sm100_short"),   # folded, short keys
    (torch.float16, 2, 8, 2, 3, 2000, 64, False, "fmha_sm100<"),        # 3 rows: [B, L, H, D] output, not folded
    (torch.bfloat16, 4, 8, 4, 1, 500, 64, True, "fmha_sm100<"),         # causal: not folded
]


def _ref(q, k, v, causal):
    with torch.no_grad():
        return F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal,
                                              enable_gqa=True).to(q.dtype)


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-H{c[2]}kv{c[3]}-{c[4]}x{c[5]}-D{c[6]}-{'c' if c[7] else 'f'}"
                                             for c in CASES])
def test_gqa_matches_reference(cuda_device, case):
    dtype, B, H, Hkv, Lq, Lk, D, causal, prefix = case
    g = torch.Generator().manual_seed(B * 100 + H * 10 + Hkv + D)
    q = torch.randn(B, H, Lq, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, Lk, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, Lk, D, generator=g).to(dtype)
    qd, kd, vd = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    assert N.attention_plan(qd, kd, vd, None, causal).startswith(prefix)
    got = cmpext3.ops.attention(qd, kd, vd, None, causal)
    torch.cuda.synchronize()
    check(got, _ref(q, k, v, causal), dtype, f"gqa {case}")
    assert N.device_status() == 0


def test_patched_sdpa_with_enable_gqa_runs_native(cuda_device, patched):
    from cmpext3 import autoselect
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, 8, 256, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1, 2, 256, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1, 2, 256, 128, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        got = F.scaled_dot_product_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                             is_causal=True, enable_gqa=True)
    torch.cuda.synchronize()
    check(got, _ref(q, k, v, True), torch.bfloat16, "patched gqa")
    assert any(line.strip().startswith("cmpext3") and "attention" in line
               for line in autoselect.format_report().splitlines())
