"""Head dims above 128 (SD1.5's deepest attention level has D = 160) on the 16-bit attention
kernel's 64-key-tile instantiation (D padded to 192), against the reference's CPU path -- stock
torch SDPA on CPU tensors (needs a B200; marked gpu).  Tolerances as in test_parity_gpu.py."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import cmpext3
from cmpext3 import _native as N
from tests.test_parity_gpu import _rand_qkv, _run_and_check, check

pytestmark = pytest.mark.gpu

LENGTHS = [(1, 1), (64, 64), (77, 200), (128, 128), (255, 257), (300, 1000), (513, 384)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("D", [136, 160, 192])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("lens", LENGTHS, ids=[f"{a}x{b}" for a, b in LENGTHS])
def test_wide_head_sweep(cuda_device, dtype, D, causal, lens):
    lq, lk = lens
    q, k, v = _rand_qkv(2, 3, lq, lk, D, dtype, seed=D * 7 + lq + 3 * lk + causal)
    assert N.attention_plan(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), None, causal) \
        .startswith("fmha_sm100<" + ("bf16" if dtype == torch.bfloat16 else "f16") + ",D192")
    _run_and_check(cuda_device, q, k, v, None, causal, f"D{D} {lens} causal={causal}")
    assert N.device_status() == 0


def test_sd15_level4_self_and_cross_attention(cuda_device):
    # 512 px SD1.5, deepest UNet level: 8x8 latents (64 tokens), 8 heads of 160; cross-attention to
    # the 77 text tokens; [B, L, H, D] memory as diffusers produces it
    for lk in (64, 77):
        q, k, v = _rand_qkv(2, 8, 64, lk, 160, torch.float16, seed=lk, layout="blhd")
        _run_and_check(cuda_device, q, k, v, None, False, f"sd15 level 4 lk={lk}")


def test_wide_head_tail_split(cuda_device):
    # 2 items on 148 SMs: the key range is split (8 ranges of 64-key tiles) and merged
    q, k, v = _rand_qkv(1, 1, 512, 4096, 160, torch.bfloat16, seed=3)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    assert "+tail-split" in N.attention_plan(qd, kd, vd, None, False)
    _run_and_check(cuda_device, q, k, v, None, False, "D160 split")


def test_wide_head_grouped_query(cuda_device):
    g = torch.Generator().manual_seed(8)
    q = torch.randn(1, 8, 300, 160, generator=g).to(torch.bfloat16)
    k = torch.randn(1, 2, 300, 160, generator=g).to(torch.bfloat16)
    v = torch.randn(1, 2, 300, 160, generator=g).to(torch.bfloat16)
    got = cmpext3.ops.attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), None, True)
    torch.cuda.synchronize()
    with torch.no_grad():
        ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=True,
                                             enable_gqa=True).to(torch.bfloat16)
    check(got, ref, torch.bfloat16, "D160 gqa")


def test_patched_sdpa_runs_d160_natively(cuda_device, patched):
    q, k, v = (t.to(cuda_device) for t in _rand_qkv(1, 8, 256, 256, 160, torch.float16, seed=1))
    with torch.no_grad():
        F.scaled_dot_product_attention(q, k, v)
    torch.cuda.synchronize()
    entries = [d.entry for d in cmpext3.autoselect.report() if d.use_native]
    assert any("D192" in (e or "") for e in entries), cmpext3.autoselect_report()
