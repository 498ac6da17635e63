"""attn_mask on the attention kernels -- boolean (packed to bits in the workspace for 16-bit calls) and additive
in the query's dtype (added to the scores in the softmax) -- against the reference's CPU path -- stock torch SDPA with the same mask on CPU tensors
(needs a B200; marked gpu).  The reference itself sent every masked call to stock; these are the
mask shapes models pass: key padding [B,1,1,Lk], a shared [Lq,Lk] pattern, per-head [B,H,Lq,Lk],
rows left with no key (output 0, as torch), masks combined with is_causal (ANDed, torch's math
path), the tail-split schedule, grouped-query heads, head dim 160, and the patched F.sdpa.
Tolerances as in test_parity_gpu.py."""
from __future__ import annotations

import ctypes

import pytest
import torch
import torch.nn.functional as F

import cmpext3
from cmpext3 import _native as N
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu


def _qkv(B, H, Lq, Lk, D, dtype, seed, Hkv=None):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, Lq, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv or H, Lk, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv or H, Lk, D, generator=g).to(dtype)
    return q, k, v, g


def _ref(q, k, v, mask, causal, gqa=False):
    with torch.no_grad():
        return F.scaled_dot_product_attention(q.float(), k.float(), v.float(), attn_mask=mask,
                                              is_causal=causal, enable_gqa=gqa).to(q.dtype)


def _run(dev, q, k, v, mask, causal, what, gqa=False):
    got = cmpext3.ops.attention(q.to(dev), k.to(dev), v.to(dev), None, causal, mask.to(dev))
    torch.cuda.synchronize()
    assert torch.isfinite(got.float()).all(), f"{what}: non-finite output"
    check(got, _ref(q, k, v, mask, causal, gqa), q.dtype, what)
    assert N.device_status() == 0
    return got


MASK_SHAPES = ["key_padding", "shared", "per_head", "per_batch_query"]


def _mask(kind, B, H, Lq, Lk, g):
    if kind == "key_padding":     # [B, 1, 1, Lk]: the last keys of each batch item are padding
        lens = torch.randint(1, Lk + 1, (B,), generator=g)
        return (torch.arange(Lk)[None, :] < lens[:, None]).view(B, 1, 1, Lk)
    if kind == "shared":          # [Lq, Lk]
        return torch.rand(Lq, Lk, generator=g) > 0.3
    if kind == "per_head":        # [B, H, Lq, Lk]
        return torch.rand(B, H, Lq, Lk, generator=g) > 0.5
    return torch.rand(B, 1, Lq, Lk, generator=g) > 0.2   # [B, 1, Lq, Lk]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("kind", MASK_SHAPES)
@pytest.mark.parametrize("D", [64, 128, 160])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("lens", [(77, 77), (300, 1000), (513, 384), (1, 200)], ids=str)
def test_boolean_mask_sweep(cuda_device, dtype, kind, D, causal, lens):
    lq, lk = lens
    q, k, v, g = _qkv(2, 3, lq, lk, D, dtype, seed=lq + 7 * lk + D + causal)
    m = _mask(kind, 2, 3, lq, lk, g)
    assert N.attention_plan(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), None, causal,
                            m.to(cuda_device)).endswith(("+mask>", "+mask+tail-split>"))
    _run(cuda_device, q, k, v, m, causal, f"{kind} D{D} {lens} causal={causal}")


def test_rows_with_no_key_output_zero(cuda_device):
    q, k, v, g = _qkv(1, 2, 300, 400, 128, torch.bfloat16, seed=4)
    m = torch.rand(300, 400, generator=g) > 0.5
    m[7] = False      # row 7: nothing in any key tile
    m[200, :] = False
    m[200, 399] = True  # row 200: only the very last key
    m[255, :128] = False  # row 255: nothing in the first key tile, keys later
    got = _run(cuda_device, q, k, v, m, False, "empty rows")
    assert torch.equal(got[:, :, 7].float().cpu(), torch.zeros(1, 2, 128))


def test_mask_with_tail_split(cuda_device):
    # 2 items on 148 SMs: split into 4 key ranges; some rows have no key in some ranges, one in none
    q, k, v, g = _qkv(1, 1, 512, 4096, 64, torch.float16, seed=5)
    m = torch.rand(512, 4096, generator=g) > 0.97
    m[10] = False
    m[11, :4000] = False
    qd, kd, vd, md = (t.to(cuda_device) for t in (q, k, v, m))
    assert "+tail-split+mask" in N.attention_plan(qd, kd, vd, None, False, md)
    _run(cuda_device, q, k, v, m, False, "split + mask")


def test_mask_with_grouped_query_heads(cuda_device):
    q, k, v, g = _qkv(2, 8, 257, 300, 128, torch.bfloat16, seed=6, Hkv=2)
    m = torch.rand(2, 8, 257, 300, generator=g) > 0.4
    _run(cuda_device, q, k, v, m, True, "gqa + mask", gqa=True)


def test_mask_broadcast_along_keys_is_materialised(cuda_device):
    # [B, H, Lq, 1]: one verdict per query row for every key
    q, k, v, g = _qkv(1, 2, 130, 200, 64, torch.bfloat16, seed=9)
    m = torch.rand(1, 2, 130, 1, generator=g) > 0.3
    _run(cuda_device, q, k, v, m, False, "mask broadcast along keys")


def test_patched_sdpa_boolean_and_additive_masks_native(cuda_device, patched):
    q, k, v, g = _qkv(1, 4, 256, 256, 128, torch.bfloat16, seed=2)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    m = torch.rand(256, 256, generator=g) > 0.5
    add = (torch.randn(256, 256, generator=g) * 2).to(torch.bfloat16)
    with torch.no_grad():
        got = F.scaled_dot_product_attention(qd, kd, vd, attn_mask=m.to(cuda_device))
        got_add = F.scaled_dot_product_attention(qd, kd, vd, attn_mask=add.to(cuda_device))
        F.scaled_dot_product_attention(qd, kd, vd, attn_mask=add.float().to(cuda_device))  # fp32 mask: stock
    torch.cuda.synchronize()
    check(got, _ref(q, k, v, m, False), torch.bfloat16, "patched sdpa mask")
    check(got_add, _ref(q, k, v, add.float(), False), torch.bfloat16, "patched sdpa additive mask")
    entries = [d.entry for d in cmpext3.autoselect.report() if d.use_native]
    assert any((e or "").endswith(("+mask>", "+mask+tail-split>")) for e in entries), cmpext3.autoselect_report()
    assert any((e or "").endswith(("+addmask>", "+addmask+tail-split>")) for e in entries), cmpext3.autoselect_report()


def _additive(kind, B, H, Lq, Lk, dtype, g):
    if kind == "padding":        # 0 / -inf key padding [B, 1, 1, Lk] (the form older models pass)
        lens = torch.randint(1, Lk + 1, (B,), generator=g)
        keep = (torch.arange(Lk)[None, :] < lens[:, None]).view(B, 1, 1, Lk)
        return torch.zeros(B, 1, 1, Lk).masked_fill(~keep, float("-inf")).to(dtype)
    if kind == "alibi":          # per-head linear distance bias [1, H, Lq, Lk]
        slopes = torch.tensor([2.0 ** (-(i + 1)) for i in range(H)]).view(1, H, 1, 1)
        dist = (torch.arange(Lk)[None, :] - torch.arange(Lq)[:, None]).abs().float()
        return (-slopes * dist).to(dtype)
    return (torch.randn(B, H, Lq, Lk, generator=g) * 3).to(dtype)   # arbitrary [B, H, Lq, Lk]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("kind", ["padding", "alibi", "random"])
@pytest.mark.parametrize("D", [64, 128, 160])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("lens", [(77, 77), (300, 1000), (1, 200)], ids=str)
def test_additive_mask_sweep(cuda_device, dtype, kind, D, causal, lens):
    lq, lk = lens
    q, k, v, g = _qkv(2, 3, lq, lk, D, dtype, seed=lq + 5 * lk + D + causal)
    m = _additive(kind, 2, 3, lq, lk, dtype, g)
    qd, kd, vd, md = (t.to(cuda_device) for t in (q, k, v, m))
    assert N.attention_plan(qd, kd, vd, None, causal, md).endswith(("+addmask>", "+addmask+tail-split>"))
    got = cmpext3.ops.attention(qd, kd, vd, None, causal, md)
    torch.cuda.synchronize()
    assert torch.isfinite(got.float()).all()
    check(got, _ref(q, k, v, m.float(), causal), dtype, f"additive {kind} D{D} {lens} causal={causal}")
    assert N.device_status() == 0


def test_additive_mask_all_minus_inf_rows_and_split(cuda_device):
    q, k, v, g = _qkv(1, 1, 512, 4096, 64, torch.float16, seed=11)
    m = torch.randn(512, 4096, generator=g).half()
    m[3] = float("-inf")
    m[4, :4000] = float("-inf")
    qd, kd, vd, md = (t.to(cuda_device) for t in (q, k, v, m))
    assert "+tail-split+addmask" in N.attention_plan(qd, kd, vd, None, False, md)
    got = cmpext3.ops.attention(qd, kd, vd, None, False, md)
    torch.cuda.synchronize()
    assert torch.isfinite(got.float()).all()
    assert torch.equal(got[0, 0, 3].float().cpu(), torch.zeros(64))
    check(got, _ref(q, k, v, m.float(), False), torch.float16, "additive split")


def test_noalloc_declines_masked_calls(cuda_device):
    q, k, v, _ = _qkv(1, 1, 64, 64, 64, torch.bfloat16, seed=1)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    m = torch.ones(64, 64, dtype=torch.bool, device=cuda_device).expand(1, 1, 64, 64)
    out = torch.empty_like(qd)
    desc = N._attn_desc(qd, kd, vd, out, 0.125, False, mask=m)
    assert N.lib.cmpx_attn_fwd_noalloc(ctypes.byref(desc), N._stream_handle(cuda_device)) == N.ERR_WORKSPACE


@pytest.mark.parametrize("kind", ["bool", "additive"])
@pytest.mark.parametrize("scale", [-0.2, 0.05, 1.7])
def test_masks_with_any_scale(cuda_device, kind, scale):
    # a negative scale flips the order of the scores: masked scores become +inf before scaling
    q, k, v, g = _qkv(1, 2, 200, 300, 64, torch.bfloat16, seed=int(abs(scale) * 100) + len(kind))
    if kind == "bool":
        m = torch.rand(200, 300, generator=g) > 0.3
    else:
        m = (torch.randn(200, 300, generator=g) * 2).to(torch.bfloat16)
        m[:, 250:] = float("-inf")
    got = cmpext3.ops.attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), scale, False,
                                m.to(cuda_device))
    torch.cuda.synchronize()
    with torch.no_grad():
        ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=scale,
                                             attn_mask=m if kind == "bool" else m.float()).to(q.dtype)
    check(got, ref, q.dtype, f"{kind} mask scale {scale}")


@pytest.mark.parametrize("kind", ["bool", "additive"])
def test_masks_with_gqa_wide_heads_and_ragged_rows(cuda_device, kind):
    q, k, v, g = _qkv(2, 6, 333, 517, 192, torch.float16, seed=21, Hkv=3)
    if kind == "bool":
        m = torch.rand(2, 1, 333, 517, generator=g) > 0.25
    else:
        m = (torch.rand(2, 6, 333, 517, generator=g) * -4).half()
    got = cmpext3.ops.attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), None, True,
                                m.to(cuda_device))
    torch.cuda.synchronize()
    check(got, _ref(q, k, v, m if kind == "bool" else m.float(), True, gqa=True), torch.float16,
          f"{kind} mask gqa D192")


def test_single_query_row_with_masks(cuda_device):
    q, k, v, g = _qkv(3, 4, 1, 777, 128, torch.bfloat16, seed=31)
    mb = torch.rand(3, 1, 1, 777, generator=g) > 0.5
    ma = torch.where(mb, 0.0, float("-inf")).to(torch.bfloat16)
    for m in (mb, ma):
        got = cmpext3.ops.attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), None, False,
                                    m.to(cuda_device))
        torch.cuda.synchronize()
        check(got, _ref(q, k, v, m if m.dtype == torch.bool else m.float(), False), torch.bfloat16, "Lq=1")


# ------------------------------------------------------------------ fp32 calls (3xTF32 kernel)
# The fp32 kernel reads the mask in place (bytes or fp32 values, 16-byte aligned rows -- the
# binding pads rows that are not) instead of packing it; the contract is fp32's 1e-4.

@pytest.mark.parametrize("kind", MASK_SHAPES)
@pytest.mark.parametrize("D", [40, 64])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("lens", [(77, 77), (300, 1000), (513, 384), (1, 200)], ids=str)
def test_fp32_boolean_mask_sweep(cuda_device, kind, D, causal, lens):
    lq, lk = lens
    q, k, v, g = _qkv(2, 3, lq, lk, D, torch.float32, seed=lq + 7 * lk + D + causal)
    m = _mask(kind, 2, 3, lq, lk, g)
    plan = N.attention_plan(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), None, causal,
                            m.to(cuda_device))
    assert plan.startswith("attn_tf32x3_sm100") and plan.endswith(("+mask>", "+mask+tail-split>")), plan
    _run(cuda_device, q, k, v, m, causal, f"fp32 {kind} D{D} {lens} causal={causal}")


@pytest.mark.parametrize("kind", ["padding", "alibi", "random"])
@pytest.mark.parametrize("D", [40, 64])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("lens", [(77, 77), (300, 1000), (1, 200)], ids=str)
def test_fp32_additive_mask_sweep(cuda_device, kind, D, causal, lens):
    lq, lk = lens
    q, k, v, g = _qkv(2, 3, lq, lk, D, torch.float32, seed=lq + 5 * lk + D + causal)
    m = _additive(kind, 2, 3, lq, lk, torch.float32, g)
    qd, kd, vd, md = (t.to(cuda_device) for t in (q, k, v, m))
    assert N.attention_plan(qd, kd, vd, None, causal, md).endswith(("+addmask>", "+addmask+tail-split>"))
    got = cmpext3.ops.attention(qd, kd, vd, None, causal, md)
    torch.cuda.synchronize()
    assert torch.isfinite(got).all()
    check(got, _ref(q, k, v, m, causal), torch.float32, f"fp32 additive {kind} D{D} {lens} causal={causal}")
    assert N.device_status() == 0


def test_fp32_rows_with_no_key_output_zero(cuda_device):
    q, k, v, g = _qkv(1, 2, 300, 400, 64, torch.float32, seed=4)
    m = torch.rand(300, 400, generator=g) > 0.5
    m[7] = False          # row 7: nothing in any key tile
    m[200, :] = False
    m[200, 399] = True    # row 200: only the very last key
    m[255, :128] = False  # row 255: nothing in the first two key tiles, keys later
    got = _run(cuda_device, q, k, v, m, False, "fp32 empty rows")
    assert torch.equal(got[:, :, 7].cpu(), torch.zeros(1, 2, 64))
    add = torch.randn(300, 400, generator=g)
    add[9] = float("-inf")
    add[10, :300] = float("-inf")
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    got = cmpext3.ops.attention(qd, kd, vd, None, False, add.to(cuda_device))
    torch.cuda.synchronize()
    assert torch.equal(got[:, :, 9].cpu(), torch.zeros(1, 2, 64))
    check(got, _ref(q, k, v, add, False), torch.float32, "fp32 additive -inf rows")


@pytest.mark.parametrize("kind", ["bool", "additive"])
@pytest.mark.parametrize("scale", [-0.2, 0.05, 1.7])
def test_fp32_masks_with_any_scale_and_gqa(cuda_device, kind, scale):
    q, k, v, g = _qkv(2, 4, 150, 170, 40, torch.float32, seed=int(scale * 100) + 3, Hkv=2)
    m = (torch.rand(2, 4, 150, 170, generator=g) > 0.4) if kind == "bool" else torch.randn(1, 4, 150, 170, generator=g)
    got = cmpext3.ops.attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), scale, False,
                                m.to(cuda_device))
    torch.cuda.synchronize()
    with torch.no_grad():
        ref = F.scaled_dot_product_attention(q, k, v, attn_mask=m, scale=scale, enable_gqa=True)
    check(got, ref, torch.float32, f"fp32 {kind} scale {scale}")


def test_fp32_patched_sdpa_masks_native(cuda_device, patched):
    q, k, v, g = _qkv(1, 4, 256, 300, 40, torch.float32, seed=12)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    m = torch.rand(256, 300, generator=g) > 0.5
    add = torch.randn(1, 1, 256, 300, generator=g)
    cmpext3.autoselect.reset()
    with torch.no_grad():
        got = F.scaled_dot_product_attention(qd, kd, vd, attn_mask=m.to(cuda_device))
        got_add = F.scaled_dot_product_attention(qd, kd, vd, attn_mask=add.to(cuda_device))
    torch.cuda.synchronize()
    check(got, _ref(q, k, v, m, False), torch.float32, "fp32 patched sdpa mask")
    check(got_add, _ref(q, k, v, add, False), torch.float32, "fp32 patched sdpa additive mask")
    entries = [d.entry for d in cmpext3.autoselect.report() if d.use_native]
    assert any("attn_tf32x3" in (e or "") and (e or "").endswith(("+mask>", "+mask+tail-split>")) for e in entries), cmpext3.autoselect_report()
    assert any("attn_tf32x3" in (e or "") and (e or "").endswith(("+addmask>", "+addmask+tail-split>")) for e in entries), cmpext3.autoselect_report()
