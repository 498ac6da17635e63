"""The einsum-attention chain's fused softmax on a B200 (marked gpu): the scores product with its
row statistics (cmpx_bmm_rowstats) and the softmax recomputed from the product's operands
(cmpx_softmax_product).

(1) bmm_rowstats returns bmm's product bit for bit, and per row and 64-column run the max of the
stored scores (exact) and the sum of exp(score - max) (float64 restatement, relative 1e-5).
(2) softmax_product recomputes the scores with the bmm kernel's instruction shape and k order and
rounds them the same way, so its softmax matches the reference's CPU path -- stock torch.softmax on
CPU -- applied to the scores the caller holds, within the parity tests' tolerances.  (The softmax is
checked against the caller's scores, not against scores recomputed on the CPU: at attention scales
-- N(0,1) inputs, k = 64, scores with a standard deviation of 8 -- one rounding step of a 16-bit
score moves its probability by tens of percent, so two different products of the same inputs give
different softmaxes by design; the end of the chain, the attention output, is compared with the
full CPU chain.)  With CMPEXT3_FUSED_SOFTMAX=1 the einsum-attention chain (cmpext3/einsum_ops.py:69-121
in the reference) routes its softmax here when the scores are untouched since the einsum; a change in
place to the scores or to an operand falls back to the row-softmax kernel that reads the scores.
"""
from __future__ import annotations

import pytest
import torch

import cmpext3
from cmpext3 import _native as N
from oracle import reference_path as RP
from tests.test_parity_gpu import check

pytestmark = pytest.mark.gpu

SHAPES = [
    # (batch, m, k, n)
    (64, 2048, 64, 2048),   # C3 scores: [4,16] heads, 2048 queries / keys, head dim 64
    (4, 300, 40, 1000),     # ragged m, k padded to 64, partial last 128-column chunk and 64-column run
    (3, 129, 128, 256),     # k = 128
    (2, 77, 80, 128),       # one 128-column chunk per row
    (5, 64, 16, 136),       # k = 16, n one 8-column past a chunk
    (1, 1, 64, 4096),
]


def _ab(shape, dtype, seed):
    bsz, m, k, n = shape
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(bsz, m, k, generator=g).to(dtype)
    b = torch.randn(bsz, n, k, generator=g).to(dtype).transpose(1, 2)  # [bsz, k, n], contiguous along k
    return a, b


def _stats64(c: torch.Tensor) -> torch.Tensor:
    """float64 restatement of the row statistics: [batch, runs, m, 2] (max, sum of exp(c - max))."""
    bsz, m, n = c.shape
    runs = (n + 63) // 64
    x = torch.full((bsz, m, runs * 64), float("-inf"), dtype=torch.float64)
    x[:, :, :n] = c.double().cpu()
    x = x.view(bsz, m, runs, 64)
    mx = x.amax(-1)
    sm = torch.exp(x - mx.unsqueeze(-1)).sum(-1)
    return torch.stack([mx, sm], -1).permute(0, 2, 1, 3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("shape", SHAPES, ids=["x".join(map(str, s)) for s in SHAPES])
def test_softmax_product_matches_reference(cuda_device, dtype, shape):
    a, b = _ab(shape, dtype, seed=sum(shape))
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    assert N.bmm_rowstats_plan(ad, bd).endswith(",rowstats>")
    c, st = N.bmm_rowstats(ad, bd)
    ref_s = N.bmm(ad, bd)
    torch.cuda.synchronize()
    # the product is bmm's product, bit for bit, and agrees with the reference's within the contract
    assert torch.equal(c, ref_s), (c.float() - ref_s.float()).abs().max().item()
    check(ref_s, RP.bmm(a, b), dtype, f"scores {shape} {dtype}", attention=False)
    # the statistics are those of the stored scores
    want = _stats64(c)
    got = st.double().cpu()
    assert torch.equal(got[..., 0], want[..., 0])
    assert torch.allclose(got[..., 1], want[..., 1], rtol=1e-5, atol=0)
    # the softmax is the reference's softmax of those scores
    assert N.softmax_product_plan(ad, bd, st).startswith("softmax_product_sm100<")
    y = N.softmax_product(ad, bd, st)
    with torch.no_grad():
        ref = RP.softmax(ref_s.cpu(), -1)
    check(y, ref, dtype, f"softmax_product {shape} {dtype}", attention=False)
    # against the row-softmax kernel reading the same scores: the same formula in fp32
    rows = N.softmax(ref_s, -1)
    assert (y.float() - rows.float()).abs().max().item() <= 2 ** -7
    assert N.device_status() == 0


def test_rows_of_infinite_scores(cuda_device):
    # a row of all -inf scores (a -inf operand entry times keys that are all +1 there) gives NaN,
    # as torch's softmax does; the other rows are unaffected
    a, b = _ab((2, 130, 64, 256), torch.bfloat16, seed=3)
    a[0, 5] = 0
    a[0, 5, 0] = float("-inf")
    b[0, 0] = 1.0
    ad, bd = a.to(cuda_device), b.to(cuda_device)
    c, st = N.bmm_rowstats(ad, bd)
    y = N.softmax_product(ad, bd, st)
    ref = RP.softmax(c.cpu(), -1)
    torch.cuda.synchronize()
    assert torch.isinf(c[0, 5]).all()
    assert torch.isnan(y[0, 5]).all() and torch.isnan(ref[0, 5]).all()
    ok = torch.ones(2, 130, dtype=torch.bool)
    ok[0, 5] = False
    check(y[ok], ref[ok], torch.bfloat16, "rows without infinities", attention=False)


def test_einsum_chain_recomputes_the_scores(cuda_device, patched, monkeypatch):
    monkeypatch.setattr(cmpext3, "_FUSED_SOFTMAX", True)  # off by default
    g = torch.Generator().manual_seed(4)
    q, k, v = (torch.randn(2, 4, 512, 64, generator=g).to(torch.bfloat16) for _ in range(3))
    qd, kd, vd = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    with torch.no_grad():
        s = torch.einsum("bhid,bhjd->bhij", qd, kd)
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("bhij,bhjd->bhid", p, vd)
    torch.cuda.synchronize()
    entries = [d.entry or "" for d in cmpext3.autoselect.report() if d.use_native]
    assert any(e.startswith("softmax_product_sm100") for e in entries), cmpext3.autoselect_report()
    assert any(e.endswith(",rowstats>") for e in entries), cmpext3.autoselect_report()
    with torch.no_grad():
        ref_s = RP.einsum("bhid,bhjd->bhij", q, k)
        ref_o = RP.einsum_attention(q, k, v)  # the whole chain on the CPU
    check(s, ref_s, torch.bfloat16, "scores", attention=False)
    check(p, RP.softmax(s.cpu(), -1), torch.bfloat16, "probabilities of the returned scores", attention=False)
    check(o, RP.einsum("bhij,bhjd->bhid", p.cpu(), v), torch.bfloat16, "values of the returned probabilities")
    check(o, ref_o, torch.bfloat16, "attention output vs the CPU chain")


def test_scores_changed_in_place_are_read_back(cuda_device, patched, monkeypatch):
    monkeypatch.setattr(cmpext3, "_FUSED_SOFTMAX", True)
    g = torch.Generator().manual_seed(5)
    q, k = (torch.randn(1, 2, 256, 64, generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(2))
    with torch.no_grad():
        s = torch.einsum("bhid,bhjd->bhij", q, k)
        s.mul_(0.125)  # scaled in place: the softmax must see the scaled scores
        p = torch.softmax(s, dim=-1)
    torch.cuda.synchronize()
    check(p, RP.softmax(s.cpu(), -1), torch.bfloat16, "scaled in place", attention=False)
