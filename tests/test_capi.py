"""The C-ABI library without a GPU: it loads, exports every declared symbol, and its host-side logic
(argument validation, tile-table plan, status strings) behaves -- no compute call is made."""
from __future__ import annotations

import ctypes
import math
import re
from pathlib import Path

import pytest

from cmpext3 import _native as N

HEADER = Path(__file__).resolve().parents[1] / "include" / "cmpx_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^CMPX_API\s+[\w\s\*]+?\b(cmpx_\w+)\s*\(", text, flags=re.M)


def test_header_declares_the_expected_entry_points():
    syms = declared_symbols()
    for name in ("cmpx_attn_fwd", "cmpx_bmm", "cmpx_status_str", "cmpx_attn_plan", "cmpx_bmm_plan",
                 "cmpx_device_status", "cmpx_attn_workspace_size", "cmpx_abi_version",
                 "cmpx_selftest_wait_timeout"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(N.LIBRARY_PATH))
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in {HEADER.name} but not exported"


def test_library_exports_nothing_undeclared():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(N.LIBRARY_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == set(declared_symbols())


def test_abi_version_and_status_strings():
    assert N.lib.cmpx_abi_version() == 7
    header = HEADER.read_text()
    m = re.search(r"#define CMPX_ABI_VERSION (\d+)", header)
    assert m and int(m.group(1)) == N.ABI_VERSION == N.lib.cmpx_abi_version()
    assert N.lib.cmpx_status_str(0) == b"ok"
    for code in range(1, 9):
        assert N.lib.cmpx_status_str(code) not in (b"ok", b"unknown status")
    assert N.lib.cmpx_status_str(12345) == b"unknown status"


def _attn(B=1, H=2, Lq=256, Lk=256, D=128, dtype=2, causal=0, scale=None, ptr=0x10000):
    d = N.AttnDesc()
    d.q = d.k = d.v = d.o = ptr
    d.batch, d.heads, d.len_q, d.len_k, d.head_dim = B, H, Lq, Lk, D
    for name, L in (("q_stride", Lq), ("k_stride", Lk), ("v_stride", Lk), ("o_stride", Lq)):
        getattr(d, name)[:] = (H * L * D, L * D, D)
    d.dtype, d.causal = dtype, causal
    d.scale = (1 / math.sqrt(D)) if scale is None else scale
    return d


def _plan(d):
    buf = ctypes.create_string_buffer(128)
    st = N.lib.cmpx_attn_plan(ctypes.byref(d), buf, 128)
    return st, buf.value.decode()


@pytest.mark.parametrize("cfg,entry", [
    (dict(B=2, H=8, Lq=4096, Lk=4096, D=40, dtype=0), "attn_tf32x3_sm100<D64"),
    (dict(B=2, H=10, Lq=4096, Lk=4096, D=64, dtype=1), "fmha_sm100<f16,D64"),
    (dict(B=2, H=10, Lq=4096, Lk=77, D=64, dtype=1), "fmha_sm100_short<f16,D64"),
    (dict(B=4, H=32, Lq=8192, Lk=8192, D=128, dtype=2, causal=1), "fmha_sm100<bf16,D128"),
    (dict(B=64, H=32, Lq=8192, Lk=8192, D=128, dtype=2, causal=1), "fmha_sm100<bf16,D128"),
])
def test_tile_table_covers_every_config(cfg, entry):
    st, name = _plan(_attn(**cfg))
    assert st == N.OK and name.startswith(entry), (st, name)


@pytest.mark.parametrize("cfg,entry", [
    (dict(Lq=4096, Lk=77, D=64, dtype=1), "fmha_sm100_short<f16,D64"),
    (dict(Lq=1, Lk=1, D=128, dtype=2), "fmha_sm100_short<bf16,D128"),
    (dict(Lq=300, Lk=128, D=40, dtype=2), "fmha_sm100_short<bf16,D64"),
    (dict(Lq=300, Lk=129, D=64, dtype=2), "fmha_sm100<bf16,D64"),      # two key tiles
    (dict(Lq=300, Lk=77, D=64, dtype=2, causal=1), "fmha_sm100<bf16,D64"),  # causal: general kernel
])
def test_short_key_sequences_take_the_streamed_kernel(cfg, entry):
    st, name = _plan(_attn(**cfg))
    assert st == N.OK and name.startswith(entry), (st, name)


@pytest.mark.parametrize("heads_kv", [0, 1, 2, 4, 8])
def test_grouped_query_heads_are_accepted(heads_kv):
    d = _attn(H=8, D=128)
    d.heads_kv = heads_kv
    st, name = _plan(d)
    assert st == N.OK and name.startswith("fmha_sm100<bf16,D128"), (st, name)


@pytest.mark.parametrize("cfg,entry", [
    (dict(D=40, dtype=0), "attn_tf32x3_sm100<D64"),
    (dict(D=64, dtype=0, causal=1), "attn_tf32x3_sm100<D64"),
    (dict(D=68, dtype=0), "attn_tf32x3_sm100<D128,128q,32kv"),   # 32-key tiles above 64
    (dict(D=100, dtype=0), "attn_tf32x3_sm100<D128"),
    (dict(D=128, dtype=0, causal=1), "attn_tf32x3_sm100<D128"),
    (dict(D=37, dtype=0), "misaligned"),                # 148-byte rows: the binding pads them
    (dict(D=160, dtype=0), None),                       # above the reference kernel's D <= 128
])
def test_fp32_tile_table(cfg, entry):
    st, name = _plan(_attn(**cfg))
    if entry is None:
        assert st == N.ERR_UNSUPPORTED_SHAPE, (st, name)
    elif entry == "misaligned":
        assert st == N.ERR_MISALIGNED, (st, name)
    else:
        assert st == N.OK and name.startswith(entry), (st, name)


@pytest.mark.parametrize("mutate,status", [
    (lambda d: setattr(d, "q", None), N.ERR_INVALID_ARGUMENT),
    (lambda d: setattr(d, "batch", -1), N.ERR_INVALID_ARGUMENT),
    (lambda d: setattr(d, "head_dim", 256), N.ERR_UNSUPPORTED_SHAPE),
    (lambda d: setattr(d, "head_dim", 36), N.ERR_UNSUPPORTED_SHAPE),
    (lambda d: setattr(d, "dtype", 7), N.ERR_UNSUPPORTED_DTYPE),
    (lambda d: setattr(d, "scale", float("nan")), N.ERR_INVALID_ARGUMENT),
    (lambda d: setattr(d, "scale", 0.0), N.ERR_UNSUPPORTED_SHAPE),
    (lambda d: setattr(d, "len_k", 0), N.ERR_UNSUPPORTED_SHAPE),
    (lambda d: setattr(d, "q", 0x10008), N.ERR_MISALIGNED),
    (lambda d: d.k_stride.__setitem__(2, 100), N.ERR_MISALIGNED),
    (lambda d: setattr(d, "causal", 2), N.ERR_INVALID_ARGUMENT),
    (lambda d: setattr(d, "heads_kv", 3), N.ERR_INVALID_ARGUMENT),   # does not divide heads=2
    (lambda d: setattr(d, "heads_kv", -1), N.ERR_INVALID_ARGUMENT),
])
def test_invalid_attention_descriptors_are_rejected_before_launch(mutate, status):
    d = _attn()
    mutate(d)
    assert _plan(d)[0] == status
    # the launch entry point rejects them the same way, without touching a device
    assert N.lib.cmpx_attn_fwd(ctypes.byref(d), None) == status


def test_null_descriptor_is_rejected():
    assert N.lib.cmpx_attn_fwd(None, None) == N.ERR_INVALID_ARGUMENT
    assert N.lib.cmpx_bmm(None, None) == N.ERR_INVALID_ARGUMENT


def _bmm(nb=64, m=2048, n=2048, k=64, dtype=2, bt=False, ptr=0x10000):
    d = N.BmmDesc()
    d.a = d.b = d.c = ptr
    d.batch, d.m, d.n, d.k = nb, m, n, k
    d.a_stride[:] = (m * k, k, 1)
    d.b_stride[:] = (k * n, 1, k) if bt else (k * n, n, 1)
    d.c_stride[:] = (m * n, n, 1)
    d.dtype = dtype
    return d


def _bplan(d):
    buf = ctypes.create_string_buffer(128)
    st = N.lib.cmpx_bmm_plan(ctypes.byref(d), buf, 128)
    return st, buf.value.decode()


def test_bmm_plan_for_the_einsum_attention_shapes():
    st, name = _bplan(_bmm(64, 2048, 2048, 64, bt=True))     # scores: B = K^T view (K-major)
    assert st == 0 and "128x128" in name and "B:k-major" in name
    st, name = _bplan(_bmm(64, 2048, 64, 2048, bt=False))    # values: B = V (N-major)
    assert st == 0 and "128x64" in name and "B:mn-major" in name

    # fp32: the 3xTF32 GEMM, which reads K-major operands only
    st, name = _bplan(_bmm(64, 2048, 2048, 64, dtype=0, bt=True))
    assert st == 0 and name.startswith("bmm_x3tf32_sm100<f32,128x128x32"), name


def _rsplan(d, stats=0x20000):
    buf = ctypes.create_string_buffer(128)
    st = N.lib.cmpx_bmm_rowstats_plan(ctypes.byref(d), stats, buf, 128)
    return st, buf.value.decode()


def _spplan(d, stats=0x20000, y=0x30000):
    buf = ctypes.create_string_buffer(128)
    st = N.lib.cmpx_softmax_product_plan(ctypes.byref(d), stats, y, buf, 128)
    return st, buf.value.decode()


def test_fused_softmax_plans_for_the_einsum_attention_scores():
    for dtype, tag in ((2, "bf16"), (1, "f16")):
        st, name = _rsplan(_bmm(64, 2048, 2048, 64, dtype=dtype, bt=True))
        assert st == 0 and name == f"bmm_sm100<{tag},128x128x64,A:k-major,B:k-major,4st,persistent,rowstats>"
        st, name = _spplan(_bmm(64, 2048, 2048, 64, dtype=dtype, bt=True))
        assert st == 0 and name == f"softmax_product_sm100<{tag},128x128,k64,rowstats>", name
    st, name = _spplan(_bmm(4, 300, 1000, 128, bt=True))
    assert st == 0 and ",k128," in name


@pytest.mark.parametrize("kw,status", [
    (dict(bt=False), "ERR_MISALIGNED"),        # B contiguous along n: the statistics need K-major B
    (dict(dtype=0), "ERR_UNSUPPORTED_DTYPE"),  # 16-bit only
    (dict(k=30), "ERR_MISALIGNED"),            # 60-byte A rows
])
def test_rowstats_plan_rejects(kw, status):
    args = dict(nb=2, m=256, n=256, k=64, bt=True)
    args.update(kw)
    assert _rsplan(_bmm(**args))[0] == getattr(N, status)
    assert _rsplan(_bmm(2, 256, 256, 64, bt=True), stats=0x20004)[0] == N.ERR_INVALID_ARGUMENT  # 4-byte aligned
    assert _rsplan(_bmm(2, 256, 256, 64, bt=True), stats=0)[0] == N.ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("kw,status", [
    (dict(k=136), "ERR_UNSUPPORTED_SHAPE"),    # head dims up to 128
    (dict(bt=False), "ERR_MISALIGNED"),
    (dict(dtype=0), "ERR_UNSUPPORTED_DTYPE"),
    (dict(ptr=0x10008), "ERR_MISALIGNED"),
])
def test_softmax_product_plan_rejects(kw, status):
    args = dict(nb=2, m=256, n=256, k=64, bt=True)
    args.update(kw)
    assert _spplan(_bmm(**args))[0] == getattr(N, status)
    assert _spplan(_bmm(2, 256, 256, 64, bt=True), stats=0)[0] == N.ERR_INVALID_ARGUMENT
    assert _spplan(_bmm(2, 256, 256, 64, bt=True), y=0x30008)[0] == N.ERR_MISALIGNED


@pytest.mark.parametrize("kw,status", [
    (dict(bt=False), "ERR_MISALIGNED"),        # B contiguous along n (MN-major): the binding copies it
    (dict(k=30), "ERR_MISALIGNED"),            # 120-byte A rows
    (dict(n=30), "ERR_MISALIGNED"),            # 120-byte C rows
    (dict(ptr=0x10004), "ERR_MISALIGNED"),     # 4-byte aligned pointers
    (dict(k=0), "ERR_UNSUPPORTED_SHAPE"),
])
def test_fp32_bmm_plan_rejects(kw, status):
    args = dict(nb=2, m=256, n=256, k=64, dtype=0, bt=True)
    args.update(kw)
    assert _bplan(_bmm(**args))[0] == getattr(N, status)


@pytest.mark.parametrize("k,chunked", [(8192, False), (8196, True), (40000, True)])
def test_fp32_bmm_plan_chunks_long_k(k, chunked):
    # past K = 8192 the product runs over K chunks (each accumulated in the tensor core's fp32,
    # then summed into C in fp32)
    st, name = _bplan(_bmm(2, 256, 256, k, dtype=0, bt=True))
    assert st == 0 and name.startswith("bmm_x3tf32_sm100<f32") and name.endswith("+k-chunks>") == chunked, name


def test_fp32_bmm_plan_single_rows_need_no_aligned_row_stride():
    # one batch item, m = 1 and n = 1: no stride is ever stepped
    st, name = _bplan(_bmm(1, 1, 1, 64, dtype=0, bt=True))
    assert st == 0 and name.startswith("bmm_x3tf32"), name
    # four items of a 1 x 1 output are 4 bytes apart: not a TMA stride
    assert _bplan(_bmm(4, 1, 1, 64, dtype=0, bt=True))[0] == N.ERR_MISALIGNED


@pytest.mark.parametrize("shape,width", [((8, 4096, 4096, 4096), "128x256"), ((1, 300, 520, 600), "128x256"),
                                         ((4, 512, 256, 256), "128x128"), ((64, 2048, 2048, 64), "128x128"),
                                         ((2, 512, 128, 1024), "128x64")])
def test_bmm_tile_width(shape, width):
    nb, m, n, k = shape  # 128x256 only for wide N with K >= 512 (compute-bound); 128x128 / 128x64 else
    st, name = _bplan(_bmm(nb, m, n, k, bt=True))
    assert st == 0 and width in name, name


def _x3_ws(nb, m, n, k):
    """The fp32 split-operand workspace: 512 bytes (256 left alone, a 16-byte flag at 256), then
    lo(A) [nb][m][k4] and lo(B) [nb][n][k4] fp32, each rounded up to 256 bytes (k4 = k rounded to 4)."""
    k4 = (k + 3) // 4 * 4
    up = lambda x: (x + 255) // 256 * 256  # noqa: E731
    return 512 + up(nb * m * k4 * 4) + up(nb * n * k4 * 4)


@pytest.mark.parametrize("shape,split", [((1, 4096, 4096, 4096), True), ((8, 2048, 2048, 2048), True),
                                         ((1, 1024, 1024, 512), True), ((2, 1024, 1024, 20000), True),
                                         ((64, 2048, 2048, 64), False), ((4, 1024, 1024, 256), False),
                                         ((4, 512, 512, 1024), False), ((1, 8192, 256, 4096), False),
                                         ((16, 128, 128, 128), False)])
def test_fp32_bmm_workspace_size(shape, split):
    # split operands when m n / (m + n) >= 512 per item (every operand tile feeds enough outputs)
    # and k >= 512 (enough K blocks per tile for the converter to be what bounds it)
    nb, m, n, k = shape
    d = _bmm(nb, m, n, k, dtype=0, bt=True)
    assert _bplan(d)[0] == 0
    assert N.lib.cmpx_bmm_workspace_size(ctypes.byref(d)) == (_x3_ws(nb, m, n, k) if split else 0)


def test_fp32_mn_major_b_is_served_through_the_workspace():
    # cmpx_bmm declines an MN-major fp32 B; with a workspace the pass writes B K-major (hi and lo)
    nb, m, n, k = 1, 4096, 4096, 4096
    d = _bmm(nb, m, n, k, dtype=0, bt=False)
    assert _bplan(d)[0] == N.ERR_MISALIGNED
    k4 = (k + 3) // 4 * 4
    assert N.lib.cmpx_bmm_workspace_size(ctypes.byref(d)) == _x3_ws(nb, m, n, k) + nb * n * k4 * 4
    # below the split rule there is no workspace schedule for it either
    assert N.lib.cmpx_bmm_workspace_size(ctypes.byref(_bmm(4, 512, 512, 1024, dtype=0, bt=False))) == 0
    # a workspace entry call without enough workspace keeps the plan's answer
    assert N.lib.cmpx_bmm_ws(ctypes.byref(d), None, 0, None) == N.ERR_MISALIGNED


def test_bmm_workspace_size_is_zero_for_16bit_and_rejected_calls():
    assert N.lib.cmpx_bmm_workspace_size(ctypes.byref(_bmm(1, 4096, 4096, 4096, dtype=2, bt=True))) == 0
    assert N.lib.cmpx_bmm_workspace_size(ctypes.byref(_bmm(2, 4096, 4096, 30, dtype=0, bt=True))) == 0  # misaligned
    assert N.lib.cmpx_bmm_workspace_size(None) == 0


def test_linear_workspace_size():
    d = _linear(m=8192, n=4096, k=4096, dtype=0)
    assert N.lib.cmpx_linear_workspace_size(ctypes.byref(d)) == _x3_ws(1, 8192, 4096, 4096)
    assert N.lib.cmpx_linear_workspace_size(ctypes.byref(_linear(m=8192, n=4096, k=4096, dtype=2))) == 0
    assert N.lib.cmpx_linear_workspace_size(ctypes.byref(_linear(m=64, n=128, k=256, dtype=0))) == 0


def test_workspace_entry_points_validate_before_launch():
    # the same plan checks as cmpx_bmm / cmpx_linear, before any device work
    assert N.lib.cmpx_bmm_ws(ctypes.byref(_bmm(2, 256, 256, 0, dtype=0, bt=True)), None, 0, None) == \
        N.ERR_UNSUPPORTED_SHAPE
    assert N.lib.cmpx_linear_ws(ctypes.byref(_linear(k=100)), None, 0, None) == N.ERR_MISALIGNED


def _linear(m=64, n=128, k=256, dtype=2, bias=True, ptr=0x10000, ldx=None, ldw=None, ldy=None):
    d = N.LinearDesc()
    d.x = d.w = d.y = ptr
    d.bias = ptr if bias else None
    d.m, d.n, d.k = m, n, k
    d.x_row_stride = ldx if ldx is not None else k
    d.w_row_stride = ldw if ldw is not None else k
    d.y_row_stride = ldy if ldy is not None else n
    d.dtype = dtype
    return d


def _lplan(d):
    buf = ctypes.create_string_buffer(128)
    st = N.lib.cmpx_linear_plan(ctypes.byref(d), buf, 128)
    return st, buf.value.decode()


def test_linear_plan_reads_the_weight_as_a_k_major_operand():
    st, name = _lplan(_linear(m=8192, n=4096, k=4096))
    assert st == 0 and "128x256" in name and "A:k-major,B:k-major" in name, name
    st, name = _lplan(_linear(m=100, n=64, k=128, dtype=1, bias=False))
    assert st == 0 and name.startswith("bmm_sm100<f16,128x64"), name
    st, name = _lplan(_linear(m=300, n=100, k=36, dtype=0))  # fp32: 16-byte rows at k, n % 4 == 0
    assert st == 0 and name.startswith("bmm_x3tf32_sm100"), name


@pytest.mark.parametrize("kw,status", [
    (dict(k=100), "ERR_MISALIGNED"),                   # 200-byte rows
    (dict(n=36), "ERR_MISALIGNED"),                    # 72-byte output rows
    (dict(ldx=100), "ERR_INVALID_ARGUMENT"),           # row stride shorter than a row
    (dict(m=-1), "ERR_INVALID_ARGUMENT"),
])
def test_linear_rejects(kw, status):
    assert _lplan(_linear(**kw))[0] == getattr(N, status)


def test_linear_rejects_misaligned_bias_and_null_pointers():
    d = _linear()
    d.bias = 0x10008
    assert _lplan(d)[0] == N.ERR_MISALIGNED
    d = _linear()
    d.w = None
    assert N.lib.cmpx_linear(ctypes.byref(d), None) == N.ERR_INVALID_ARGUMENT


def test_bmm_rejects_misaligned_rows():
    d = _bmm(2, 64, 62, 64)  # N*2 bytes = 124, not a 16-byte multiple
    assert _bplan(d)[0] == N.ERR_MISALIGNED


@pytest.mark.parametrize("cfg,entry", [
    (dict(B=2, H=8, Lq=256, Lk=256, D=160, dtype=1), "fmha_sm100<f16,D192,2x128q,64kv"),    # SD1.5 level 4
    (dict(B=1, H=4, Lq=1000, Lk=1000, D=192, dtype=2, causal=1), "fmha_sm100<bf16,D192,2x128q,64kv"),
    (dict(B=2, H=8, Lq=4096, Lk=77, D=160, dtype=1), "fmha_sm100<f16,D192"),               # not the short kernel
])
def test_plan_for_head_dims_above_128(cfg, entry):
    st, name = _plan(_attn(**cfg))
    assert st == 0 and name.startswith(entry), name


@pytest.mark.parametrize("D", [200, 256])
def test_head_dims_above_192_are_outside_the_table(D):
    assert _plan(_attn(D=D))[0] == N.ERR_UNSUPPORTED_SHAPE


def _with_mask(d, strides):
    d.mask = 0x20000
    d.mask_stride[:] = strides
    return d


def test_mask_is_packed_in_the_workspace():
    # [B, 1, Lq, Lk] key/query mask broadcast over heads: B x Lq rows of ceil(Lk/32) words (a
    # multiple of 4), 256-byte aligned, after the 256 bytes of work counters
    d = _with_mask(_attn(B=2, H=8, Lq=300, Lk=77, D=64, dtype=2, causal=1), (300 * 77, 0, 77, 1))
    rows, words = 2 * 300, 4
    packed = (rows * words * 4 + 255) // 256 * 256
    assert N.lib.cmpx_attn_workspace_size(ctypes.byref(d)) == 256 + packed
    d.workspace, d.workspace_bytes = 0x10000, 256  # too small for the packed mask
    assert N.lib.cmpx_attn_fwd(ctypes.byref(d), None) == N.ERR_WORKSPACE


@pytest.mark.parametrize("strides,status", [
    ((0, 0, 77, 2), N.ERR_INVALID_ARGUMENT),    # keys not contiguous
    ((-1, 0, 77, 1), N.ERR_INVALID_ARGUMENT),
])
def test_mask_stride_rules(strides, status):
    d = _with_mask(_attn(Lq=64, Lk=77, dtype=2), strides)
    assert _plan(d)[0] == status


def test_additive_mask_rules():
    d = _with_mask(_attn(Lq=64, Lk=80, dtype=1), (0, 0, 80, 1))
    d.mask_kind = 1
    st, name = _plan(d)
    assert st == 0 and name.endswith("+addmask>"), name
    assert N.lib.cmpx_attn_workspace_size(ctypes.byref(d)) == 256  # nothing to pack
    d.mask_stride[2] = 77   # 154-byte rows: no 16-byte vector loads
    assert _plan(d)[0] == N.ERR_MISALIGNED
    d.mask_stride[2] = 80
    d.mask_kind = 7
    assert _plan(d)[0] == N.ERR_INVALID_ARGUMENT


def test_mask_plans_on_the_16bit_and_fp32_kernels():
    d = _with_mask(_attn(Lq=64, Lk=77, dtype=2), (0, 0, 77, 1))
    st, name = _plan(d)
    assert st == 0 and name.startswith("fmha_sm100<bf16") and name.endswith("+mask>"), name
    # fp32 reads the mask in place with 16-byte loads: rows 16-byte aligned (the binding pads them)
    d = _with_mask(_attn(Lq=64, Lk=77, D=40, dtype=0), (0, 0, 80, 1))
    st, name = _plan(d)
    assert st == 0 and name.startswith("attn_tf32x3_sm100") and name.endswith("+mask>"), name
    d = _with_mask(_attn(Lq=64, Lk=77, D=40, dtype=0), (0, 0, 77, 1))
    assert _plan(d)[0] == N.ERR_MISALIGNED
    d = _with_mask(_attn(Lq=64, Lk=77, D=40, dtype=0), (0, 0, 80, 1))
    d.mask_kind = 1
    st, name = _plan(d)
    assert st == 0 and name.endswith("+addmask>"), name
    assert N.lib.cmpx_attn_workspace_size(ctypes.byref(d)) == 0   # no packing for fp32
    # one query row: its row stride is never stepped and need not be aligned
    d = _with_mask(_attn(B=1, H=1, Lq=1, Lk=200, D=40, dtype=0), (200, 200, 200, 1))
    assert _plan(d)[0] == 0


def test_workspace_contract():
    assert N.lib.cmpx_attn_workspace_size(ctypes.byref(_attn(dtype=2))) == 256
    assert N.lib.cmpx_attn_workspace_size(ctypes.byref(_attn(dtype=1))) == 256
    # fp32: no split here, but two 128-row items per head share split K / V^T operands
    assert N.lib.cmpx_attn_workspace_size(ctypes.byref(_attn(dtype=0))) == 1024 + 4 * 2 * 256 * 128 * 4
    assert N.lib.cmpx_attn_workspace_size(ctypes.byref(_attn(Lq=128, dtype=0))) == 0  # one item per head
    assert N.lib.cmpx_attn_workspace_size(None) == 0
    d = _attn(dtype=2)  # valid shape, no workspace: rejected before any device work
    assert N.lib.cmpx_attn_fwd(ctypes.byref(d), None) == N.ERR_WORKSPACE
    d.workspace, d.workspace_bytes = 0x10000, 8  # too small
    assert N.lib.cmpx_attn_fwd(ctypes.byref(d), None) == N.ERR_WORKSPACE
    d.workspace, d.workspace_bytes = 0x10004, 256  # misaligned
    assert N.lib.cmpx_attn_fwd(ctypes.byref(d), None) == N.ERR_WORKSPACE


def _split_bytes(items, n_kv, dp, sms=148):
    """Workspace of the tail split: work counters, then per range (m, l) and fp32 O for 256 rows."""
    rem = items % sms
    per_range = 8 if items < sms else 4  # every item cut: at least 8 key tiles a range; else 4
    split = min(sms // rem, n_kv // per_range, 8) if rem and n_kv >= 16 else 1  # items of < 16 tiles: never
    if split < 2:
        return 256
    ranges = rem * split
    up = lambda x: (x + 255) // 256 * 256
    return 256 + up(ranges * 256 * 2 * 4) + ranges * 256 * dp * 4


@pytest.mark.parametrize("cfg", [
    dict(B=2, H=10, Lq=4096, Lk=4096, D=64, dtype=1),    # SD1.5 self-attention: 320 items, 24 split 6 ways
    dict(B=1, H=1, Lq=512, Lk=4096, D=128, dtype=2),    # 2 items, 4 ranges of 8 key tiles each
    dict(B=1, H=2, Lq=1024, Lk=2048, D=96, dtype=2),    # padded head dim: fp32 rows of 128
])
def test_workspace_size_covers_the_tail_split(cfg):
    d = _attn(**cfg)
    items = (cfg["Lq"] + 255) // 256 * cfg["H"] * cfg["B"]
    want = _split_bytes(items, (cfg["Lk"] + 127) // 128, 64 if cfg["D"] <= 64 else 128)
    assert want > 256
    # (no device here: the size is computed for a 148-SM B200)
    assert N.lib.cmpx_attn_workspace_size(ctypes.byref(d)) == want


@pytest.mark.parametrize("cfg", [
    dict(B=4, H=32, Lq=8192, Lk=8192, D=128, dtype=2, causal=1),  # causal: never split
    dict(B=2, H=10, Lq=4096, Lk=77, D=64, dtype=1),               # short keys: its own kernel
    dict(B=1, H=2, Lq=256, Lk=256, D=128, dtype=2),               # too few key tiles to split
    dict(B=1, H=148, Lq=256, Lk=4096, D=64, dtype=1),             # full waves only
    dict(B=2, H=8, Lq=1024, Lk=1024, D=80, dtype=1),              # 64 items < SMs, 8 key tiles: not cut
    dict(B=4, H=40, Lq=1024, Lk=1024, D=64, dtype=1),             # 640 items, tail of 48, 8 key tiles: not cut
])
def test_workspace_size_without_split(cfg):
    assert N.lib.cmpx_attn_workspace_size(ctypes.byref(_attn(**cfg))) == 256


def _f32_split_bytes(items, tiles, dp, sms=148):
    """fp32 tail split: 256 bytes of 8-bit item counters, then per key range 128 rows of
    (O [dp], m, l, 2 pad) fp32.  Fewer items than SMs: every item cut, ranges of >= 8 key tiles."""
    if 0 < items < sms:
        split = min(sms // items, 8, tiles // 8)
        return 256 + items * split * 128 * (dp + 4) * 4 if split >= 2 else 0
    rem = items % sms
    if rem == 0 or 2 * rem > sms:
        return 0
    split = min(sms // rem, 8, tiles // 4)  # at least 4 key tiles per range
    return 256 + rem * split * 128 * (dp + 4) * 4 if split >= 2 else 0


def _f32_workspace(cfg, split_bytes, dp):
    """The split's bytes, then (when every (b, h) has two or more 128-row items and an item reads
    four or more key tiles) K hi / lo and V^T hi / lo, fp32, B * H * lk_pad * dp each, from the
    next 1024-byte boundary."""
    bn = 64 if dp == 64 else 32
    if (cfg["Lq"] + 127) // 128 < 2 or (cfg["Lk"] + bn - 1) // bn < 4:
        return split_bytes
    lk_pad = (cfg["Lk"] + 63) // 64 * 64
    off = (max(256, split_bytes) + 1023) // 1024 * 1024
    return off + 4 * cfg["B"] * cfg["H"] * lk_pad * dp * 4


@pytest.mark.parametrize("cfg,split", [
    (dict(B=2, H=8, Lq=4096, Lk=4096, D=40, dtype=0), True),     # C1: 512 items, 68 cut 2 ways
    (dict(B=1, H=150, Lq=128, Lk=4096, D=64, dtype=0), True),    # 2 tail items cut 8 ways
    (dict(B=1, H=75, Lq=512, Lk=1024, D=128, dtype=0), True),    # D = 128, 32-key tiles
    (dict(B=2, H=8, Lq=4096, Lk=4096, D=40, dtype=0, causal=1), False),  # causal: never split
    (dict(B=1, H=248, Lq=128, Lk=4096, D=64, dtype=0), False),   # 100 tail items: more than half a wave
    (dict(B=1, H=148, Lq=256, Lk=4096, D=64, dtype=0), False),   # full waves only
    (dict(B=2, H=8, Lq=4096, Lk=77, D=40, dtype=0), False),      # 2 key tiles per item: no split, no pre-pass
    (dict(B=2, H=8, Lq=1024, Lk=77, D=80, dtype=0), False),      # 3 key tiles of 32: neither
    (dict(B=1, H=218, Lq=128, Lk=256, D=64, dtype=0), False),    # 4 key tiles: pre-pass not used (1 row tile), no split
    (dict(B=2, H=8, Lq=128, Lk=8192, D=64, dtype=0), True),      # 16 items < SMs: every item cut 8 ways
    (dict(B=1, H=8, Lq=256, Lk=4096, D=128, dtype=0), True),     # 16 items, 32-key tiles: cut 8 ways
    (dict(B=2, H=8, Lq=1024, Lk=512, D=64, dtype=0), False),     # 128 items < SMs but 8 key tiles: 1 range each
])
def test_fp32_workspace_covers_its_tail_split(cfg, split):
    d = _attn(**cfg)
    dp = 64 if cfg["D"] <= 64 else 128
    items = (cfg["Lq"] + 127) // 128 * cfg["H"] * cfg["B"]
    sb = 0 if cfg.get("causal") else _f32_split_bytes(
        items, (cfg["Lk"] + (63 if dp == 64 else 31)) // (64 if dp == 64 else 32), dp)
    assert (sb > 0) == split
    assert N.lib.cmpx_attn_workspace_size(ctypes.byref(d)) == _f32_workspace(cfg, sb, dp)
    st, name = _plan(d)
    assert st == 0 and name.endswith("+tail-split>") == split, name


@pytest.mark.skipif(__import__("torch").cuda.is_available(),
                    reason="fake pointers: on a GPU host this call would launch a kernel")
def test_minimum_workspace_is_accepted_for_split_shapes():
    # 256 bytes is enough for any 16-bit call (it then runs unsplit): the call gets past the
    # workspace check and stops at the device lookup on this GPU-less host.
    d = _attn(B=2, H=10, Lq=4096, Lk=4096, D=64, dtype=1)
    d.workspace, d.workspace_bytes = 0x10000, 256
    assert N.lib.cmpx_attn_fwd(ctypes.byref(d), None) == N.ERR_DEVICE


def _gqa(B, H, Hkv, Lq, Lk, D, dtype=2, causal=0, blhd_out=False):
    d = _attn(B=B, H=H, Lq=Lq, Lk=Lk, D=D, dtype=dtype, causal=causal)
    d.k_stride[:] = (Hkv * Lk * D, Lk * D, D)
    d.v_stride[:] = (Hkv * Lk * D, Lk * D, D)
    if blhd_out:  # the binding's [B, L, H, D] output layout
        d.o_stride[:] = (Lq * H * D, D, H * D)
    d.heads_kv = Hkv
    return d


def test_one_row_grouped_query_calls_are_folded():
    # decode [8, 32, 1, 4096, 128] with 8 key/value heads: the 4 query heads of a key/value head
    # run as one head of 4 rows -- 64 items of 32 key tiles, which (fewer items than SMs) are cut
    # into 2 ranges of 16 tiles; unfolded, 256 one-row items would not be split at all
    for blhd in (False, True):  # one query row: any row stride folds
        d = _gqa(8, 32, 8, 1, 4096, 128, blhd_out=blhd)
        st, name = _plan(d)
        assert st == 0 and name.endswith("+tail-split>"), name
        ranges = 64 * 2
        up = lambda x: (x + 255) // 256 * 256  # noqa: E731
        assert N.lib.cmpx_attn_workspace_size(ctypes.byref(d)) == 256 + up(ranges * 256 * 2 * 4) + ranges * 256 * 128 * 4
    # not folded: causal, several rows in a [B, L, H, D] output, equal head counts
    for d in (_gqa(8, 32, 8, 1, 4096, 128, causal=1), _gqa(8, 32, 8, 3, 4096, 128, blhd_out=True),
              _gqa(8, 32, 32, 1, 4096, 128)):
        st, name = _plan(d)
        assert st == 0 and not name.endswith("+tail-split>"), name
