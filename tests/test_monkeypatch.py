"""Dispatch logic of the monkeypatch layer (CPU only; native ops replaced by MagicMocks).

Mirrors the reference's tests for the path's ops (tests/test_cmpext3_monkeypatch.py there:
TestGradSafe :31, TestUsable :56, TestEnableDisable :93-186, TestMatmul :245-305, TestBmm :313-356,
TestScaledDotProductAttention :858-925, TestAutoselect :476-649) against this package's wrappers.
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import cmpext3
from conftest import STOCK_SOFTMAX, STOCK_UNPATCHED, force_eligible


def assert_called_once_with_tensors(mock_fn, *expected_args, **expected_kwargs):
    assert mock_fn.call_count == 1, f"expected 1 call, got {mock_fn.call_count}"
    got_args, got_kwargs = mock_fn.call_args
    assert len(got_args) == len(expected_args)
    for got, want in zip(got_args, expected_args):
        if isinstance(want, torch.Tensor):
            assert isinstance(got, torch.Tensor) and torch.equal(got, want)
        else:
            assert got == want, f"arg mismatch: got {got!r} want {want!r}"
    assert got_kwargs == expected_kwargs


class TestGradSafe:
    def test_true_when_grad_disabled(self):
        x = torch.randn(2, requires_grad=True)
        with torch.no_grad():
            assert cmpext3._grad_safe(x) is True

    def test_true_in_inference_mode(self):
        x = torch.randn(2, requires_grad=True)
        with torch.inference_mode():
            assert cmpext3._grad_safe(x) is True

    def test_false_when_any_tensor_requires_grad(self):
        assert cmpext3._grad_safe(torch.randn(2), torch.randn(2, requires_grad=True)) is False

    def test_true_when_no_tensor_requires_grad(self):
        assert cmpext3._grad_safe(torch.randn(2), torch.randn(2)) is True

    def test_non_tensor_args_are_ignored(self):
        assert cmpext3._grad_safe(1, "x", None) is True


class TestUsable:
    def test_true_for_non_tensor_args(self):
        assert cmpext3._usable(1, "x", None) is True

    def test_false_for_cpu_tensor(self):
        assert cmpext3._usable(torch.randn(2)) is False

    @pytest.mark.parametrize("dtype,ok", [(torch.int64, False), (torch.float64, False),
                                          (torch.float16, True), (torch.float32, True),
                                          (torch.bfloat16, True)])
    def test_dtype_gate_on_fake_cuda_tensor(self, monkeypatch, dtype, ok):
        x = torch.zeros(2, dtype=dtype)
        monkeypatch.setattr(torch.Tensor, "is_cuda", property(lambda self: True))
        assert cmpext3._usable(x) is ok


class TestEnableDisable:
    def test_enable_installs_expected_targets(self, patched):
        assert cmpext3.is_enabled() is True
        assert torch.matmul is cmpext3._patched_matmul
        assert torch.bmm is cmpext3._patched_bmm
        assert torch.einsum is cmpext3._patched_einsum
        assert F.scaled_dot_product_attention is cmpext3._patched_sdpa
        assert F.linear is cmpext3._patched_linear

    def test_disable_ops_pins_named_ops_to_stock(self, monkeypatch):
        assert not cmpext3.is_enabled()
        monkeypatch.setattr(cmpext3, "_DISABLED_OPS", frozenset({"attention", "einsum"}))
        stock_sdpa, stock_einsum = F.scaled_dot_product_attention, torch.einsum
        cmpext3.enable()
        try:
            assert F.scaled_dot_product_attention is stock_sdpa
            assert torch.einsum is stock_einsum
            assert torch.bmm is cmpext3._patched_bmm
        finally:
            cmpext3.disable()

    def test_disable_restores_original_callables(self, patched):
        orig_bmm = cmpext3._ORIGINALS[(torch, "bmm")]
        orig_sdpa = cmpext3._ORIGINALS[(F, "scaled_dot_product_attention")]
        cmpext3.disable()
        assert torch.bmm is orig_bmm
        assert F.scaled_dot_product_attention is orig_sdpa
        assert cmpext3.is_enabled() is False
        cmpext3.enable()

    def test_enable_is_idempotent(self, patched):
        first = cmpext3._ORIGINALS[(torch, "bmm")]
        cmpext3.enable()
        assert cmpext3._ORIGINALS[(torch, "bmm")] is first
        assert torch.bmm is cmpext3._patched_bmm

    def test_disable_without_enable_is_noop(self):
        assert cmpext3.is_enabled() is False
        cmpext3.disable()
        assert cmpext3.is_enabled() is False

    def test_ops_alias_is_native_module(self, native):
        assert cmpext3.ops is native

    def test_real_ops_module_is_the_ctypes_binding(self):
        from cmpext3 import _native
        assert cmpext3.ops is _native or cmpext3._C is _native
        assert callable(_native.attention) and callable(_native.bmm)

    def test_deliberately_unpatched_ops_untouched(self, patched):
        for (target, name), stock_fn in STOCK_UNPATCHED.items():
            assert getattr(target, name) is stock_fn, f"{name} was patched"

    def test_scripted_code_still_compiles_against_patched_bmm(self, patched):
        @torch.jit.script
        def f(a, b):
            return torch.bmm(a, b)
        a, b = torch.randn(2, 3, 4), torch.randn(2, 4, 5)
        assert torch.allclose(f(a, b), cmpext3._ORIGINALS[(torch, "bmm")](a, b))


class TestMatmul:
    def test_2d_calls_native_bmm_unsqueezed(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        a, b = torch.randn(64, 128), torch.randn(128, 256)
        native.bmm.return_value = torch.zeros(1, 64, 256)
        got = torch.matmul(a, b)
        assert_called_once_with_tensors(native.bmm, a.unsqueeze(0), b.unsqueeze(0))
        assert got.shape == (64, 256)

    def test_3d_calls_native_bmm_directly(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        a, b = torch.randn(2, 64, 128), torch.randn(2, 128, 256)
        sentinel = torch.zeros(2, 64, 256)
        native.bmm.return_value = sentinel
        assert torch.matmul(a, b) is sentinel
        assert_called_once_with_tensors(native.bmm, a, b)

    def test_small_3d_takes_the_small_matrix_kernel(self, patched, native, monkeypatch):
        # M*K*N <= 32768 per item: the reference's small-matrix route (its __init__.py:440-464),
        # here the native small-matrix kernel rather than the tiled GEMM
        force_eligible(monkeypatch)
        a, b = torch.randn(2, 3, 4), torch.randn(2, 4, 5)
        sentinel = torch.zeros(2, 3, 5)
        native.bmm_small.return_value = sentinel
        assert torch.matmul(a, b) is sentinel
        native.bmm.assert_not_called()
        assert_called_once_with_tensors(native.bmm_small, a, b)

    def test_small_route_threshold(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        monkeypatch.setattr(cmpext3, "_SMALL_BMM_MAX_MKN", 59)
        a, b = torch.randn(2, 3, 4), torch.randn(2, 4, 5)  # M*K*N = 60 > 59: the tiled GEMM
        native.bmm.return_value = torch.zeros(2, 3, 5)
        torch.bmm(a, b)
        native.bmm_small.assert_not_called()
        assert native.bmm.call_count == 1

    def test_falls_back_when_not_cuda(self, patched, native):
        a, b = torch.randn(2, 3), torch.randn(3, 4)
        got = torch.matmul(a, b)
        native.bmm.assert_not_called()
        assert torch.equal(got, cmpext3._ORIGINALS[(torch, "matmul")](a, b))

    def test_falls_back_on_dtype_mismatch(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        with pytest.raises(RuntimeError):
            torch.matmul(torch.randn(2, 3), torch.randn(3, 4, dtype=torch.float16))
        native.bmm.assert_not_called()

    def test_falls_back_on_unsupported_ndim(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        a, b = torch.randn(4), torch.randn(4)
        got = torch.matmul(a, b)
        native.bmm.assert_not_called()
        assert torch.equal(got, cmpext3._ORIGINALS[(torch, "matmul")](a, b))

    def test_respects_out_kwarg(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        a, b = torch.randn(2, 3), torch.randn(3, 4)
        out, expected = torch.empty(2, 4), torch.empty(2, 4)
        torch.matmul(a, b, out=out)
        cmpext3._ORIGINALS[(torch, "matmul")](a, b, out=expected)
        native.bmm.assert_not_called()
        assert torch.equal(out, expected)

    def test_falls_back_on_native_runtime_error(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        native.bmm.side_effect = RuntimeError("boom")
        a, b = torch.randn(2, 64, 128), torch.randn(2, 128, 64)
        got = torch.matmul(a, b)
        native.bmm.assert_called_once()
        assert torch.equal(got, cmpext3._ORIGINALS[(torch, "matmul")](a, b))


class TestBmm:
    def test_calls_native_when_eligible(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        a, b = torch.randn(2, 64, 128), torch.randn(2, 128, 256)
        sentinel = torch.zeros(2, 64, 256)
        native.bmm.return_value = sentinel
        assert torch.bmm(a, b) is sentinel
        assert_called_once_with_tensors(native.bmm, a, b)

    def test_transposed_view_reaches_native_uncopied(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        a = torch.randn(2, 64, 128)
        kt = torch.randn(2, 256, 128).transpose(1, 2)  # [2, 128, 256] view, K-contiguous
        native.bmm.return_value = torch.zeros(2, 64, 256)
        torch.bmm(a, kt)
        got_b = native.bmm.call_args[0][1]
        assert got_b.data_ptr() == kt.data_ptr() and got_b.stride() == kt.stride()

    def test_falls_back_when_not_cuda(self, patched, native):
        a, b = torch.randn(2, 3, 4), torch.randn(2, 4, 5)
        got = torch.bmm(a, b)
        native.bmm.assert_not_called()
        assert torch.equal(got, cmpext3._ORIGINALS[(torch, "bmm")](a, b))

    def test_falls_back_on_dtype_mismatch(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        with pytest.raises(RuntimeError):
            torch.bmm(torch.randn(2, 3, 4), torch.randn(2, 4, 5, dtype=torch.float16))
        native.bmm.assert_not_called()

    def test_respects_out_kwarg(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        a, b = torch.randn(2, 3, 4), torch.randn(2, 4, 5)
        out, expected = torch.empty(2, 3, 5), torch.empty(2, 3, 5)
        torch.bmm(a, b, out=out)
        cmpext3._ORIGINALS[(torch, "bmm")](a, b, out=expected)
        native.bmm.assert_not_called()
        assert torch.equal(out, expected)

    def test_falls_back_on_native_runtime_error(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        native.bmm.side_effect = RuntimeError("boom")
        a, b = torch.randn(2, 64, 128), torch.randn(2, 128, 64)
        got = torch.bmm(a, b)
        native.bmm.assert_called_once()
        assert torch.equal(got, cmpext3._ORIGINALS[(torch, "bmm")](a, b))

    def test_autograd_live_goes_to_stock(self, patched, native, monkeypatch):
        monkeypatch.setattr(cmpext3, "_usable", lambda *a, **k: True)
        a = torch.randn(2, 64, 128, requires_grad=True)
        b = torch.randn(2, 128, 64)
        torch.bmm(a, b)
        native.bmm.assert_not_called()


class TestLinear:
    """The reference's gates for F.linear (cmpext3/__init__.py:410-420)."""

    def test_calls_native_when_eligible(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        x, w, b = torch.randn(4, 16, 64), torch.randn(32, 64), torch.randn(32)
        sentinel = torch.zeros(4, 16, 32)
        native.linear.return_value = sentinel
        assert F.linear(x, w, b) is sentinel
        args = native.linear.call_args[0]
        assert args[0] is x and args[1] is w and args[2] is b

    def test_nn_linear_module_reaches_native(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        layer = torch.nn.Linear(64, 32)
        native.linear.return_value = torch.zeros(8, 32)
        with torch.no_grad():
            layer(torch.randn(8, 64))
        native.linear.assert_called_once()

    def test_falls_back_when_not_cuda(self, patched, native):
        x, w = torch.randn(3, 8), torch.randn(5, 8)
        got = F.linear(x, w)
        native.linear.assert_not_called()
        assert torch.equal(got, cmpext3._ORIGINALS[(F, "linear")](x, w))

    def test_fp16_odd_out_features_goes_to_stock(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        x, w = torch.randn(4, 8).half(), torch.randn(5, 8).half()
        F.linear(x, w)
        native.linear.assert_not_called()

    def test_1d_input_or_3d_weight_goes_to_stock(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        F.linear(torch.randn(8), torch.randn(4, 8))
        with pytest.raises(RuntimeError):
            F.linear(torch.randn(2, 8), torch.randn(1, 4, 8))
        native.linear.assert_not_called()

    def test_autograd_live_goes_to_stock(self, patched, native, monkeypatch):
        monkeypatch.setattr(cmpext3, "_usable", lambda *a, **k: True)
        layer = torch.nn.Linear(8, 4)  # its weight requires grad
        layer(torch.randn(2, 8))
        native.linear.assert_not_called()

    def test_falls_back_on_native_runtime_error(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        native.linear.side_effect = RuntimeError("linear: input/weight must share one dtype among float16/bfloat16")
        x, w, b = torch.randn(4, 8), torch.randn(6, 8), torch.randn(6)
        got = F.linear(x, w, b)
        native.linear.assert_called_once()
        assert torch.equal(got, cmpext3._ORIGINALS[(F, "linear")](x, w, b))

    def test_disable_ops_linear_pins_stock(self, monkeypatch):
        monkeypatch.setattr(cmpext3, "_DISABLED_OPS", frozenset({"linear"}))
        stock = F.linear
        cmpext3.enable()
        try:
            assert F.linear is stock
        finally:
            cmpext3.disable()


class TestSoftmax:
    """softmax is diverted only for the last dimension of a tensor a patched einsum / bmm / matmul
    returned (the middle step of an attention chain); every other softmax runs stock."""

    CALLS = {
        "torch": lambda x, **kw: torch.softmax(x, -1, **kw),
        "F": lambda x, **kw: F.softmax(x, dim=-1, **kw),
        "Tensor": lambda x, **kw: x.softmax(-1, **kw),
    }

    @pytest.mark.parametrize("form", ["torch", "F", "Tensor"])
    def test_softmax_of_einsum_scores_routes_to_native(self, patched, native, monkeypatch, form):
        force_eligible(monkeypatch)
        q, k = torch.randn(1, 2, 64, 32), torch.randn(1, 2, 96, 32)
        native.bmm.return_value = torch.zeros(2, 64, 96)
        s = torch.einsum("bhid,bhjd->bhij", q, k)
        native.softmax.return_value = torch.ones(1, 2, 64, 96)
        got = self.CALLS[form](s)
        native.softmax.assert_called_once()
        assert native.softmax.call_args[0][0] is s and native.softmax.call_args[0][1] == -1
        assert torch.equal(got, torch.ones(1, 2, 64, 96))

    @pytest.mark.parametrize("form", ["torch", "F", "Tensor"])
    def test_softmax_of_any_other_tensor_is_stock(self, patched, native, monkeypatch, form):
        force_eligible(monkeypatch)
        x = torch.randn(3, 5, 7)
        got = self.CALLS[form](x)
        native.softmax.assert_not_called()
        assert torch.equal(got, STOCK_SOFTMAX["torch"](x, -1))

    def test_other_dim_or_dtype_is_stock(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        native.bmm.return_value = torch.randn(2, 64, 64)  # M*K*N above the small-matrix route
        s = torch.bmm(torch.randn(2, 64, 32), torch.randn(2, 32, 64))
        torch.softmax(s, 1)
        torch.softmax(s, -1, dtype=torch.float64)
        F.softmax(s)  # implicit dim: stock (with torch's warning)
        native.softmax.assert_not_called()

    @pytest.fixture
    def fused(self, monkeypatch):
        monkeypatch.setattr(cmpext3, "_FUSED_SOFTMAX", True)

    def test_fused_softmax_is_off_by_default(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        native.bmm.side_effect = lambda a, b: torch.zeros(a.shape[0], a.shape[1], b.shape[2], dtype=a.dtype)
        bf = torch.bfloat16
        s = torch.einsum("bhid,bhjd->bhij", torch.randn(1, 2, 64, 32).to(bf), torch.randn(1, 2, 256, 32).to(bf))
        native.softmax.return_value = torch.ones(1, 2, 64, 256, dtype=bf)
        torch.softmax(s, -1)
        native.bmm_rowstats.assert_not_called()
        native.softmax_product.assert_not_called()
        assert native.bmm.call_count == 1 and native.softmax.call_count == 1

    def _bf16_scores(self, native):
        # einsum scores of 16-bit q, k with a 32-wide head dim and 256 keys: the planner's bmm
        # operands are contiguous along the head dim, so the product is computed with its row
        # statistics and its operands are recorded
        q = torch.randn(1, 2, 64, 32).to(torch.bfloat16)
        k = torch.randn(1, 2, 256, 32).to(torch.bfloat16)
        self.stats = []

        def rowstats(a, b):
            st = torch.zeros(a.shape[0], (b.shape[2] + 63) // 64, a.shape[1], 2)
            self.stats.append(st)
            return torch.zeros(a.shape[0], a.shape[1], b.shape[2], dtype=a.dtype), st
        native.bmm_rowstats.side_effect = rowstats
        return q, k, torch.einsum("bhid,bhjd->bhij", q, k)

    def test_softmax_of_recorded_scores_recomputes_them_from_the_operands(self, patched, native, monkeypatch, fused):
        force_eligible(monkeypatch)
        q, k, s = self._bf16_scores(native)
        native.bmm.assert_not_called()
        assert native.bmm_rowstats.call_count == 1
        native.softmax_product.return_value = torch.full((2, 64, 256), 0.5, dtype=torch.bfloat16)
        got = torch.softmax(s, -1)
        native.softmax.assert_not_called()
        assert native.softmax_product.call_count == 1
        a, b, stats = native.softmax_product.call_args[0]
        assert torch.equal(a, q.reshape(2, 64, 32)) and torch.equal(b, k.reshape(2, 256, 32).transpose(1, 2))
        assert stats is self.stats[0]  # the statistics the scores product returned
        assert got.shape == s.shape and "softmax_product" in cmpext3.autoselect_report()

    def test_scores_changed_in_place_are_read_not_recomputed(self, patched, native, monkeypatch, fused):
        force_eligible(monkeypatch)
        _, _, s = self._bf16_scores(native)
        s.mul_(2)  # the recorded operands no longer describe s
        native.softmax.return_value = torch.ones(1, 2, 64, 256, dtype=torch.bfloat16)
        torch.softmax(s, -1)
        native.softmax_product.assert_not_called()
        assert native.softmax.call_count == 1

    def test_operand_changed_in_place_is_not_recomputed(self, patched, native, monkeypatch, fused):
        force_eligible(monkeypatch)
        q, _, s = self._bf16_scores(native)
        q.add_(1)
        native.softmax.return_value = torch.ones(1, 2, 64, 256, dtype=torch.bfloat16)
        torch.softmax(s, -1)
        native.softmax_product.assert_not_called()

    def test_only_attention_shaped_products_carry_row_statistics(self, patched, native, monkeypatch, fused):
        force_eligible(monkeypatch)
        native.bmm.side_effect = lambda a, b: torch.zeros(a.shape[0], a.shape[1], b.shape[2], dtype=a.dtype)
        native.bmm_rowstats.side_effect = lambda a, b: (
            torch.zeros(a.shape[0], a.shape[1], b.shape[2], dtype=a.dtype),
            torch.zeros(a.shape[0], (b.shape[2] + 63) // 64, a.shape[1], 2))
        bf = torch.bfloat16
        torch.bmm(torch.randn(2, 64, 64).to(bf), torch.randn(2, 256, 64).to(bf).transpose(1, 2))
        assert native.bmm_rowstats.call_count == 1 and native.bmm.call_count == 0
        torch.bmm(torch.randn(2, 64, 64), torch.randn(2, 256, 64).transpose(1, 2))  # fp32
        torch.bmm(torch.randn(2, 64, 256).to(bf), torch.randn(2, 256, 256).to(bf))  # k > 128
        torch.bmm(torch.randn(2, 64, 64).to(bf), torch.randn(2, 64, 256).to(bf))  # B contiguous along n
        torch.bmm(torch.randn(2, 64, 64).to(bf), torch.randn(2, 96, 64).to(bf).transpose(1, 2))  # n < 128
        assert native.bmm_rowstats.call_count == 1 and native.bmm.call_count == 4

    def test_declined_native_softmax_falls_back_to_stock(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        native.bmm.return_value = torch.randn(2, 64, 64)  # M*K*N above the small-matrix route
        s = torch.bmm(torch.randn(2, 64, 32), torch.randn(2, 32, 64))
        native.softmax.side_effect = RuntimeError("outside the tile table")
        got = torch.softmax(s, -1)
        assert torch.allclose(got, STOCK_SOFTMAX["torch"](s, -1))

    def test_einsum_softmax_einsum_chain(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q, k, v = torch.randn(1, 2, 64, 32), torch.randn(1, 2, 96, 32), torch.randn(1, 2, 96, 32)
        native.bmm.side_effect = lambda a, b: a @ b  # Tensor.__matmul__ is not patched
        native.softmax.side_effect = lambda x, dim: STOCK_SOFTMAX["torch"](x, dim)
        s = torch.einsum("bhid,bhjd->bhij", q, k)
        o = torch.einsum("bhij,bhjd->bhid", torch.softmax(s, dim=-1), v)
        assert native.bmm.call_count == 2 and native.softmax.call_count == 1
        ref = STOCK_SOFTMAX["torch"](q @ k.transpose(-1, -2), -1) @ v
        assert torch.allclose(o, ref, atol=1e-5)

    def test_disable_restores_every_softmax(self):
        cmpext3.enable()
        cmpext3.disable()
        assert torch.softmax is STOCK_SOFTMAX["torch"]
        assert F.softmax is STOCK_SOFTMAX["F"]
        assert torch.Tensor.softmax is STOCK_SOFTMAX["Tensor"]

    def test_dead_products_leave_the_registry(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        native.bmm.side_effect = lambda a, b: torch.zeros(a.shape[0], a.shape[1], b.shape[2])
        before = len(cmpext3._PRODUCED)
        for _ in range(50):
            torch.bmm(torch.randn(2, 3, 4), torch.randn(2, 4, 5))
        assert len(cmpext3._PRODUCED) <= before + 1


class TestEinsum:
    def test_attention_scores_equation_routes_to_native_bmm(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q, k = torch.randn(1, 2, 64, 32), torch.randn(1, 2, 96, 32)
        native.bmm.return_value = torch.zeros(2, 64, 96)
        got = torch.einsum("bhid,bhjd->bhij", q, k)
        native.bmm.assert_called_once()
        a, b = native.bmm.call_args[0]
        assert a.shape == (2, 64, 32) and b.shape == (2, 32, 96)
        assert b.stride(1) == 1, "K^T must reach bmm as a view (contiguous along the contraction)"
        assert got.shape == (1, 2, 64, 96)

    def test_unsupported_equation_goes_to_stock(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        x = torch.randn(4, 4)
        got = torch.einsum("ii->i", x)
        native.bmm.assert_not_called()
        assert torch.equal(got, torch.diagonal(x))

    def test_sublist_format_goes_to_stock(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        a, b = torch.randn(3, 4), torch.randn(4, 5)
        got = torch.einsum(a, [0, 1], b, [1, 2], [0, 2])
        native.bmm.assert_not_called()
        assert torch.allclose(got, a @ b)

    def test_mixed_dtypes_go_to_stock(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        with pytest.raises(RuntimeError):
            torch.einsum("ij,jk->ik", torch.randn(3, 4), torch.randn(4, 5, dtype=torch.float64))
        native.bmm.assert_not_called()

    def test_native_error_falls_back_to_stock_einsum(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        native.bmm.side_effect = RuntimeError("boom")
        a, b = torch.randn(2, 64, 128), torch.randn(2, 128, 64)
        got = torch.einsum("bij,bjk->bik", a, b)
        assert torch.allclose(got, cmpext3._ORIGINALS[(torch, "einsum")]("bij,bjk->bik", a, b))


class TestScaledDotProductAttention:
    def _qkv(self, *shape):
        return torch.randn(*shape), torch.randn(*shape), torch.randn(*shape)

    def test_calls_native_when_eligible(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q, k, v = self._qkv(1, 2, 3, 4)
        native.attention.return_value = "native-result"
        assert F.scaled_dot_product_attention(q, k, v) == "native-result"
        assert_called_once_with_tensors(native.attention, q, k, v, None, False)

    def test_calls_native_when_is_causal(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q, k, v = self._qkv(1, 2, 3, 4)
        native.attention.return_value = "native-result"
        assert F.scaled_dot_product_attention(q, k, v, is_causal=True) == "native-result"
        assert_called_once_with_tensors(native.attention, q, k, v, None, True)

    def test_passes_explicit_scale(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q, k, v = self._qkv(1, 2, 3, 4)
        native.attention.return_value = "native-result"
        F.scaled_dot_product_attention(q, k, v, scale=0.25)
        assert_called_once_with_tensors(native.attention, q, k, v, 0.25, False)

    def test_falls_back_when_float_attn_mask_of_another_dtype_given(self, patched, native, monkeypatch):
        # an additive mask runs natively only in the query's dtype; others stay stock (the
        # reference sent every masked call to stock)
        force_eligible(monkeypatch)
        q, k, v = (t.to(torch.bfloat16) for t in self._qkv(1, 2, 3, 4))
        F.scaled_dot_product_attention(q, k, v, attn_mask=torch.zeros(3, 3))  # fp32 mask, bf16 query
        native.attention.assert_not_called()

    def test_additive_attn_mask_in_the_query_dtype_runs_native(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q, k, v = self._qkv(1, 2, 3, 4)
        m = torch.zeros(3, 3)
        native.attention.return_value = torch.zeros(1, 2, 3, 4)
        F.scaled_dot_product_attention(q, k, v, attn_mask=m)
        assert native.attention.call_args[0][5] is m

    def test_boolean_attn_mask_runs_native(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q, k, v = self._qkv(1, 2, 3, 4)
        m = torch.ones(3, 3, dtype=torch.bool).tril()
        native.attention.return_value = torch.zeros(1, 2, 3, 4)
        F.scaled_dot_product_attention(q, k, v, attn_mask=m)
        args = native.attention.call_args[0]
        assert args[5] is m and args[4] is False

    def test_native_mask_error_falls_back_to_stock(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        native.attention.side_effect = RuntimeError("attn_mask does not broadcast")
        q, k, v = self._qkv(1, 2, 3, 4)
        m = torch.rand(3, 3) > 0.5
        got = F.scaled_dot_product_attention(q, k, v, attn_mask=m)
        ref = cmpext3._ORIGINALS[(F, "scaled_dot_product_attention")](q, k, v, attn_mask=m)
        assert torch.equal(got, ref)

    def test_falls_back_when_dropout_nonzero(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q, k, v = self._qkv(1, 2, 3, 4)
        F.scaled_dot_product_attention(q, k, v, dropout_p=0.1)
        native.attention.assert_not_called()

    def test_falls_back_on_non_4d_query(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q, k, v = self._qkv(2, 3, 4)
        F.scaled_dot_product_attention(q, k, v)
        native.attention.assert_not_called()

    def test_falls_back_when_not_cuda(self, patched, native):
        q, k, v = self._qkv(1, 2, 3, 4)
        got = F.scaled_dot_product_attention(q, k, v)
        native.attention.assert_not_called()
        want = cmpext3._ORIGINALS[(F, "scaled_dot_product_attention")](q, k, v)
        assert torch.equal(got, want)

    def test_falls_back_on_native_runtime_error(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        native.attention.side_effect = RuntimeError("boom")
        q, k, v = self._qkv(1, 2, 3, 4)
        got = F.scaled_dot_product_attention(q, k, v)
        native.attention.assert_called_once()
        assert got.shape == q.shape

    def test_gqa_heads_go_to_native(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q = torch.randn(1, 4, 3, 8)
        k, v = torch.randn(1, 2, 3, 8), torch.randn(1, 2, 3, 8)
        native.attention.return_value = torch.zeros(1, 4, 3, 8)
        got = F.scaled_dot_product_attention(q, k, v, enable_gqa=True)
        native.attention.assert_called_once()
        assert native.attention.call_args[0][1] is k and got.shape == q.shape

    def test_unequal_heads_without_enable_gqa_stay_stock(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q = torch.randn(1, 4, 3, 8)
        k, v = torch.randn(1, 2, 3, 8), torch.randn(1, 2, 3, 8)
        with pytest.raises(RuntimeError):  # torch's own shape error, as without the patch
            F.scaled_dot_product_attention(q, k, v)
        native.attention.assert_not_called()


class TestDispatchRecord:
    """The per-signature record that replaced the reference's runtime race (cmpext3.autoselect)."""

    def test_first_call_records_tile_entry(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        q, k, v = torch.randn(1, 2, 3, 4), torch.randn(1, 2, 3, 4), torch.randn(1, 2, 3, 4)
        native.attention.return_value = "native-result"
        F.scaled_dot_product_attention(q, k, v)
        (d,) = cmpext3.autoselect.report()
        assert d.use_native and d.entry == "fake-attention-entry"
        assert "fake-attention-entry" in cmpext3.autoselect_report()

    def test_kernel_that_raises_is_never_called_again(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        native.bmm.side_effect = RuntimeError("unsupported shape")
        a, b = torch.randn(2, 64, 128), torch.randn(2, 128, 64)
        for _ in range(3):
            torch.bmm(a, b)
        assert native.bmm.call_count == 1
        (d,) = cmpext3.autoselect.report()
        assert not d.use_native and "RuntimeError" in d.note

    def test_one_off_failure_does_not_overturn_a_good_decision(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        a, b = torch.randn(2, 64, 128), torch.randn(2, 128, 64)
        native.bmm.return_value = torch.zeros(2, 64, 64)
        torch.bmm(a, b)
        native.bmm.side_effect = RuntimeError("transient")
        got = torch.bmm(a, b)
        assert torch.equal(got, cmpext3._ORIGINALS[(torch, "bmm")](a, b))
        native.bmm.side_effect = None
        assert torch.equal(torch.bmm(a, b), torch.zeros(2, 64, 64))
        assert cmpext3.autoselect.report()[0].use_native

    def test_record_off_always_calls_kernel(self, patched, native, monkeypatch):
        force_eligible(monkeypatch)
        monkeypatch.setattr(cmpext3.autoselect, "_ENABLED", False)
        native.bmm.side_effect = RuntimeError("unsupported")
        a, b = torch.randn(2, 64, 128), torch.randn(2, 128, 64)
        torch.bmm(a, b)
        torch.bmm(a, b)
        assert native.bmm.call_count == 2
        assert cmpext3.autoselect.report() == []

    def test_record_is_capped_per_op(self, monkeypatch):
        monkeypatch.setattr(cmpext3.autoselect, "_MAX_SIGNATURES_PER_OP", 4)
        for i in range(10):
            cmpext3.autoselect.choose("op", ("k", i), lambda: 1, lambda: 0)
        assert len(cmpext3.autoselect.report()) == 4

    def test_mismatch_rule(self):
        from cmpext3.autoselect import _mismatch
        assert _mismatch(torch.ones(4) * (1 + 1e-6), torch.ones(4)) is None
        assert "exceeds" in _mismatch(torch.full((4,), 10.0), torch.zeros(4) + 1)
        assert "NaN" in _mismatch(torch.full((4,), float("nan")), torch.zeros(4))
        assert "shape" in _mismatch(torch.zeros(3), torch.zeros(4))
