"""Which real models' attention and matmul calls the library serves natively, decided on the CPU
from the C ABI's plan entry points (the tile table is a fixed function of the shape, so no GPU is
needed to know whether a call would run a kernel of this library or be declined to stock torch).

Every shape below must plan to one of this library's kernels.  The list covers common real model
shapes -- diffusion UNets (SD1.5 / SDXL self- and cross-attention, every head dim of their blocks),
a ViT, LLaMA-style language models with grouped-query heads, prefill and decode -- in the dtypes those
models run in, plus the einsum-attention chain and the small-matrix bmm regime.  A shape that starts
to plan "none" is a regression: the call would silently go back to stock torch.
"""
from __future__ import annotations

import ctypes
import math

import pytest

from cmpext3 import _native as N

F32, F16, BF16 = 0, 1, 2


def _attn(B, H, Lq, Lk, D, dtype, causal=0, heads_kv=0):
    d = N.AttnDesc()
    d.q = d.k = d.v = d.o = 0x10000
    d.batch, d.heads, d.len_q, d.len_k, d.head_dim = B, H, Lq, Lk, D
    hk = heads_kv or H
    d.q_stride[:] = (H * Lq * D, Lq * D, D)
    d.o_stride[:] = (H * Lq * D, Lq * D, D)
    d.k_stride[:] = (hk * Lk * D, Lk * D, D)
    d.v_stride[:] = (hk * Lk * D, Lk * D, D)
    d.dtype, d.causal, d.heads_kv = dtype, causal, heads_kv
    d.scale = 1 / math.sqrt(D)
    return d


def _plan_attn(d):
    buf = ctypes.create_string_buffer(128)
    st = N.lib.cmpx_attn_plan(ctypes.byref(d), buf, 128)
    return st, buf.value.decode()


ATTENTION = [
    # model, (B, H, Lq, Lk, D), dtype, causal, heads_kv
    ("SD1.5 self 64x64 latents", (2, 8, 4096, 4096, 40), F16, 0, 0),
    ("SD1.5 self, fp32", (2, 8, 4096, 4096, 40), F32, 0, 0),
    ("SD1.5 cross (77 text tokens)", (2, 8, 4096, 77, 40), F16, 0, 0),
    ("SD1.5 cross, fp32", (2, 8, 4096, 77, 40), F32, 0, 0),
    ("SD1.5 mid block (D = 160)", (2, 8, 64, 64, 160), F16, 0, 0),
    ("SD1.5 down block 2 (D = 80)", (2, 8, 1024, 1024, 80), F16, 0, 0),
    ("SD1.5 down block 2, fp32 (D = 80)", (2, 8, 1024, 1024, 80), F32, 0, 0),
    ("SDXL self", (2, 10, 4096, 4096, 64), F16, 0, 0),
    ("SDXL cross", (2, 10, 4096, 77, 64), F16, 0, 0),
    ("SDXL self, 32x32 block", (2, 20, 1024, 1024, 64), BF16, 0, 0),
    ("LLaMA-2 7B prefill", (1, 32, 4096, 4096, 128), BF16, 1, 0),
    ("LLaMA-3 8B prefill (GQA 32/8)", (1, 32, 8192, 8192, 128), BF16, 1, 8),
    ("Mistral 7B prefill (GQA 32/8)", (4, 32, 2048, 2048, 128), F16, 1, 8),
    ("decode step (one query row, 4096 keys)", (8, 32, 1, 4096, 128), BF16, 0, 8),
    ("ViT-L/14 (257 tokens, D = 64)", (32, 16, 257, 257, 64), F16, 0, 0),
    ("fp32 LLaMA-style (D = 128, causal)", (1, 32, 2048, 2048, 128), F32, 1, 0),
]


@pytest.mark.parametrize("name,shape,dtype,causal,heads_kv", ATTENTION, ids=[a[0] for a in ATTENTION])
def test_model_attention_shapes_run_natively(name, shape, dtype, causal, heads_kv):
    st, entry = _plan_attn(_attn(*shape, dtype, causal, heads_kv))
    assert st == 0 and entry != "none", (name, st, entry)


def _bmm(nb, m, k, n, dtype, b_kmajor):
    d = N.BmmDesc()
    d.a = d.b = d.c = 0x10000
    d.batch, d.m, d.n, d.k = nb, m, n, k
    d.a_stride[:] = (m * k, k, 1)
    d.b_stride[:] = (k * n, 1, k) if b_kmajor else (k * n, n, 1)
    d.c_stride[:] = (m * n, n, 1)
    d.dtype = dtype
    return d


def _plan_bmm(d, fn):
    buf = ctypes.create_string_buffer(128)
    st = fn(ctypes.byref(d), buf, 128)
    return st, buf.value.decode()


GEMM = [
    # model, (batch, m, k, n), dtype, B contiguous along k (a transposed view)
    ("einsum-attention scores (C3)", (64, 2048, 64, 2048), BF16, True),
    ("einsum-attention values (C3)", (64, 2048, 2048, 64), BF16, False),
    ("einsum-attention scores, fp32", (64, 2048, 64, 2048), F32, True),
    ("LLaMA-7B MLP up (as bmm)", (1, 4096, 4096, 11008), BF16, True),
    ("fp32 GEMM, K = 16384", (1, 1024, 16384, 1024), F32, True),
    ("fp16 batched heads", (128, 512, 64, 512), F16, False),
]


@pytest.mark.parametrize("name,shape,dtype,bk", GEMM, ids=[g[0] for g in GEMM])
def test_model_gemm_shapes_run_natively(name, shape, dtype, bk):
    st, entry = _plan_bmm(_bmm(*shape, dtype, bk), N.lib.cmpx_bmm_plan)
    assert st == 0 and entry != "none", (name, st, entry)


SMALL = [
    ("FEM element blocks (reference's example)", (20000, 24, 24, 3), F32),
    ("tiny heads", (4096, 16, 8, 16), F16),
    ("3x3 rotations", (100000, 3, 3, 3), BF16),
]


@pytest.mark.parametrize("name,shape,dtype", SMALL, ids=[s[0] for s in SMALL])
def test_small_products_run_natively(name, shape, dtype):
    nb, m, k, n = shape
    assert m * k * n <= 32768  # the reference's small-matrix route
    st, entry = _plan_bmm(_bmm(nb, m, k, n, dtype, False), N.lib.cmpx_bmm_small_plan)
    assert st == 0 and entry.startswith("bmm_small<"), (name, st, entry)
