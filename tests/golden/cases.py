"""Case list and seeded input generators shared by make_golden.py and the tests.

Inputs are regenerated from their seeds (torch.Generator on the CPU) instead of being stored; the
golden file keeps a sha256 of every input's bytes so a change in the generator is caught.
"""
from __future__ import annotations

import hashlib

import numpy as np

# (name, dtype, B, H, Lq, Lk, D, causal, scale, kv_kind)
SDPA_CASES = [
    ("f32_d40_self", "float32", 1, 2, 128, 128, 40, False, None, "randn"),
    ("f32_d64_causal_odd", "float32", 1, 2, 97, 97, 64, True, None, "randn"),
    ("f32_d128_cross", "float32", 2, 1, 70, 150, 128, False, None, "randn"),
    ("f16_d64_self", "float16", 1, 2, 256, 256, 64, False, None, "randn"),
    ("f16_d64_cross77", "float16", 1, 2, 200, 77, 64, False, None, "text_proj"),
    ("f16_d40_self", "float16", 1, 1, 200, 200, 40, False, None, "randn"),
    ("f16_d128_causal", "float16", 1, 2, 160, 160, 128, True, None, "randn"),
    ("bf16_d128_causal", "bfloat16", 1, 2, 300, 300, 128, True, None, "randn"),
    ("bf16_d128_causal_lq_lt_lk", "bfloat16", 1, 1, 130, 257, 128, True, None, "randn"),
    ("bf16_d128_causal_lq_gt_lk", "bfloat16", 1, 1, 257, 130, 128, True, None, "randn"),
    ("bf16_d64_scale", "bfloat16", 2, 1, 64, 192, 64, False, 0.3, "randn"),
    ("bf16_d64_negscale", "bfloat16", 1, 1, 64, 64, 64, False, -0.125, "randn"),
    ("bf16_d128_single_row", "bfloat16", 1, 1, 1, 33, 128, True, None, "randn"),
]

# (name, dtype, batch, m, k, n)
BMM_CASES = [
    ("bf16_bmm", "bfloat16", 2, 64, 96, 80),
    ("f16_bmm", "float16", 3, 130, 72, 64),
    ("f32_bmm", "float32", 2, 33, 17, 45),
]

# (name, dtype, input shape, out_features, bias)
LINEAR_CASES = [
    ("bf16_linear_bias", "bfloat16", (2, 37, 96), 80, True),
    ("f16_linear", "float16", (130, 72), 64, False),
    ("f16_linear_bias_3d", "float16", (3, 17, 128), 136, True),
    ("f32_linear_bias", "float32", (33, 40), 24, True),
]

EINSUM_ATTN_SHAPE = (1, 2, 128, 64)


def torch_dtype(name: str):
    import torch
    return {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[name]


def sdpa_inputs(i: int):
    """q, k, v (CPU tensors in the case's dtype) for SDPA_CASES[i]."""
    import torch
    name, dtn, B, H, Lq, Lk, D, causal, scale, kv_kind = SDPA_CASES[i]
    dt = torch_dtype(dtn)
    g = torch.Generator().manual_seed(1000 + i)
    q = torch.randn(B, H, Lq, D, generator=g).to(dt)
    if kv_kind == "text_proj":
        # cross-attention K/V projected from N(0,1) text states through N(0, 0.02) weights
        text = torch.randn(B, Lk, 2048, generator=g)
        wk = torch.randn(2048, H * D, generator=g) * 0.02
        wv = torch.randn(2048, H * D, generator=g) * 0.02
        k = (text @ wk).view(B, Lk, H, D).transpose(1, 2).contiguous().to(dt)
        v = (text @ wv).view(B, Lk, H, D).transpose(1, 2).contiguous().to(dt)
    else:
        k = torch.randn(B, H, Lk, D, generator=g).to(dt)
        v = torch.randn(B, H, Lk, D, generator=g).to(dt)
    return q, k, v


def bmm_inputs(i: int):
    import torch
    name, dtn, nb, m, k, n = BMM_CASES[i]
    dt = torch_dtype(dtn)
    g = torch.Generator().manual_seed(2000 + i)
    a = torch.randn(nb, m, k, generator=g).to(dt)
    b = torch.randn(nb, k, n, generator=g).to(dt)
    return a, b


def linear_inputs(i: int):
    """x, weight, bias (or None) for LINEAR_CASES[i]: N(0,1) inputs, N(0, 1/in_features) weights
    and N(0,1) biases, the scale of an initialised nn.Linear."""
    import torch
    name, dtn, shape, n, has_bias = LINEAR_CASES[i]
    dt = torch_dtype(dtn)
    g = torch.Generator().manual_seed(4000 + i)
    x = torch.randn(*shape, generator=g).to(dt)
    w = (torch.randn(n, shape[-1], generator=g) / shape[-1] ** 0.5).to(dt)
    b = torch.randn(n, generator=g).to(dt) if has_bias else None
    return x, w, b


def einsum_attn_inputs():
    import torch
    g = torch.Generator().manual_seed(3000)
    return tuple(torch.randn(*EINSUM_ATTN_SHAPE, generator=g).to(torch.bfloat16) for _ in range(3))


def planner_inputs(cases):
    """float64 operands for the planner cases, drawn in order from one seed-0 generator."""
    import torch
    g = torch.Generator().manual_seed(0)
    return [[torch.randn(*s, generator=g, dtype=torch.float64) for s in shapes] for _, shapes in cases]


def digest(t) -> str:
    """sha256 of a tensor's bytes (bfloat16 through its 16-bit pattern)."""
    import torch
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def to_numpy(t) -> np.ndarray:
    """Exact numpy copy of a tensor: bfloat16 -> uint16 bit pattern, others as they are."""
    import torch
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()
