"""Generates the golden vectors in tests/golden/*.npz by running the REFERENCE package itself.

Run (in a container that has the reference checkout; it is not needed afterwards):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference /path/to/torch-cmp-patch

What it does:
  * imports the reference's ``cmpext3`` package from its checkout with a stub ``cmpext3._native``
    (the reference's own test conftest does the same, tests/conftest.py:42-46 there; its CUDA
    extension cannot be built for a CPU), with the monkeypatch ENABLED and NVML changes off
    (CMPEXT3_NVML_BOOST=0);
  * calls the patched ``F.scaled_dot_product_attention``, ``torch.bmm``, ``F.linear`` and ``torch.einsum`` on seeded
    CPU tensors -- the reference's wrappers route those to stock PyTorch (``_usable`` is False for CPU
    tensors), which is the reference's own CPU implementation of the path;
  * runs the reference planner ``cmpext3.einsum_ops.einsum`` on the equations of its own planner test
    (tests/test_einsum.py CASES, read from that file with ``ast``, not executed) in float64;
  * stores the outputs in their own precision (bfloat16 as its raw 16-bit pattern in a uint16 array;
    ``tests/golden/__init__.py``'s ``load`` turns them back) plus a sha256 of every input.  Inputs are
    regenerated from their seeds by tests/golden/cases.py, shared with the tests.
"""
from __future__ import annotations

import argparse
import ast
import math
import os
import sys
import types
from pathlib import Path
from unittest.mock import MagicMock

import numpy as np

HERE = Path(__file__).resolve().parent

sys.path.insert(0, str(HERE))
import cases as C  # noqa: E402  (tests/golden/cases.py)


def _load_reference(ref_root: Path):
    os.environ["CMPEXT3_AUTOPATCH"] = "1"
    os.environ["CMPEXT3_NVML_BOOST"] = "0"
    os.environ["CMPEXT3_AUTOSELECT"] = "0"
    sys.dont_write_bytecode = True
    fake = types.ModuleType("cmpext3._native")
    for name in ["linear", "bmm", "conv2d", "conv3d", "conv_transpose2d", "upsample_scaling",
                 "attention", "embedding", "group_norm", "layer_norm", "rmsnorm", "gelu", "silu",
                 "swish", "mish", "softmax", "softplus", "softsign", "softshrink", "tanh", "erf"]:
        setattr(fake, name, MagicMock(name=name, side_effect=AssertionError("native called on CPU")))
    sys.modules["cmpext3._native"] = fake
    sys.path.insert(0, str(ref_root))
    import cmpext3  # the reference package
    assert Path(cmpext3.__file__).resolve().is_relative_to(ref_root.resolve()), cmpext3.__file__
    assert cmpext3.is_enabled()
    return cmpext3


def _einsum_cases(ref_root: Path):
    tree = ast.parse((ref_root / "tests" / "test_einsum.py").read_text())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(getattr(t, "id", "") == "CASES" for t in node.targets):
            return ast.literal_eval(node.value)
    raise RuntimeError("CASES not found in the reference planner test")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("CMPX_REFERENCE_ROOT", ""))
    args = ap.parse_args()
    ref_root = Path(args.reference)
    if not (ref_root / "cmpext3" / "__init__.py").exists():
        raise SystemExit("--reference must point at the torch-cmp-patch checkout")

    ref = _load_reference(ref_root)
    import torch
    import torch.nn.functional as F
    torch.set_num_threads(min(8, os.cpu_count() or 1))

    out = {}
    for i, (name, dtn, B, H, Lq, Lk, D, causal, scale, kv_kind) in enumerate(C.SDPA_CASES):
        q, k, v = C.sdpa_inputs(i)
        with torch.no_grad():
            o = F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=scale)
        assert F.scaled_dot_product_attention is ref._patched_sdpa
        for key, t in (("q", q), ("k", k), ("v", v)):
            out[f"sdpa/{name}/{key}_sha256"] = np.array(C.digest(t))
        out[f"sdpa/{name}/o"] = C.to_numpy(o)

    for i, (name, dtn, nb, m, k, n) in enumerate(C.BMM_CASES):
        a, b = C.bmm_inputs(i)
        with torch.no_grad():
            c = torch.bmm(a, b)
        assert torch.bmm is ref._patched_bmm
        out[f"bmm/{name}/a_sha256"] = np.array(C.digest(a))
        out[f"bmm/{name}/b_sha256"] = np.array(C.digest(b))
        out[f"bmm/{name}/c"] = C.to_numpy(c)

    for i, (name, dtn, shape, n, has_bias) in enumerate(C.LINEAR_CASES):
        x, w, b = C.linear_inputs(i)
        with torch.no_grad():
            y = F.linear(x, w, b)
        assert F.linear is ref._patched_linear
        for key, t in (("x", x), ("w", w)) + ((("b", b),) if b is not None else ()):
            out[f"linear/{name}/{key}_sha256"] = np.array(C.digest(t))
        out[f"linear/{name}/y"] = C.to_numpy(y)

    # einsum-routed attention (the bf16 einsum -> softmax -> einsum workload, small)
    q, k, v = C.einsum_attn_inputs()
    with torch.no_grad():
        s = torch.einsum("bhid,bhjd->bhij", q, k)
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("bhij,bhjd->bhid", p, v)
    assert torch.einsum is ref._patched_einsum
    for key, t in (("q", q), ("k", k), ("v", v)):
        out[f"einsum_attn/{key}_sha256"] = np.array(C.digest(t))
    out["einsum_attn/s"] = C.to_numpy(s)
    out["einsum_attn/o"] = C.to_numpy(o)

    # the reference planner itself, on its own planner-test equations (float64)
    cases = _einsum_cases(ref_root)
    for i, ((eq, shapes), ops) in enumerate(zip(cases, C.planner_inputs(cases))):
        r = ref.einsum_ops.einsum(eq, ops)
        out[f"planner/{i}/eq"] = np.array(eq)
        out[f"planner/{i}/shapes"] = np.array(repr(shapes))
        out[f"planner/{i}/out"] = r.numpy()
    out["planner/count"] = np.array(len(cases))

    ref.disable()
    np.savez_compressed(HERE / "reference_cpu_path.npz", **out)
    print(f"wrote {HERE / 'reference_cpu_path.npz'} ({len(out)} arrays)")


if __name__ == "__main__":
    main()
