"""Golden vectors produced by the reference package itself (see make_golden.py)."""
from __future__ import annotations

from pathlib import Path

import numpy as np

PATH = Path(__file__).resolve().parent / "reference_cpu_path.npz"


def load() -> dict:
    """All arrays, with bfloat16 entries (stored as uint16 bit patterns) returned as torch tensors
    of dtype bfloat16 and every other array as numpy."""
    import torch
    z = np.load(PATH)
    out = {}
    for key in z.files:
        a = z[key]
        if a.dtype == np.uint16:
            out[key] = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
        else:
            out[key] = a
    return out
