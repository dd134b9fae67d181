"""Golden vectors produced by the reference's own kernels (see make_golden.py)."""
from __future__ import annotations

import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load(name: str) -> dict:
    """Loads ``name``.npz; uint16 arrays are bf16 bit patterns, float32 arrays
    fp32 tensors, 0-d arrays Python floats."""
    out = {}
    with np.load(os.path.join(HERE, name + ".npz")) as z:
        for k in z.files:
            a = z[k]
            if a.ndim == 0:
                out[k] = float(a)
            elif a.dtype == np.uint16:
                out[k] = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
            else:
                out[k] = torch.from_numpy(a.astype(np.float32))
    return out
