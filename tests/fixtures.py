"""Loader for the golden fixtures under tests/golden/ (written by tests/golden/make_fixtures.py
from the reference's own ops run unmodified on a NumPy stand-in for jax)."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    """Dict of arrays of tests/golden/<name>_fixtures.npz; bf16-packed arrays come back as
    float32 with the same values."""
    out = {}
    with np.load(os.path.join(GOLDEN, f"{name}_fixtures.npz")) as z:
        for k in z.files:
            v = z[k]
            if k.endswith("@bf16"):
                v = (v.astype(np.uint32) << 16).view(np.float32)
                k = k[:-5]
            out[k] = v
    return out


def case(d, prefix):
    """Sub-dict of entries '<prefix>/<key>' -> key."""
    n = len(prefix) + 1
    return {k[n:]: v for k, v in d.items() if k.startswith(prefix + "/")}
