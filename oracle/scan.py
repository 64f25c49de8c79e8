"""ctypes wrapper of oracle/ssd_scan.c (float64 token-by-token recurrence, OpenMP).

TEST INFRASTRUCTURE ONLY (see oracle/ssd_ref.py): the checker for full-size parity tests.
``build()`` compiles ``oracle/_build/libssd_scan.so`` with gcc; ``ssd_scan()`` builds it on
first use if it is missing.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "ssd_scan.c")
LIB = os.path.join(HERE, "_build", "libssd_scan.so")

_vp, _i64, _i32, _f64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_double


class _Args(ctypes.Structure):
    _fields_ = [("b", _i64), ("L", _i64), ("H", _i64), ("P", _i64), ("G", _i64), ("N", _i64),
                ("h0", _i64), ("h1", _i64), ("x", _vp), ("dt", _vp), ("A", _vp), ("B", _vp), ("C", _vp),
                ("D", _vp), ("D_ndim", _i32), ("dt_softplus", _i32), ("z", _vp), ("dt_bias", _vp),
                ("dt_min", _f64), ("dt_max", _f64), ("init", _vp), ("seq_idx", _vp), ("cu_seqlens", _vp),
                ("num_seqs", _i64), ("out", _vp), ("final_states", _vp), ("varlen_states", _vp)]


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", SRC, "-o", LIB, "-lm"]
    subprocess.run(cmd, check=True, capture_output=True)
    return LIB


_lib = None


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        _lib.ssd_scan_f64.argtypes = [ctypes.POINTER(_Args)]
        _lib.ssd_scan_f64.restype = ctypes.c_int
    return _lib


def _c(a, dt):
    return None if a is None else np.ascontiguousarray(a, dtype=dt)


def ssd_scan(x, dt, A, B, C, D=None, z=None, dt_bias=None, initial_states=None, seq_idx=None,
             cu_seqlens=None, dt_softplus=False, dt_limit=(0.0, math.inf), heads=None):
    """Returns (out, final_states, varlen_states or None), float64; only heads
    ``range(*heads)`` are computed (others are zero)."""
    x, dt, A, B, C = (_c(v, np.float32) for v in (x, dt, A, B, C))
    D, z, dt_bias, init = (_c(v, np.float32) for v in (D, z, dt_bias, initial_states))
    seq_idx, cu = _c(seq_idx, np.int32), _c(cu_seqlens, np.int32)
    b, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    h0, h1 = heads if heads is not None else (0, H)
    out = np.zeros((b, L, H, P))
    final = np.zeros((b, H, P, N))
    ns = 0 if cu is None else len(cu) - 1
    varlen = np.zeros((ns, H, P, N)) if cu is not None else None
    p = lambda a: None if a is None else a.ctypes.data
    args = _Args(b=b, L=L, H=H, P=P, G=G, N=N, h0=h0, h1=h1, x=p(x), dt=p(dt), A=p(A), B=p(B), C=p(C),
                 D=p(D), D_ndim=0 if D is None else D.ndim, dt_softplus=int(bool(dt_softplus)), z=p(z),
                 dt_bias=p(dt_bias), dt_min=float(dt_limit[0]), dt_max=float(dt_limit[1]), init=p(init),
                 seq_idx=p(seq_idx), cu_seqlens=p(cu), num_seqs=ns, out=p(out), final_states=p(final),
                 varlen_states=p(varlen))
    rc = _load().ssd_scan_f64(ctypes.byref(args))
    if rc:
        raise RuntimeError(f"ssd_scan_f64 failed ({rc})")
    return out, final, varlen
