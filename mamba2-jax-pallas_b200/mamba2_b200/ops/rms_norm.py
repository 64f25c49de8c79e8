"""B200 replacement for ``src/mamba2_jax/ops/rms_norm.py`` (the step after the SSD).

The Mamba2 mixer calls it on the SSD output reshaped to (batch, seqlen, d_ssm) with
``group_size = d_ssm // ngroups`` (``modules/mamba2.py:401-406``), i.e. one group's heads
per normalisation group.
"""
from __future__ import annotations

import torch

from .. import _lib


def _rows2d(t: torch.Tensor, hidden: int):
    """(rows, hidden) view with a contiguous last axis and one row stride, else a copy."""
    t2 = t.reshape(-1, hidden)
    if t2.stride(1) != 1 or (t2.shape[0] > 1 and t2.stride(0) < hidden):
        t2 = t2.contiguous()
    return t2


def rms_norm_gated(x, weight, z=None, eps=1e-5, group_size=None, norm_before_gate=True, *, out_dtype=None):
    """RMSNorm over groups of the last axis with optional SiLU gate; ``rms_norm.py:15-92``.

    x (..., hidden) float32 or bfloat16; weight (hidden,); z of x's shape or None.
    norm_before_gate=True: ``x / rms * weight * silu(z)``; False: ``rms-normalise
    x * silu(z)``, then ``* weight``.  Returns x's shape in the promotion of the dtypes of x,
    weight and z (as JAX's arithmetic would), computed in float32 and rounded once.
    Keyword-only extension: ``out_dtype`` (float32 or bfloat16) overrides that promotion, so
    a caller that wants bf16 (the layer's out_proj input) gets it from the same pass instead
    of a separate cast.
    """
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise ValueError("x must be a CUDA tensor (no CPU path)")
    hidden = x.shape[-1]
    gs = hidden if group_size is None else int(group_size)
    if gs <= 0 or hidden % gs != 0:
        raise ValueError(f"hidden size {hidden} is not divisible by group_size {gs}")
    if tuple(weight.shape) != (hidden,):
        raise ValueError(f"weight must be ({hidden},)")
    if z is not None and tuple(z.shape) != tuple(x.shape):
        raise ValueError("z must have x's shape")
    if out_dtype is None:
        out_dtype = x.dtype
        for t in (weight, z):
            if t is not None:
                out_dtype = torch.promote_types(out_dtype, t.dtype)
    elif out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
    x2 = _rows2d(x, hidden)
    if z is not None and not z.is_cuda:
        raise ValueError("z must be a CUDA tensor (no CPU path)")
    z2 = None if z is None else _rows2d(z, hidden)
    w = _lib.dev(weight, "weight")
    _lib.dtype_code(w)
    out = torch.empty(x.shape, device=x.device, dtype=out_dtype)
    rows = x2.shape[0]
    if rows == 0 or hidden == 0:
        return out
    o2 = out.view(-1, hidden)
    p = _lib.RmsNormParams(rows=rows, hidden=hidden, group_size=gs,
                           x_stride_row=x2.stride(0) if rows > 1 else hidden,
                           z_stride_row=(z2.stride(0) if rows > 1 else hidden) if z2 is not None else hidden,
                           out_stride_row=hidden, x_dtype=_lib.dtype_code(x2),
                           z_dtype=_lib.dtype_code(z2) if z2 is not None else 0,
                           weight_dtype=_lib.dtype_code(w), out_dtype=_lib.dtype_code(o2),
                           norm_before_gate=int(bool(norm_before_gate)), eps=float(eps))
    p.x, p.z, p.weight, p.out = x2.data_ptr(), _lib.ptr(z2), w.data_ptr(), o2.data_ptr()
    _lib.check(_lib.load().ssd_rms_norm_gated(p, _lib.stream_of(out)))
    return out
