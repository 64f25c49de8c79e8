"""B200 replacement for ``src/mamba2_jax/ops/causal_conv1d.py`` (the step before the SSD).

``causal_conv1d`` takes x as (batch, dim, seqlen) like the reference, at any strides: the
Mamba2 layer passes a transposed view of its channels-last (batch, seqlen, dim) activations,
which the kernel reads in place, and the output is allocated in the same layout so that the
layer's transpose back is free.
"""
from __future__ import annotations

import torch

from .. import _lib


def _weight2d(weight: torch.Tensor) -> torch.Tensor:
    if weight.dim() == 3:
        if weight.shape[1] != 1:
            raise ValueError("weight must be (dim, width) or (dim, 1, width)")
        weight = weight[:, 0, :]
    if weight.dim() != 2:
        raise ValueError("weight must be (dim, width) or (dim, 1, width)")
    return weight


def _param(t, name):
    """Weight or bias as stored (f32 or bf16 are read by the kernels directly; other
    dtypes are cast to f32), contiguous, on the device."""
    if t is None:
        return None
    return _lib.dev(t, name, None if t.dtype in (torch.float32, torch.bfloat16) else torch.float32)


def _promote(*ts) -> torch.dtype:
    dt = ts[0].dtype
    for t in ts[1:]:
        if t is not None:
            dt = torch.promote_types(dt, t.dtype)
    return dt


def causal_conv1d(x, weight, bias=None, activation=None, seq_idx=None):
    """Causal depthwise conv over the last axis; ``causal_conv1d.py:18-85``.

    x (batch, dim, seqlen) float32 or bfloat16; weight (dim, width) or (dim, 1, width) of
    x's dtype; bias (dim,) or None; activation "silu" or anything else for none (as the
    reference); seq_idx (batch, seqlen) integer ids or None.  Returns (batch, dim, seqlen)
    in the promotion of x's and bias's dtypes, computed in float32 and rounded once.
    """
    if x.dim() != 3:
        raise ValueError("x must be (batch, dim, seqlen)")
    w = _weight2d(weight)
    b, d, L = x.shape
    if w.shape[0] != d:
        raise ValueError(f"weight has {w.shape[0]} channels, x has {d}")
    if w.dtype != x.dtype:
        # lax.conv_general_dilated requires equal operand dtypes
        raise TypeError(f"x ({x.dtype}) and weight ({w.dtype}) must have the same dtype")
    if bias is not None and tuple(bias.shape) != (d,):
        raise ValueError("bias must be (dim,)")
    if seq_idx is not None and tuple(seq_idx.shape) != (b, L):
        raise ValueError("seq_idx must be (batch, seqlen)")
    if not x.is_cuda:
        raise ValueError("x must be a CUDA tensor (no CPU path)")
    out_dtype = _promote(x, bias)
    if x.stride(1) == 1:
        out = torch.empty((b, L, d), device=x.device, dtype=out_dtype).transpose(1, 2)
    else:
        out = torch.empty((b, d, L), device=x.device, dtype=out_dtype)
    wt = _param(w, "weight")
    bt = _param(bias, "bias")
    sq = _lib.dev(seq_idx, "seq_idx", torch.int32)
    p = _lib.Conv1dParams(batch=b, dim=d, seqlen=L,
                          x_stride_b=x.stride(0), x_stride_d=x.stride(1), x_stride_t=x.stride(2),
                          out_stride_b=out.stride(0), out_stride_d=out.stride(1),
                          out_stride_t=out.stride(2), width=w.shape[1], dtype=_lib.dtype_code(x),
                          out_dtype=_lib.dtype_code(out), silu=int(activation == "silu"))
    p.x, p.weight, p.bias = x.data_ptr(), wt.data_ptr(), _lib.ptr(bt)
    p.seq_idx, p.out = _lib.ptr(sq), out.data_ptr()
    p.weight_dtype, p.bias_dtype = _lib.dtype_code(wt), (_lib.dtype_code(bt) if bt is not None else 0)
    _lib.check(_lib.load().ssd_causal_conv1d_fwd(p, _lib.stream_of(out)))
    return out


def causal_conv1d_update(x_new, conv_state, weight, bias=None, activation=None, *, inplace: bool = False):
    """One decode step; ``causal_conv1d.py:88-139``.  Returns ``(new_conv_state, out)``.

    The state (batch, dim, width) shifts left by one and takes x_new (batch, dim) in its last
    slot; out = act(bias + sum_j weight[:, j] * state[:, :, j]).  Like the reference this
    returns a new state (in the promotion of the state's and x_new's dtypes); with
    ``inplace=True`` the given state is updated and returned (it must already have that
    dtype and a contiguous width axis).
    """
    w = _weight2d(weight)
    if conv_state.dim() != 3 or x_new.dim() != 2:
        raise ValueError("conv_state must be (batch, dim, width) and x_new (batch, dim)")
    b, d, k = conv_state.shape
    if tuple(x_new.shape) != (b, d) or tuple(w.shape) != (d, k):
        raise ValueError("shape mismatch between x_new, conv_state and weight")
    if bias is not None and tuple(bias.shape) != (d,):
        raise ValueError("bias must be (dim,)")
    if not conv_state.is_cuda:
        raise ValueError("conv_state must be a CUDA tensor (no CPU path)")
    st_dtype = _promote(conv_state, x_new)
    if inplace:
        if conv_state.dtype != st_dtype or conv_state.stride(2) != 1:
            raise ValueError("inplace=True needs a state of the promoted dtype with a contiguous width axis")
        st = conv_state
    else:
        st = conv_state.to(st_dtype).clone(memory_format=torch.contiguous_format)
    out_dtype = _promote(st, w, bias)
    out = torch.empty((b, d), device=conv_state.device, dtype=out_dtype)
    xt = _lib.dev(x_new, "x_new")
    wt = _param(w, "weight")
    bt = _param(bias, "bias")
    p = _lib.Conv1dUpdateParams(batch=b, dim=d, state_stride_b=st.stride(0), state_stride_d=st.stride(1),
                                width=k, x_dtype=_lib.dtype_code(xt), state_dtype=_lib.dtype_code(st),
                                out_dtype=_lib.dtype_code(out), silu=int(activation == "silu"))
    p.x_new, p.conv_state, p.weight = xt.data_ptr(), st.data_ptr(), wt.data_ptr()
    p.bias, p.out = _lib.ptr(bt), out.data_ptr()
    p.weight_dtype, p.bias_dtype = _lib.dtype_code(wt), (_lib.dtype_code(bt) if bt is not None else 0)
    _lib.check(_lib.load().ssd_causal_conv1d_update(p, _lib.stream_of(out)))
    return st, out
