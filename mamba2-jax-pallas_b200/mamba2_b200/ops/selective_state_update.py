"""B200 replacement for ``src/mamba2_jax/ops/selective_state_update.py:22-123``."""

from __future__ import annotations

import torch

from .. import _lib


def selective_state_update(state, x, dt, A, B, C, D=None, z=None, dt_bias=None,
                           dt_softplus: bool = False, *, inplace: bool = False):
    """Single-token SSM step.  Returns ``(new_state, out)`` like the reference.

    The reference is functional and returns a new state; by default this copies
    ``state`` first to keep that contract.  With ``inplace=True`` the float32 state
    tensor itself is updated (no copy) and returned - the decode-loop fast path.
    """
    b, H, P, N = state.shape
    G = B.shape[1]
    if state.dtype != torch.float32:
        raise TypeError("state must be float32")
    if tuple(x.shape) != (b, H, P) or tuple(B.shape) != (b, G, N) or tuple(C.shape) != (b, G, N):
        raise ValueError("shape mismatch")
    if dt.dim() not in (2, 3) or tuple(dt.shape[:2]) != (b, H) or (dt.dim() == 3 and dt.shape[2] != P):
        raise ValueError("dt must be (b,H) or (b,H,P)")
    if tuple(A.shape) not in ((H,), (H, P, N)):
        raise ValueError("A must be (H,) or (H,P,N)")
    if not state.is_cuda:
        raise ValueError("state must be a CUDA tensor (no CPU path)")
    if inplace:
        if not state.is_contiguous():
            raise ValueError("inplace=True needs a contiguous state")
        st = state
    else:
        st = state.clone(memory_format=torch.contiguous_format)
    dtype = _lib.dtype_code(x)
    tdt = _lib.torch_dtype(dtype)
    dtc = _lib.dev(dt, "dt")
    if dtc.dtype not in (torch.float32, torch.bfloat16):
        dtc = dtc.float()
    t = dict(x=_lib.dev(x, "x"), A=_lib.dev(A, "A", torch.float32), B=_lib.dev(B, "B", tdt),
             C=_lib.dev(C, "C", tdt), D=_lib.dev(D, "D", torch.float32), z=_lib.dev(z, "z", tdt),
             bias=_lib.dev(dt_bias, "dt_bias", torch.float32))
    out = torch.empty((b, H, P), device=state.device, dtype=torch.float32)
    p = _lib.SsuParams(batch=b, nheads=H, headdim=P, ngroups=G, dstate=N, dtype=dtype,
                       dt_dtype=_lib.dtype_code(dtc), dt_ndim=dt.dim(), A_ndim=A.dim(),
                       D_ndim=0 if D is None else D.dim(),
                       dt_bias_ndim=0 if dt_bias is None else dt_bias.dim(),
                       dt_softplus=int(bool(dt_softplus)))
    p.state, p.x, p.dt, p.A = st.data_ptr(), t["x"].data_ptr(), dtc.data_ptr(), t["A"].data_ptr()
    p.B, p.C, p.D, p.z = t["B"].data_ptr(), t["C"].data_ptr(), _lib.ptr(t["D"]), _lib.ptr(t["z"])
    p.dt_bias, p.out = _lib.ptr(t["bias"]), out.data_ptr()
    _lib.check(_lib.load().ssd_selective_state_update(p, _lib.stream_of(out)))
    return st, out
