"""B200 replacements for the five SSD stage functions and the varlen states.

Signatures follow the reference's Triton-compatible aliases; tile keyword arguments
(BM, BK, BN, num_stages) are accepted and ignored, since the B200 kernels choose
their own tiles.
  chunk_cumsum_fwd   src/mamba2_jax/kernels/chunk_cumsum_fwd.py:288-302
  chunk_state_fwd    src/mamba2_jax/kernels/chunk_state_fwd.py:424-441
  state_passing_fwd  src/mamba2_jax/kernels/state_passing_fwd.py:348-363
  bmm_chunk_fwd      src/mamba2_jax/kernels/bmm_chunk_fwd.py:381-400
  chunk_scan_fwd     src/mamba2_jax/kernels/chunk_scan_fwd.py:579-600
  chunk_state_varlen_mosaic  src/mamba2_jax/kernels/chunk_state_fwd.py:448-597
"""

from __future__ import annotations

import math

import torch

from .. import _lib


def chunk_cumsum_fwd(dt, A, chunk_size: int, dt_bias=None, dt_softplus: bool = False,
                     dt_limit=(0.0, float("inf"))):
    """dt (b,L,H) -> (dA_cumsum, dt_out), both (b,H,nc,Q) float32."""
    b, L, H = dt.shape
    if tuple(A.shape) != (H,):
        raise ValueError(f"A.shape={tuple(A.shape)} != ({H},)")
    if dt_bias is not None and tuple(dt_bias.shape) != (H,):
        raise ValueError(f"dt_bias must be ({H},)")
    dtc = _lib.dev(dt, "dt")
    if dtc.dtype not in (torch.float32, torch.bfloat16):
        dtc = dtc.float()
    A_ = _lib.dev(A, "A", torch.float32)
    bias = _lib.dev(dt_bias, "dt_bias", torch.float32)
    nc = math.ceil(L / chunk_size)
    dA = torch.empty((b, H, nc, chunk_size), device=dt.device, dtype=torch.float32)
    dto = torch.empty_like(dA)
    lo, hi = _lib.limits(dt_limit)
    _lib.check(_lib.load().ssd_chunk_cumsum_fwd(
        dtc.data_ptr(), _lib.dtype_code(dtc), A_.data_ptr(), _lib.ptr(bias), int(bool(dt_softplus)),
        lo, hi, b, L, H, chunk_size, dA.data_ptr(), dto.data_ptr(), _lib.stream_of(dA)))
    return dA, dto


def chunk_state_fwd(x, B, dt, dA_cumsum, seq_idx=None, BM: int = 64, BK: int = 64, BN: int = 64,
                    num_stages: int = 2):
    """x (b,L,H,P), B (b,L,G,N), dt/dA_cumsum (b,H,nc,Q) -> states (b,nc,H,P,N) f32."""
    b, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    _, _, nc, Q = dt.shape
    if tuple(dt.shape) != (b, H, nc, Q) or tuple(dA_cumsum.shape) != tuple(dt.shape):
        raise ValueError("dt / dA_cumsum must be (b,H,nc,Q)")
    if nc != math.ceil(L / Q):
        raise ValueError("nchunks != ceil(seqlen / chunk_size)")
    dtype = _lib.dtype_code(x)
    tdt = _lib.torch_dtype(dtype)
    xc, Bc = _lib.dev(x, "x"), _lib.dev(B, "B", tdt)
    dtc, dAc = _lib.dev(dt, "dt", torch.float32), _lib.dev(dA_cumsum, "dA_cumsum", torch.float32)
    si = _lib.dev(seq_idx, "seq_idx", torch.int32)
    states = torch.empty((b, nc, H, P, N), device=x.device, dtype=torch.float32)
    _lib.check(_lib.load().ssd_chunk_state_fwd(
        xc.data_ptr(), Bc.data_ptr(), dtype, dtc.data_ptr(), dAc.data_ptr(), _lib.ptr(si),
        b, L, H, P, G, N, Q, states.data_ptr(), _lib.stream_of(states)))
    return states


def state_passing_fwd(states, dA_chunk_cumsum, initial_states=None, seq_idx=None,
                      chunk_size=None, out_dtype=None):
    """states (b,nc,H,dim), dA_chunk_cumsum (b,H,nc) -> (out (b,nc,H,dim), final (b,H,dim))."""
    b, nc, H, dim = states.shape
    if tuple(dA_chunk_cumsum.shape) != (b, H, nc):
        raise ValueError(f"dA_chunk_cumsum must be ({b},{H},{nc})")
    if initial_states is not None and tuple(initial_states.shape) != (b, H, dim):
        raise ValueError(f"initial_states must be ({b},{H},{dim})")
    seqlen = 0
    if seq_idx is not None:
        if chunk_size is None:
            raise ValueError("seq_idx requires chunk_size")
        seqlen = seq_idx.shape[-1]
    out_dtype = states.dtype if out_dtype is None else out_dtype
    code = _lib.dtype_code(torch.empty(0, dtype=out_dtype))
    st = _lib.dev(states, "states", torch.float32)
    dA = _lib.dev(dA_chunk_cumsum, "dA_chunk_cumsum", torch.float32)
    init = _lib.dev(initial_states, "initial_states", torch.float32)
    si = _lib.dev(seq_idx, "seq_idx", torch.int32)
    out = torch.empty((b, nc, H, dim), device=states.device, dtype=out_dtype)
    final = torch.empty((b, H, dim), device=states.device, dtype=torch.float32)
    _lib.check(_lib.load().ssd_state_passing_fwd(
        st.data_ptr(), dA.data_ptr(), nc, 1, _lib.ptr(init), _lib.ptr(si), b, nc, H, dim, seqlen,
        0 if chunk_size is None else int(chunk_size), out.data_ptr(), code, final.data_ptr(),
        _lib.stream_of(out)))
    return out, final


def bmm_chunk_fwd(a, b, chunk_size: int, seq_idx=None, causal: bool = False, output_dtype=None,
                  BM: int = 64, BK: int = 64, BN: int = 64, num_stages: int = 2):
    """a, b (batch,L,G,K) -> CB (batch,nc,G,Q,Q) (float32 unless output_dtype)."""
    bs, L, G, K = a.shape
    if tuple(b.shape) != tuple(a.shape):
        raise ValueError("a and b must have the same shape")
    dtype = _lib.dtype_code(a)
    ac, bc = _lib.dev(a, "a"), _lib.dev(b, "b", _lib.torch_dtype(dtype))
    si = _lib.dev(seq_idx, "seq_idx", torch.int32)
    nc = math.ceil(L / chunk_size)
    out = torch.empty((bs, nc, G, chunk_size, chunk_size), device=a.device, dtype=torch.float32)
    _lib.check(_lib.load().ssd_bmm_chunk_fwd(
        ac.data_ptr(), bc.data_ptr(), dtype, _lib.ptr(si), int(bool(causal)), bs, L, G, K,
        chunk_size, out.data_ptr(), _lib.stream_of(out)))
    if output_dtype is not None and output_dtype != torch.float32:
        out = out.to(output_dtype)
    return out


def chunk_scan_fwd(cb, x, dt, dA_cumsum, C, states, D=None, z=None, seq_idx=None,
                   BM: int = 64, BK: int = 64, BN: int = 64, num_stages: int = 2):
    """-> (out, out_x): out (b,L,H,P) f32; out_x the pre-gate output when z is given."""
    b, L, H, P = x.shape
    G, N = C.shape[2], C.shape[3]
    _, _, nc, Q = dt.shape
    if tuple(cb.shape) != (b, nc, G, Q, Q):
        raise ValueError(f"cb must be ({b},{nc},{G},{Q},{Q})")
    if tuple(states.shape) != (b, nc, H, P, N):
        raise ValueError(f"states must be ({b},{nc},{H},{P},{N})")
    dtype = _lib.dtype_code(x)
    tdt = _lib.torch_dtype(dtype)
    st = _lib.dev(states, "states")
    if st.dtype not in (torch.float32, torch.bfloat16):
        st = st.float()
    t = dict(cb=_lib.dev(cb, "cb", torch.float32), x=_lib.dev(x, "x"),
             dt=_lib.dev(dt, "dt", torch.float32), dA=_lib.dev(dA_cumsum, "dA_cumsum", torch.float32),
             C=_lib.dev(C, "C", tdt), D=_lib.dev(D, "D", torch.float32), z=_lib.dev(z, "z", tdt),
             si=_lib.dev(seq_idx, "seq_idx", torch.int32))
    out = torch.empty((b, L, H, P), device=x.device, dtype=torch.float32)
    out_x = torch.empty_like(out) if z is not None else None
    _lib.check(_lib.load().ssd_chunk_scan_fwd(
        t["cb"].data_ptr(), t["x"].data_ptr(), dtype, t["dt"].data_ptr(), t["dA"].data_ptr(),
        t["C"].data_ptr(), st.data_ptr(), _lib.dtype_code(st), _lib.ptr(t["D"]),
        0 if D is None else D.dim(), _lib.ptr(t["z"]), _lib.ptr(t["si"]), b, L, H, P, G, N, Q,
        out.data_ptr(), _lib.ptr(out_x), _lib.stream_of(out)))
    return out, out_x


def chunk_state_varlen_mosaic(B, x, dt, dA_cumsum, cu_seqlens, chunk_states, BM: int = 64,
                              BK: int = 64, BN: int = 64, num_stages: int = 2):
    """B (T,G,N), x (T,H,P), dt/dA_cumsum (H,nc,Q), chunk_states (nc,H,P,N) -> (S,H,P,N) f32."""
    T, H, P = x.shape
    G, N = B.shape[1], B.shape[2]
    _, nc, Q = dt.shape
    if tuple(chunk_states.shape) != (nc, H, P, N):
        raise ValueError(f"chunk_states must be ({nc},{H},{P},{N})")
    dtype = _lib.dtype_code(x)
    cs = _lib.dev(chunk_states, "chunk_states")
    if cs.dtype not in (torch.float32, torch.bfloat16):
        cs = cs.float()
    Bc = _lib.dev(B, "B", _lib.torch_dtype(dtype))
    xc = _lib.dev(x, "x")
    dtc, dAc = _lib.dev(dt, "dt", torch.float32), _lib.dev(dA_cumsum, "dA_cumsum", torch.float32)
    cu = _lib.dev(cu_seqlens, "cu_seqlens", torch.int32)
    S = cu.shape[0] - 1
    out = torch.empty((S, H, P, N), device=x.device, dtype=torch.float32)
    _lib.check(_lib.load().ssd_chunk_state_varlen_fwd(
        Bc.data_ptr(), xc.data_ptr(), dtype, dtc.data_ptr(), dAc.data_ptr(), cu.data_ptr(), S,
        cs.data_ptr(), _lib.dtype_code(cs), T, H, P, G, N, Q, out.data_ptr(), _lib.stream_of(out)))
    return out
