"""B200 replacement for ``src/mamba2_jax/kernels/ssd_combined.py``.

``mamba_chunk_scan_combined_fwd`` keeps the reference signature (``ssd_combined.py:46-63``)
and return convention (``:194-203``).  Inputs are torch CUDA tensors; the computation runs
in ``libssd_b200.so`` (``ssd_combined_fwd``) on the current CUDA stream.  Outputs are
float32, as in the reference (``chunk_scan_fwd.py:547-550``).
"""

from __future__ import annotations

import math

import torch

from .. import _lib


def _fwd_params(x, dt, A, B, C, chunk_size, D, z, dt_bias, initial_states, seq_idx,
                cu_seqlens, dt_softplus, dt_limit, flags):
    if x.dim() != 4 or dt.dim() != 3 or B.dim() != 4 or C.dim() != 4:
        raise ValueError("expected x (b,L,H,P), dt (b,L,H), B/C (b,L,G,N)")
    b, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    if tuple(dt.shape) != (b, L, H) or tuple(B.shape) != (b, L, G, N) or tuple(C.shape) != (b, L, G, N):
        raise ValueError(f"shape mismatch: x{tuple(x.shape)} dt{tuple(dt.shape)} "
                         f"B{tuple(B.shape)} C{tuple(C.shape)}")
    if tuple(A.shape) != (H,):
        raise ValueError(f"A.shape={tuple(A.shape)} != ({H},)")
    dtype = _lib.dtype_code(x)
    tdt = _lib.torch_dtype(dtype)
    t = dict(
        x=_lib.dev(x, "x"), dt=_lib.dev(dt, "dt"), A=_lib.dev(A, "A", torch.float32),
        B=_lib.dev(B, "B", tdt), C=_lib.dev(C, "C", tdt),
        D=_lib.dev(D, "D", torch.float32), z=_lib.dev(z, "z", tdt),
        dt_bias=_lib.dev(dt_bias, "dt_bias", torch.float32),
        initial_states=_lib.dev(initial_states, "initial_states", torch.float32),
        seq_idx=_lib.dev(seq_idx, "seq_idx", torch.int32),
        cu_seqlens=_lib.dev(cu_seqlens, "cu_seqlens", torch.int32),
    )
    if t["dt"].dtype not in (torch.float32, torch.bfloat16):
        t["dt"] = t["dt"].float()
    if D is not None and tuple(D.shape) not in ((H,), (H, P)):
        raise ValueError(f"D must be ({H},) or ({H},{P})")
    if z is not None and tuple(z.shape) != (b, L, H, P):
        raise ValueError("z must match x")
    if dt_bias is not None and tuple(dt_bias.shape) != (H,):
        raise ValueError(f"dt_bias must be ({H},)")
    if initial_states is not None and tuple(initial_states.shape) != (b, H, P, N):
        raise ValueError(f"initial_states must be ({b},{H},{P},{N})")
    if seq_idx is not None and tuple(seq_idx.shape) != (b, L):
        raise ValueError(f"seq_idx must be ({b},{L})")
    lo, hi = _lib.limits(dt_limit)
    p = _lib.SsdFwdParams(
        batch=b, seqlen=L, nheads=H, headdim=P, ngroups=G, dstate=N, chunk_size=int(chunk_size),
        dtype=dtype, dt_dtype=_lib.dtype_code(t["dt"]), dt_softplus=int(bool(dt_softplus)),
        D_ndim=0 if D is None else D.dim(), dt_min=lo, dt_max=hi,
        num_seqs=0 if cu_seqlens is None else int(cu_seqlens.shape[0]) - 1, flags=flags)
    for k in ("x", "dt", "A", "B", "C", "D", "z", "dt_bias", "initial_states", "seq_idx", "cu_seqlens"):
        setattr(p, k, _lib.ptr(t[k]))
    return p, t


def mamba_chunk_scan_combined_fwd(
    x, dt, A, B, C, chunk_size: int, D=None, z=None, dt_bias=None, initial_states=None,
    seq_idx=None, cu_seqlens=None, dt_softplus: bool = False,
    dt_limit: tuple = (0.0, float("inf")), return_final_states: bool = False,
    return_varlen_states: bool = False, *, round_states: bool = False,
    force_simt: bool = False, bf16_mma: bool = False, return_out_x: bool = False, workspace=None,
    check_status: bool = False,
):
    """Mamba2 SSD chunked-scan forward (reference ``ssd_combined.py:46-203``).

    Returns ``out`` | ``(out, final_states)`` | ``(out, varlen_states)`` |
    ``(out, final_states, varlen_states)`` exactly as ``ssd_combined.py:194-203``.
    Keyword-only extensions: ``round_states`` rounds the passed chunk states to the input
    dtype before the output stage (the reference does, ``ssd_combined.py:140``);
    ``force_simt`` selects the fp32 CUDA-core pipeline; ``bf16_mma`` runs fp32 inputs on the
    tensor-core pipeline with bf16 MMA operands (the reference's Pallas kernels do the same
    for fp32 inputs), instead of exact fp32 on the CUDA cores; ``return_out_x`` appends the
    pre-gate output; ``workspace`` is an optional preallocated uint8 CUDA tensor;
    ``check_status`` waits for the call and raises ``SsdError`` (SSD_ERR_TIMEOUT) if a bounded
    wait inside the fused kernel gave up (the default leaves the call asynchronous).
    """
    if not return_varlen_states:
        cu_seqlens = None
    elif cu_seqlens is None:
        raise ValueError("return_varlen_states requires cu_seqlens")
    flags = (_lib.SSD_FLAG_ROUND_STATES if round_states else 0) | \
            (_lib.SSD_FLAG_FORCE_SIMT if force_simt else 0) | \
            (_lib.SSD_FLAG_BF16_MMA if bf16_mma else 0)
    p, t = _fwd_params(x, dt, A, B, C, chunk_size, D, z, dt_bias, initial_states, seq_idx,
                       cu_seqlens, dt_softplus, dt_limit, flags)
    b, L, H, P = x.shape
    N = B.shape[3]
    dev = x.device
    out = torch.empty((b, L, H, P), device=dev, dtype=torch.float32)
    p.out = out.data_ptr()
    out_x = None
    if return_out_x and z is not None:
        out_x = torch.empty_like(out)
        p.out_x = out_x.data_ptr()
    final = None
    if return_final_states:
        final = torch.empty((b, H, P, N), device=dev, dtype=torch.float32)
        p.final_states = final.data_ptr()
    varlen = None
    if cu_seqlens is not None:
        varlen = torch.empty((p.num_seqs, H, P, N), device=dev, dtype=torch.float32)
        p.varlen_states = varlen.data_ptr()
    lib = _lib.load()
    nbytes = lib.ssd_combined_workspace_bytes(p)
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(max(nbytes, 1), device=dev, dtype=torch.uint8)
    _lib.check(lib.ssd_combined_fwd(p, workspace.data_ptr(), workspace.numel(), _lib.stream_of(out)))
    if check_status:
        _lib.check_device_status(workspace)
    res = [out]
    if return_final_states:
        res.append(final)
    if cu_seqlens is not None:
        res.append(varlen)
    if return_out_x:
        res.append(out_x)
    return res[0] if len(res) == 1 else tuple(res)


def workspace_bytes(x, dt, A, B, C, chunk_size, **kw) -> int:
    """Bytes of scratch ``mamba_chunk_scan_combined_fwd`` needs for these inputs."""
    p, _ = _fwd_params(x, dt, A, B, C, chunk_size, kw.get("D"), kw.get("z"), kw.get("dt_bias"),
                       kw.get("initial_states"), kw.get("seq_idx"), kw.get("cu_seqlens"),
                       kw.get("dt_softplus", False), kw.get("dt_limit", (0.0, math.inf)),
                       kw.get("flags", 0))
    return _lib.load().ssd_combined_workspace_bytes(p)
