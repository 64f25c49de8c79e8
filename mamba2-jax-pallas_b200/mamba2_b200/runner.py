"""Static-shape launcher for serving loops: binds device tensors to a prepared
``ssd_fwd_params_t`` once, so each step is a single C-ABI call (and can be captured in
a CUDA graph, since the library neither allocates nor synchronises)."""

from __future__ import annotations

import math

import torch

from . import _lib
from .kernels.ssd_combined import _fwd_params


class SsdForward:
    """Preallocated outputs + workspace for repeated ``ssd_combined_fwd`` calls on fixed
    device tensors (the tensors must stay alive and keep their storage)."""

    def __init__(self, x, dt, A, B, C, chunk_size, D=None, z=None, dt_bias=None,
                 initial_states=None, seq_idx=None, cu_seqlens=None, dt_softplus=False,
                 dt_limit=(0.0, math.inf), return_final_states=False, flags=0):
        for name, t in (("x", x), ("dt", dt), ("B", B), ("C", C), ("z", z)):
            if t is not None and not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous for a bound launcher")
        self.p, self._keep = _fwd_params(x, dt, A, B, C, chunk_size, D, z, dt_bias, initial_states,
                                         seq_idx, cu_seqlens, dt_softplus, dt_limit, flags)
        b, L, H, P = x.shape
        N = B.shape[3]
        self.out = torch.empty((b, L, H, P), device=x.device, dtype=torch.float32)
        self.p.out = self.out.data_ptr()
        self.final = None
        if return_final_states:
            self.final = torch.empty((b, H, P, N), device=x.device, dtype=torch.float32)
            self.p.final_states = self.final.data_ptr()
        self.varlen = None
        if cu_seqlens is not None:
            self.varlen = torch.empty((self.p.num_seqs, H, P, N), device=x.device, dtype=torch.float32)
            self.p.varlen_states = self.varlen.data_ptr()
        self.lib = _lib.load()
        n = self.lib.ssd_combined_workspace_bytes(self.p)
        self.workspace = torch.empty(max(n, 1), device=x.device, dtype=torch.uint8)
        self.uses_tc = bool(self.lib.ssd_combined_uses_tensor_cores(self.p))
        self.launches_per_step = int(self.lib.ssd_combined_num_launches(self.p))

    def __call__(self, stream=None):
        s = torch.cuda.current_stream(self.out.device) if stream is None else stream
        _lib.check(self.lib.ssd_combined_fwd(self.p, self.workspace.data_ptr(),
                                             self.workspace.numel(), s.cuda_stream))
        return self.out

    def graph(self):
        """Capture one call into a torch.cuda.CUDAGraph (replay with ``g.replay()``)."""
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.out.device)
        s.wait_stream(torch.cuda.current_stream(self.out.device))
        with torch.cuda.stream(s):
            self(s)  # warm-up outside capture
        torch.cuda.current_stream(self.out.device).wait_stream(s)
        with torch.cuda.graph(g):
            self()
        return g
