"""The Mamba2 mixer layer wired from the B200 kernels (``src/mamba2_jax/modules/mamba2.py:81-560``).

One layer, as the reference composes it:

    u (b, L, d_model) -> in_proj -> [z0 | x0 | z | xBC | dt]
    xBC -> causal_conv1d (SiLU, seq_idx masks)                     ssd_causal_conv1d_fwd
    x, B, C -> SSD chunked scan (dt bias + softplus, D skip)        ssd_combined_fwd
    y -> gated RMSNorm with z, group = d_ssm / ngroups             ssd_rms_norm_gated
    [silu(z0) x0 | y] -> out_proj

and the single-token decode step of ``Mamba2._step`` (``:437-520``) with
``ssd_causal_conv1d_update`` and ``ssd_selective_state_update``.  The two projections are
plain bf16 GEMMs (torch.matmul, i.e. cuBLAS); every other stage runs in libssd_b200.so.
The conv output stays channels-last, so the layer's transposes cost nothing.

Parameters are random-initialised with the reference's initialisers' distributions
(``_dt_bias_init``, ``_A_log_init``; projections ~ N(0, 1/fan_in)), stored in bf16 except
dt_bias, A_log, D and the norm weight (f32).  The reference's tensor-parallel wrappers
(``distributed/tensor_parallel.py``) are not mirrored: the layer runs on one GPU, and
multi-GPU runs shard its heads (mamba2_b200.sharding).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..kernels.ssd_combined import mamba_chunk_scan_combined_fwd
from ..ops.causal_conv1d import causal_conv1d, causal_conv1d_update
from ..ops.rms_norm import rms_norm_gated
from ..ops.selective_state_update import selective_state_update


class Mamba2:
    """A Mamba2 mixer layer with the reference's attributes and call convention
    (``out = layer(u)``; with ``inference_params`` it returns ``(out, new_params)``)."""

    def __init__(self, d_model, d_state=128, d_conv=4, expand=2, headdim=64, d_ssm=None, ngroups=1,
                 A_init_range=(1.0, 16.0), D_has_hdim=False, rmsnorm=True, norm_before_gate=False,
                 dt_min=0.001, dt_max=0.1, dt_init_floor=1e-4, dt_limit=(0.0, float("inf")), bias=False,
                 conv_bias=True, chunk_size=256, device="cuda", seed=0):
        self.d_model, self.d_state, self.d_conv, self.headdim = d_model, d_state, d_conv, headdim
        self.ngroups, self.D_has_hdim, self.rmsnorm = ngroups, D_has_hdim, rmsnorm
        self.norm_before_gate, self.dt_limit, self.chunk_size = norm_before_gate, dt_limit, chunk_size
        self.d_inner = expand * d_model
        self.d_ssm = self.d_inner if d_ssm is None else d_ssm
        self.d_mlp = self.d_inner - self.d_ssm
        if self.d_ssm % headdim:
            raise ValueError(f"d_ssm ({self.d_ssm}) must be divisible by headdim ({headdim})")
        self.nheads = self.d_ssm // headdim
        if self.nheads % ngroups:
            raise ValueError(f"nheads ({self.nheads}) must be divisible by ngroups ({ngroups})")
        self.conv_dim = self.d_ssm + 2 * ngroups * d_state
        self.d_in_proj = 2 * self.d_inner + 2 * ngroups * d_state + self.nheads

        g = torch.Generator(device="cpu").manual_seed(seed)
        bf = torch.bfloat16
        dev = torch.device(device)

        def normal(shape, std):
            return (torch.randn(shape, generator=g) * std).to(dev)

        H = self.nheads
        self.in_proj_kernel = normal((d_model, self.d_in_proj), 1 / math.sqrt(d_model)).to(bf)
        self.out_proj_kernel = normal((self.d_inner, d_model), 1 / math.sqrt(self.d_inner)).to(bf)
        self.in_proj_bias = torch.zeros(self.d_in_proj, device=dev).to(bf) if bias else None
        self.out_proj_bias = torch.zeros(d_model, device=dev).to(bf) if bias else None
        self.conv1d_weight = normal((self.conv_dim, d_conv), 1 / math.sqrt(d_conv)).to(bf)
        self.conv1d_bias = (0.1 * torch.randn(self.conv_dim, generator=g)).to(dev).to(bf) if conv_bias else None
        # dt_bias = softplus^-1(dt), dt log-uniform in [dt_min, dt_max], floored (_dt_bias_init)
        dt = torch.exp(torch.rand(H, generator=g) * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
        dt = dt.clamp(min=dt_init_floor)
        self.dt_bias = (dt + torch.log(-torch.expm1(-dt))).to(dev)
        # A_log = log U[A_init_range] (_A_log_init); A = -exp(A_log)
        lo, hi = A_init_range
        self.A_log = torch.log(torch.rand(H, generator=g) * (hi - lo) + lo).to(dev)
        self.D = torch.ones(self.d_ssm if D_has_hdim else H, device=dev)
        self.norm_weight = torch.ones(self.d_ssm, device=dev) if rmsnorm else None

    # ------------------------------------------------------------------
    def _split(self, zxbcdt):
        sizes = [self.d_mlp, self.d_mlp, self.d_ssm, self.conv_dim, self.nheads]
        return torch.split(zxbcdt, sizes, dim=-1)

    def _tail(self, y, z, z0, x0):
        """Gated RMSNorm, MLP bypass and output projection (steps 7-9)."""
        if self.rmsnorm:
            # bf16 straight from the norm pass (out_proj's input dtype): no separate cast
            y = rms_norm_gated(y, self.norm_weight, z=z, group_size=self.d_ssm // self.ngroups,
                               norm_before_gate=self.norm_before_gate, out_dtype=torch.bfloat16)
        y = y.to(torch.bfloat16)
        if self.d_mlp > 0:
            y = torch.cat([F.silu(z0.float()).to(torch.bfloat16) * x0, y], dim=-1)
        out = y @ self.out_proj_kernel
        if self.out_proj_bias is not None:
            out = out + self.out_proj_bias
        return out

    def __call__(self, u, seq_idx=None, cu_seqlens=None, inference_params=None):
        """Forward of ``modules/mamba2.py:179-425``; u (b, L, d_model) bf16 on the GPU."""
        if inference_params is not None and inference_params.get("seqlen_offset", 0) > 0:
            return self.step(u, inference_params)
        b, L, _ = u.shape
        A = -torch.exp(self.A_log)
        zxbcdt = u @ self.in_proj_kernel
        if self.in_proj_bias is not None:
            zxbcdt = zxbcdt + self.in_proj_bias
        z0, x0, z, xBC, dt = self._split(zxbcdt)
        new_conv_state = None
        if inference_params is not None:
            xt = xBC.transpose(1, 2)
            new_conv_state = (xt[:, :, -self.d_conv:] if L >= self.d_conv
                              else F.pad(xt, (self.d_conv - L, 0))).contiguous()
        # channels-last in and out: (b, conv_dim, L) views of (b, L, conv_dim) storage
        xBC = causal_conv1d(xBC.transpose(1, 2), self.conv1d_weight, bias=self.conv1d_bias,
                            activation="silu", seq_idx=seq_idx).transpose(1, 2)
        GN = self.ngroups * self.d_state
        x = xBC[..., :self.d_ssm].reshape(b, L, self.nheads, self.headdim)
        B = xBC[..., self.d_ssm:self.d_ssm + GN].reshape(b, L, self.ngroups, self.d_state)
        C = xBC[..., self.d_ssm + GN:].reshape(b, L, self.ngroups, self.d_state)
        D = self.D.reshape(self.nheads, self.headdim) if self.D_has_hdim else self.D
        z_scan = None if self.rmsnorm else z.reshape(b, L, self.nheads, self.headdim)
        res = mamba_chunk_scan_combined_fwd(
            x, dt.contiguous(), A, B, C, self.chunk_size, D=D, z=z_scan, dt_bias=self.dt_bias,
            seq_idx=seq_idx, cu_seqlens=cu_seqlens, dt_softplus=True, dt_limit=self.dt_limit,
            return_final_states=inference_params is not None)
        y, final = (res if inference_params is not None else (res, None))
        out = self._tail(y.reshape(b, L, self.d_ssm), z, z0, x0)
        if inference_params is not None:
            return out, {"conv_state": new_conv_state, "ssm_state": final,
                         "seqlen_offset": inference_params.get("seqlen_offset", 0) + L}
        return out

    def step(self, u, inference_params):
        """One decode token (``Mamba2._step``, ``modules/mamba2.py:437-520``); u (b, 1, d_model)."""
        A = -torch.exp(self.A_log)
        zxbcdt = u[:, 0] @ self.in_proj_kernel
        if self.in_proj_bias is not None:
            zxbcdt = zxbcdt + self.in_proj_bias
        z0, x0, z, xBC, dt = self._split(zxbcdt)
        conv_state, xBC = causal_conv1d_update(xBC, inference_params["conv_state"], self.conv1d_weight,
                                               bias=self.conv1d_bias, activation="silu")
        GN = self.ngroups * self.d_state
        x = xBC[:, :self.d_ssm].reshape(-1, self.nheads, self.headdim)
        B = xBC[:, self.d_ssm:self.d_ssm + GN].reshape(-1, self.ngroups, self.d_state)
        C = xBC[:, self.d_ssm + GN:].reshape(-1, self.ngroups, self.d_state)
        D = self.D.reshape(self.nheads, self.headdim) if self.D_has_hdim else self.D
        z_step = None if self.rmsnorm else z.reshape(-1, self.nheads, self.headdim)
        ssm_state, y = selective_state_update(inference_params["ssm_state"], x, dt.contiguous(), A, B, C,
                                              D=D, z=z_step, dt_bias=self.dt_bias, dt_softplus=True)
        out = self._tail(y.reshape(-1, self.d_ssm), z, z0, x0)[:, None]
        return out, {"conv_state": conv_state, "ssm_state": ssm_state,
                     "seqlen_offset": inference_params["seqlen_offset"] + 1}


def allocate_inference_cache(batch_size, layer: Mamba2, device="cuda"):
    """Zero decode caches of ``modules/mamba2.py:562-``: conv_state (b, conv_dim, d_conv) and
    ssm_state (b, H, P, N) float32."""
    return {"conv_state": torch.zeros(batch_size, layer.conv_dim, layer.d_conv, device=device),
            "ssm_state": torch.zeros(batch_size, layer.nheads, layer.headdim, layer.d_state, device=device),
            "seqlen_offset": 0}
