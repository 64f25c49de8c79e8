"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configs.

The reference benchmarks synthetic tensors only (``benchmarks/bench_model_forward.py:183-190``);
no dataset is involved.  Values are drawn in float32 with
``numpy.random.default_rng(seed)`` and then cast to the config's input dtype; the
checker consumes the cast values.

Distributions (shared by every config):
  x ~ N(0,1) (b,L,H,P);  dt_raw ~ N(0,1) (b,L,H);
  dt0 = exp(U[ln 1e-3, ln 0.1]) per head, dt_bias = dt0 + log(-expm1(-dt0))
  (inverse softplus, the Mamba2 initialisation of ``modules/mamba2.py:608-616``);
  A = -exp(ln U[1,16]) per head;  B, C ~ N(0,1) (b,L,G,N);  D = 1 per head;
  dt_softplus on, dt_limit (0, inf).
"""

from __future__ import annotations

import dataclasses
import math

import numpy as np


@dataclasses.dataclass(frozen=True)
class SsdConfig:
    name: str
    batch: int
    seqlen: int
    nheads: int
    headdim: int
    ngroups: int
    dstate: int
    chunk_size: int
    dtype: str = "bf16"          # "f32" or "bf16": x, dt, B, C, z
    has_z: bool = False
    has_init: bool = False
    return_final: bool = False
    varlen_seqs: int = 0         # >0: packed varlen row with this many sequences
    varlen_range: tuple = (256, 4096)

    @property
    def nchunks(self):
        return -(-self.seqlen // self.chunk_size)

    @property
    def tokens(self):
        return self.batch * self.seqlen


@dataclasses.dataclass(frozen=True)
class SsuConfig:
    name: str
    batch: int
    nheads: int
    headdim: int
    ngroups: int
    dstate: int
    dtype: str = "bf16"          # x, z, dt, B, C; state is always f32
    steps: int = 1000


CONFIGS = {
    "c0": SsdConfig("mamba2-130m", 1, 2048, 24, 64, 1, 128, 256, "f32"),
    "c1": SsdConfig("mamba2-2.7b", 8, 2048, 80, 64, 1, 128, 256, "bf16", has_z=True),
    "c2": SsdConfig("nemotron-h-8b", 1, 4096, 128, 64, 8, 128, 128, "bf16",
                    has_init=True, return_final=True),
    "c3": SsdConfig("nemotron-h-47b-varlen", 1, 32768, 256, 64, 8, 256, 128, "bf16",
                    return_final=True, varlen_seqs=16),
    "c4": SsuConfig("nemotron-h-8b-decode", 256, 128, 64, 8, 128, "bf16"),
}


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` (RNE for bf16); returns float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    if dtype == "f32":
        return a
    u = a.view(np.uint32).astype(np.uint64)
    u = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def varlen_lengths(rng, nseq, total, lo, hi):
    """``nseq`` lengths ~ U[lo, hi], rescaled to sum ``total`` (floor; residual on the last)."""
    raw = rng.integers(lo, hi + 1, size=nseq).astype(np.float64)
    lens = np.floor(raw * (total / raw.sum())).astype(np.int64)
    lens = np.maximum(lens, 1)
    lens[-1] += total - lens.sum()
    assert lens.sum() == total and (lens > 0).all()
    return lens


def make_ssd_inputs(cfg: SsdConfig, seed: int):
    """Return a dict of float32 numpy arrays (already rounded to cfg.dtype) + flags."""
    rng = np.random.default_rng(seed)
    b, L, H, P, G, N = cfg.batch, cfg.seqlen, cfg.nheads, cfg.headdim, cfg.ngroups, cfg.dstate
    f = lambda shape: rng.standard_normal(size=shape, dtype=np.float32)
    x = round_to(f((b, L, H, P)), cfg.dtype)
    dt = round_to(f((b, L, H)), cfg.dtype)
    dt0 = np.exp(rng.uniform(math.log(1e-3), math.log(0.1), size=H))
    dt_bias = (dt0 + np.log(-np.expm1(-dt0))).astype(np.float32)
    A = (-np.exp(np.log(rng.uniform(1.0, 16.0, size=H)))).astype(np.float32)
    Bm = round_to(f((b, L, G, N)), cfg.dtype)
    Cm = round_to(f((b, L, G, N)), cfg.dtype)
    D = np.ones(H, np.float32)
    z = round_to(f((b, L, H, P)), cfg.dtype) if cfg.has_z else None
    init = (0.1 * f((b, H, P, N))).astype(np.float32) if cfg.has_init else None
    seq_idx = cu = None
    if cfg.varlen_seqs:
        assert b == 1
        lens = varlen_lengths(rng, cfg.varlen_seqs, L, *cfg.varlen_range)
        cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        seq_idx = np.repeat(np.arange(len(lens), dtype=np.int32), lens)[None]
    return dict(x=x, dt=dt, A=A, B=Bm, C=Cm, D=D, z=z, dt_bias=dt_bias,
                initial_states=init, seq_idx=seq_idx, cu_seqlens=cu,
                dt_softplus=True, dt_limit=(0.0, math.inf))


def make_ssu_inputs(cfg: SsuConfig, seed: int):
    rng = np.random.default_rng(seed)
    b, H, P, G, N = cfg.batch, cfg.nheads, cfg.headdim, cfg.ngroups, cfg.dstate
    f = lambda shape: rng.standard_normal(size=shape, dtype=np.float32)
    state = (0.1 * f((b, H, P, N))).astype(np.float32)
    x = round_to(f((b, H, P)), cfg.dtype)
    z = round_to(f((b, H, P)), cfg.dtype)
    dt = round_to(f((b, H)), cfg.dtype)
    dt0 = np.exp(rng.uniform(math.log(1e-3), math.log(0.1), size=H))
    dt_bias = (dt0 + np.log(-np.expm1(-dt0))).astype(np.float32)
    A = (-np.exp(np.log(rng.uniform(1.0, 16.0, size=H)))).astype(np.float32)
    Bm = round_to(f((b, G, N)), cfg.dtype)
    Cm = round_to(f((b, G, N)), cfg.dtype)
    D = np.ones(H, np.float32)
    return dict(state=state, x=x, dt=dt, A=A, B=Bm, C=Cm, D=D, z=z, dt_bias=dt_bias,
                dt_softplus=True)


def scaled(cfg: SsdConfig, **kw) -> SsdConfig:
    """A smaller variant of ``cfg`` (for parity tests the checker finishes in seconds)."""
    return dataclasses.replace(cfg, **kw)
