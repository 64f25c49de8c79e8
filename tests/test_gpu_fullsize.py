"""Full-size parity: the BASELINE configurations c0-c3 at their own sizes against the float64
token-by-token recurrence (oracle/ssd_scan.c, itself pinned to the reference's outputs in
tests/test_golden.py), one head group at a time.

Inputs follow mamba2_b200.synthetic's distributions but are drawn on the GPU (seeded torch
generator) and copied to the host as float32, because generating c3's 2 GB of x with NumPy
takes minutes.  Bounds: rel-L2 <= 1e-4 for float32 inputs, 1e-2 for
bf16 inputs, per head group, for out, final states and varlen states.
"""
import math

import numpy as np
import pytest
import torch

from gpu_util import TOL, rel_l2
from mamba2_b200 import synthetic as S

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mamba2_b200._lib as L
    L.load()


def gpu_inputs(cfg, seed):
    """Device tensors with the synthetic configs' distributions (values rounded to the
    input dtype on the device)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    rng = np.random.default_rng(seed)
    b, L, H, P, G, N = cfg.batch, cfg.seqlen, cfg.nheads, cfg.headdim, cfg.ngroups, cfg.dstate
    tdt = torch.bfloat16 if cfg.dtype == "bf16" else torch.float32
    rn = lambda *shape: torch.randn(shape, generator=g, device="cuda").to(tdt)
    d = dict(x=rn(b, L, H, P), dt=rn(b, L, H), B=rn(b, L, G, N), C=rn(b, L, G, N))
    d["z"] = rn(b, L, H, P) if cfg.has_z else None
    dt0 = np.exp(rng.uniform(math.log(1e-3), math.log(0.1), size=H))
    d["dt_bias"] = torch.from_numpy((dt0 + np.log(-np.expm1(-dt0))).astype(np.float32)).cuda()
    d["A"] = torch.from_numpy((-np.exp(np.log(rng.uniform(1.0, 16.0, size=H)))).astype(np.float32)).cuda()
    d["D"] = torch.ones(H, device="cuda")
    d["initial_states"] = (0.1 * torch.randn((b, H, P, N), generator=g, device="cuda")) if cfg.has_init else None
    d["seq_idx"] = d["cu_seqlens"] = None
    if cfg.varlen_seqs:
        lens = S.varlen_lengths(rng, cfg.varlen_seqs, L, *cfg.varlen_range)
        cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        d["cu_seqlens"] = torch.from_numpy(cu).cuda()
        d["seq_idx"] = torch.from_numpy(np.repeat(np.arange(len(lens), dtype=np.int32), lens)[None]).cuda()
    return d


def host(t, sl=None):
    if t is None:
        return None
    if sl is not None:
        t = t[sl]
    return t.float().cpu().numpy() if t.is_floating_point() else t.cpu().numpy()


def check_by_group(cfg, d, res, varlen):
    """Compare every head group of the GPU result with the recurrence on that group alone."""
    from oracle import scan
    out, final = res[0], res[1]
    vs = res[2] if varlen else None
    H, G = cfg.nheads, cfg.ngroups
    r = H // G
    tol = TOL[cfg.dtype]
    seq, cu = host(d["seq_idx"]), host(d["cu_seqlens"])
    worst = 0.0
    for g in range(G):
        hs = slice(g * r, (g + 1) * r)
        o, f, v = scan.ssd_scan(
            host(d["x"], (slice(None), slice(None), hs)), host(d["dt"], (slice(None), slice(None), hs)),
            host(d["A"], hs), host(d["B"], (slice(None), slice(None), slice(g, g + 1))),
            host(d["C"], (slice(None), slice(None), slice(g, g + 1))), D=host(d["D"], hs),
            z=host(d["z"], (slice(None), slice(None), hs)), dt_bias=host(d["dt_bias"], hs),
            initial_states=host(d["initial_states"], (slice(None), hs)), seq_idx=seq, cu_seqlens=cu,
            dt_softplus=True)
        e = [rel_l2(out[:, :, hs], o), rel_l2(final[:, hs], f)]
        if varlen:
            e.append(rel_l2(vs[:, hs], v))
        assert max(e) <= tol, f"{cfg.name} group {g}: rel-L2 {e} > {tol}"
        worst = max(worst, *e)
    return worst


@pytest.mark.parametrize("key", ["c0", "c1", "c2", "c3"])
def test_full_size_vs_recurrence(key):
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    cfg = S.CONFIGS[key]
    d = gpu_inputs(cfg, 7000 + int(key[1]))
    varlen = d["cu_seqlens"] is not None
    res = mamba_chunk_scan_combined_fwd(
        d["x"], d["dt"], d["A"], d["B"], d["C"], cfg.chunk_size, D=d["D"], z=d["z"], dt_bias=d["dt_bias"],
        initial_states=d["initial_states"], seq_idx=d["seq_idx"], cu_seqlens=d["cu_seqlens"],
        dt_softplus=True, return_final_states=True, return_varlen_states=varlen)
    torch.cuda.synchronize()
    assert all(torch.isfinite(t).all() for t in res)
    worst = check_by_group(cfg, d, res, varlen)
    print(f"{key}: worst rel-L2 over groups {worst:.3e}")
