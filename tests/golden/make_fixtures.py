"""Generate the golden fixtures in this directory by running the REFERENCE's own code.

    python tests/golden/make_fixtures.py [--reference PATH]

PATH (default /root/reference, the upstream checkout of AlexG1105/mamba2-jax-pallas) must
hold ``src/mamba2_jax/ops/``.  The four pure-JAX op files there are loaded unmodified, by
file path, with ``tests/golden/jaxshim`` standing in for ``jax`` (JAX is not installable
in this image):

    ops/ssd_naive.py               mamba_chunk_scan_combined_naive  (:325-397)
    ops/selective_state_update.py  selective_state_update           (:22-123)
    ops/rms_norm.py                rms_norm_gated                   (:15-92)
    ops/causal_conv1d.py           causal_conv1d, causal_conv1d_update

Each op runs with the stand-in in float64 (``ref64``, the tight pin for the float64
oracle) and, for float32 inputs and the small op fixtures, also in float32 as JAX computes
on CPU (``ref32``).  Inputs come from the seeded
generators of ``mamba2_b200.synthetic`` and are stored in the fixture (bf16 cases as
bf16-representable float32 values), so the tests never regenerate them.

The reference's ``ssd_naive`` ignores ``seq_idx``; the packed-varlen fixture is therefore
built from per-sequence runs (each sequence from a zero state), which is the semantics the
kernel path's seq_idx rules compose to.  Each per-sequence run uses chunk_size = the
sequence length, so no padding enters (``ssd_naive`` pads raw dt before the bias, which
decays final states through padded positions; the kernel path pads processed dt with 0,
``chunk_cumsum_fwd.py:228-231``).  For the same reason the ragged fixture ``c0r`` stores
the final states of a run with chunk_size = L (``final_kernel``) beside the padded run's
(``final``).

Writes ssd_fixtures.npz, ssu_fixtures.npz, norm_fixtures.npz, conv_fixtures.npz.
"""
from __future__ import annotations

import argparse
import importlib.util
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "mamba2-jax-pallas_b200"))

from mamba2_b200 import synthetic as S  # noqa: E402

OPS = ("ssd_naive", "selective_state_update", "rms_norm", "causal_conv1d")


def load_reference(ref_root: str, f64: bool):
    """Load the reference's op modules with the NumPy stand-in for jax (fresh imports)."""
    os.environ["JAXSHIM_F64"] = "1" if f64 else "0"
    for k in [k for k in sys.modules if k == "jax" or k.startswith("jax.")]:
        del sys.modules[k]
    shim = os.path.join(HERE, "jaxshim")
    if shim not in sys.path:
        sys.path.insert(0, shim)
    import jax  # noqa: F401  (the stand-in)
    mods = {}
    for name in OPS:
        path = os.path.join(ref_root, "src", "mamba2_jax", "ops", name + ".py")
        spec = importlib.util.spec_from_file_location(f"refops_{name}_{int(f64)}", path)
        m = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(m)
        mods[name] = m
    return mods


def cast(a, f64):
    if a is None:
        return None
    a = np.asarray(a)
    if a.dtype.kind == "f":
        return a.astype(np.float64 if f64 else np.float32)
    return a


# ---------------------------------------------------------------------------
# cases
# ---------------------------------------------------------------------------

def ssd_cases():
    """(name, config, seed, D override, z, init, final, chunk runs)"""
    cases = {}
    c = S.scaled(S.CONFIGS["c0"], seqlen=512, nheads=2)                        # fp32, G=1, Q=256
    cases["c0s"] = (c, 11, {})
    c = S.SsdConfig("c0-ragged", 1, 300, 2, 32, 1, 64, 64, "f32", return_final=True)
    cases["c0r"] = (c, 12, {"D2": True})                                        # ragged L, D (H,P)
    c = S.scaled(S.CONFIGS["c1"], batch=2, seqlen=256, nheads=2)               # bf16, z, Q=256
    cases["c1s"] = (c, 13, {})
    c = S.scaled(S.CONFIGS["c2"], seqlen=384, nheads=4, ngroups=2)             # init + final, G=2
    cases["c2s"] = (c, 14, {})
    return cases


def gen_ssd(ref64, ref32):
    out = {}
    for name, (cfg, seed, opt) in ssd_cases().items():
        inp = S.make_ssd_inputs(cfg, seed)
        if opt.get("D2"):
            rng = np.random.default_rng(seed + 100)
            inp["D"] = rng.standard_normal((cfg.nheads, cfg.headdim)).astype(np.float32)
        keys = ("x", "dt", "A", "B", "C", "D", "z", "dt_bias", "initial_states")
        for k in keys:
            if inp[k] is not None:
                out[f"{name}/{k}"] = inp[k]
        out[f"{name}/meta"] = np.array([cfg.chunk_size, int(cfg.dtype == "bf16")], np.int64)
        for tag, ref, f64 in (("ref64", ref64, True), ("ref32", ref32, False)):
            if tag == "ref32" and cfg.dtype == "bf16":
                continue    # bf16 cases keep the float64 run only (fixture size)
            a = {k: cast(inp[k], f64) for k in keys}
            res = ref["ssd_naive"].mamba_chunk_scan_combined_naive(
                a["x"], a["dt"], a["A"], a["B"], a["C"], cfg.chunk_size, D=a["D"], z=a["z"],
                dt_bias=a["dt_bias"], initial_states=a["initial_states"], dt_softplus=True,
                dt_limit=(0.0, float("inf")), return_final_states=True)
            out[f"{name}/{tag}/out"] = np.asarray(res[0], np.float32)
            out[f"{name}/{tag}/final"] = np.asarray(res[1], np.float32)
            if name == "c0r":
                # same inputs, chunk_size = L: no padded positions, so the final state is the
                # kernel path's (the output does not depend on the chunking)
                r2 = ref["ssd_naive"].mamba_chunk_scan_combined_naive(
                    a["x"], a["dt"], a["A"], a["B"], a["C"], cfg.seqlen, D=a["D"], z=a["z"],
                    dt_bias=a["dt_bias"], initial_states=a["initial_states"], dt_softplus=True,
                    dt_limit=(0.0, float("inf")), return_final_states=True)
                out[f"{name}/{tag}/out_chunkL"] = np.asarray(r2[0], np.float32)
                out[f"{name}/{tag}/final_kernel"] = np.asarray(r2[1], np.float32)
    # packed varlen (c3-shaped: G=1 here to keep the fixture small, N=256, Q=128)
    cfg = S.SsdConfig("c3-packed", 1, 384, 2, 64, 1, 256, 128, "bf16", return_final=True)
    inp = S.make_ssd_inputs(cfg, 15)
    lens = np.array([150, 57, 177], np.int64)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    seq_idx = np.repeat(np.arange(len(lens), dtype=np.int32), lens)[None]
    name = "c3p"
    for k in ("x", "dt", "A", "B", "C", "D", "dt_bias"):
        out[f"{name}/{k}"] = inp[k]
    out[f"{name}/seq_idx"] = seq_idx
    out[f"{name}/cu_seqlens"] = cu
    out[f"{name}/meta"] = np.array([cfg.chunk_size, 1], np.int64)
    for tag, ref, f64 in (("ref64", ref64, True),):
        a = {k: cast(inp[k], f64) for k in ("x", "dt", "A", "B", "C", "D", "dt_bias")}
        outs, finals = [], []
        for s, e in zip(cu[:-1], cu[1:]):
            sl = slice(int(s), int(e))
            o, f = ref["ssd_naive"].mamba_chunk_scan_combined_naive(
                a["x"][:, sl], a["dt"][:, sl], a["A"], a["B"][:, sl], a["C"][:, sl], int(e - s),
                D=a["D"], dt_bias=a["dt_bias"], dt_softplus=True, dt_limit=(0.0, float("inf")),
                return_final_states=True)
            outs.append(np.asarray(o, np.float32))
            finals.append(np.asarray(f, np.float32)[0])
        out[f"{name}/{tag}/out"] = np.concatenate(outs, axis=1)
        out[f"{name}/{tag}/varlen_states"] = np.stack(finals)
    return out


def gen_ssu(ref64, ref32):
    out = {}
    cfg = S.SsuConfig("c4s", 2, 8, 64, 2, 64)
    u = S.make_ssu_inputs(cfg, 21)
    keys = ("state", "x", "dt", "A", "B", "C", "D", "z", "dt_bias")
    for k in keys:
        out[f"c4s/{k}"] = u[k]
    # the broadcast-free variant: dt (b,H,P), A (H,P,N), D and dt_bias (H,P)
    rng = np.random.default_rng(22)
    b, H, P, G, N = cfg.batch, cfg.nheads, cfg.headdim, cfg.ngroups, cfg.dstate
    v = dict(u)
    v["dt"] = S.round_to(rng.standard_normal((b, H, P)).astype(np.float32), "bf16")
    v["A"] = (-np.exp(rng.uniform(0.0, math.log(16.0), (H, P, N)))).astype(np.float32)
    v["D"] = rng.standard_normal((H, P)).astype(np.float32)
    v["dt_bias"] = (0.5 * rng.standard_normal((H, P)) - 3.0).astype(np.float32)
    for k in keys:
        if k != "state":            # shared with c4s
            out[f"c4v/{k}"] = v[k]
    for case, inp in (("c4s", u), ("c4v", v)):
        for tag, ref, f64 in (("ref64", ref64, True), ("ref32", ref32, False)):
            a = {k: cast(inp[k], f64) for k in keys}
            st, o = ref["selective_state_update"].selective_state_update(
                a["state"], a["x"], a["dt"], a["A"], a["B"], a["C"], D=a["D"], z=a["z"],
                dt_bias=a["dt_bias"], dt_softplus=True)
            out[f"{case}/{tag}/state"] = np.asarray(st, np.float32)
            out[f"{case}/{tag}/out"] = np.asarray(o, np.float32)
    return out


def gen_norm(ref64, ref32):
    out = {}
    rng = np.random.default_rng(31)
    y = rng.standard_normal((2, 8, 2048)).astype(np.float32)
    z = S.round_to(rng.standard_normal((2, 8, 2048)).astype(np.float32), "bf16")
    w = (1.0 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    out["y"], out["z"], out["w"] = y, z, w
    for case, gs, nbg, usez in (("g256", 256, True, True), ("g256_gate_first", 256, False, True),
                                ("full", None, True, True), ("g1024_noz", 1024, True, False)):
        for tag, ref, f64 in (("ref64", ref64, True), ("ref32", ref32, False)):
            o = ref["rms_norm"].rms_norm_gated(cast(y, f64), cast(w, f64), z=cast(z, f64) if usez else None,
                                               eps=1e-5, group_size=gs, norm_before_gate=nbg)
            out[f"{case}/{tag}/out"] = np.asarray(o, np.float32)
    return out


def gen_conv(ref64, ref32):
    out = {}
    rng = np.random.default_rng(41)
    x = S.round_to(rng.standard_normal((2, 64, 96)).astype(np.float32), "bf16")
    w = S.round_to((0.5 * rng.standard_normal((64, 4))).astype(np.float32), "bf16")
    bias = rng.standard_normal(64).astype(np.float32)
    seq = np.concatenate([np.zeros(30, np.int32), np.ones(3, np.int32), np.full(63, 2, np.int32)])
    seq_idx = np.stack([seq, np.zeros(96, np.int32)])
    state = S.round_to(rng.standard_normal((2, 64, 4)).astype(np.float32), "bf16")
    xn = S.round_to(rng.standard_normal((2, 64)).astype(np.float32), "bf16")
    out.update(x=x, w=w, bias=bias, seq_idx=seq_idx, state=state, x_new=xn)
    for tag, ref, f64 in (("ref64", ref64, True), ("ref32", ref32, False)):
        m = ref["causal_conv1d"]
        out[f"plain/{tag}/out"] = np.asarray(m.causal_conv1d(cast(x, f64), cast(w, f64)), np.float32)
        out[f"silu_bias/{tag}/out"] = np.asarray(
            m.causal_conv1d(cast(x, f64), cast(w, f64), bias=cast(bias, f64), activation="silu"), np.float32)
        out[f"seq/{tag}/out"] = np.asarray(
            m.causal_conv1d(cast(x, f64), cast(w, f64), bias=cast(bias, f64), activation="silu",
                            seq_idx=seq_idx), np.float32)
        ns, o = m.causal_conv1d_update(cast(xn, f64), cast(state, f64), cast(w, f64), bias=cast(bias, f64),
                                       activation="silu")
        out[f"update/{tag}/state"] = np.asarray(ns, np.float32)
        out[f"update/{tag}/out"] = np.asarray(o, np.float32)
    return out


def pack(a):
    """float32 arrays whose values are all bf16-representable are stored as their upper 16
    bits (key suffix "@bf16"); tests/fixtures.py restores them."""
    a = np.asarray(a)
    if a.dtype == np.float32:
        u = np.ascontiguousarray(a).view(np.uint32)
        if not (u & 0xFFFF).any():
            return (u >> 16).astype(np.uint16), True
    return a, False


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    ref64 = load_reference(args.reference, True)
    ref32 = load_reference(args.reference, False)
    for fname, fn in (("ssd_fixtures.npz", gen_ssd), ("ssu_fixtures.npz", gen_ssu),
                      ("norm_fixtures.npz", gen_norm), ("conv_fixtures.npz", gen_conv)):
        d = fn(ref64, ref32)
        d = {k: pack(v) for k, v in d.items()}
        np.savez_compressed(os.path.join(HERE, fname), **{(k + "@bf16" if p else k): v for k, (v, p) in d.items()})
        print(fname, sum(v.nbytes for v, _ in d.values()) // 1024, "KiB raw")


if __name__ == "__main__":
    main()
