"""The float64 oracle against golden outputs of the REFERENCE's own code.

tests/golden/*.npz were produced by tests/golden/make_fixtures.py, which runs the
reference's unmodified ops/ssd_naive.py, ops/selective_state_update.py, ops/rms_norm.py
and ops/causal_conv1d.py on a NumPy stand-in for jax, in float64 (``ref64``) and float32
(``ref32``).  Bounds: 1e-6 rel-L2 against ref64 (the fixture stores float32, about 6e-8
of rounding) and 2e-5 against ref32 (the reference's own float32 arithmetic).
"""
import numpy as np
import pytest

import fixtures as F
from oracle import ssd_ref as R

TOL64, TOL32 = 1e-6, 2e-5
SSD = F.load("ssd")


def _tags(c):
    return [t for t in ("ref64", "ref32") if f"{t}/out" in c]


def _tol(tag):
    return TOL64 if tag == "ref64" else TOL32


@pytest.mark.parametrize("name", ["c0s", "c1s", "c2s"])
def test_ssd_combined_matches_reference(name):
    c = F.case(SSD, name)
    Q = int(c["meta"][0])
    out, final = R.ssd_combined(c["x"], c["dt"], c["A"], c["B"], c["C"], Q, D=c["D"], z=c.get("z"),
                                dt_bias=c["dt_bias"], initial_states=c.get("initial_states"),
                                dt_softplus=True, return_final_states=True, pad_mode="naive")
    for tag in _tags(c):
        assert R.rel_l2(out, c[f"{tag}/out"]) <= _tol(tag), tag
        assert R.rel_l2(final, c[f"{tag}/final"]) <= _tol(tag), tag


def test_ssd_ragged_both_pad_modes():
    """L = 300 with chunk 64: the output is independent of the padding rule; the final state
    follows ssd_naive's padded-raw-dt rule in pad_mode="naive" and the kernel path's (no
    padded positions: the reference run with chunk_size = L) in pad_mode="kernel"."""
    c = F.case(SSD, "c0r")
    Q = int(c["meta"][0])
    kw = dict(D=c["D"], dt_bias=c["dt_bias"], dt_softplus=True, return_final_states=True)
    out_n, fin_n = R.ssd_combined(c["x"], c["dt"], c["A"], c["B"], c["C"], Q, pad_mode="naive", **kw)
    out_k, fin_k = R.ssd_combined(c["x"], c["dt"], c["A"], c["B"], c["C"], Q, pad_mode="kernel", **kw)
    for tag in _tags(c):
        tol = _tol(tag)
        assert R.rel_l2(out_n, c[f"{tag}/out"]) <= tol
        assert R.rel_l2(out_k, c[f"{tag}/out_chunkL"]) <= tol
        assert R.rel_l2(fin_n, c[f"{tag}/final"]) <= tol
        assert R.rel_l2(fin_k, c[f"{tag}/final_kernel"]) <= tol
    # and the two reference final states really differ (the pin is not vacuous)
    assert R.rel_l2(c["ref64/final"], c["ref64/final_kernel"]) > 1e-3


def test_ssd_packed_varlen_matches_per_sequence_reference():
    """Packed row with seq_idx resets: outputs and varlen states equal the reference run on
    each sequence alone (from a zero state)."""
    c = F.case(SSD, "c3p")
    Q = int(c["meta"][0])
    out, vs = R.ssd_combined(c["x"], c["dt"], c["A"], c["B"], c["C"], Q, D=c["D"], dt_bias=c["dt_bias"],
                             seq_idx=c["seq_idx"], cu_seqlens=c["cu_seqlens"], dt_softplus=True,
                             return_varlen_states=True)
    assert R.rel_l2(out, c["ref64/out"]) <= TOL64
    assert R.rel_l2(vs, c["ref64/varlen_states"]) <= TOL64


@pytest.mark.parametrize("name", ["c4s", "c4v"])
def test_selective_state_update_matches_reference(name):
    d = F.load("ssu")
    c = F.case(d, name)
    state = d["c4s/state"]
    st, out = R.selective_state_update(state, c["x"], c["dt"], c["A"], c["B"], c["C"], D=c["D"], z=c["z"],
                                       dt_bias=c["dt_bias"], dt_softplus=True)
    for tag in ("ref64", "ref32"):
        assert R.rel_l2(st, c[f"{tag}/state"]) <= _tol(tag)
        assert R.rel_l2(out, c[f"{tag}/out"]) <= _tol(tag)


@pytest.mark.parametrize("case,gs,nbg,usez", [("g256", 256, True, True), ("g256_gate_first", 256, False, True),
                                              ("full", None, True, True), ("g1024_noz", 1024, True, False)])
def test_rms_norm_gated_matches_reference(case, gs, nbg, usez):
    d = F.load("norm")
    o = R.rms_norm_gated(d["y"], d["w"], z=d["z"] if usez else None, eps=1e-5, group_size=gs, norm_before_gate=nbg)
    for tag in ("ref64", "ref32"):
        assert R.rel_l2(o, d[f"{case}/{tag}/out"]) <= _tol(tag)


def test_causal_conv1d_matches_reference():
    d = F.load("conv")
    x, w, b, seq = d["x"], d["w"], d["bias"], d["seq_idx"]
    for tag in ("ref64", "ref32"):
        tol = _tol(tag)
        assert R.rel_l2(R.causal_conv1d(x, w), d[f"plain/{tag}/out"]) <= tol
        assert R.rel_l2(R.causal_conv1d(x, w, b, "silu"), d[f"silu_bias/{tag}/out"]) <= tol
        assert R.rel_l2(R.causal_conv1d(x, w, b, "silu", seq_idx=seq), d[f"seq/{tag}/out"]) <= tol
        ns, o = R.causal_conv1d_update(d["x_new"], d["state"], w, b, "silu")
        assert R.rel_l2(ns, d[f"update/{tag}/state"]) <= tol
        assert R.rel_l2(o, d[f"update/{tag}/out"]) <= tol


def test_fixtures_are_bf16_where_the_case_is_bf16():
    """bf16 cases hold bf16-representable inputs, so the CUDA path reads the same values."""
    for name in ("c1s", "c2s", "c3p"):
        c = F.case(SSD, name)
        for k in ("x", "B", "C"):
            u = np.ascontiguousarray(c[k], np.float32).view(np.uint32)
            assert not (u & 0xFFFF).any(), (name, k)


def test_recurrent_scan_oracle_matches_reference():
    """oracle/ssd_scan.c (the token-by-token recurrence used by the full-size GPU tests)
    against the same reference fixtures."""
    from oracle import scan
    for name in ("c0s", "c1s", "c2s"):
        c = F.case(SSD, name)
        o, f, _ = scan.ssd_scan(c["x"], c["dt"], c["A"], c["B"], c["C"], D=c["D"], z=c.get("z"),
                                dt_bias=c["dt_bias"], initial_states=c.get("initial_states"), dt_softplus=True)
        assert R.rel_l2(o, c["ref64/out"]) <= TOL64 and R.rel_l2(f, c["ref64/final"]) <= TOL64, name
    c = F.case(SSD, "c0r")
    o, f, _ = scan.ssd_scan(c["x"], c["dt"], c["A"], c["B"], c["C"], D=c["D"], dt_bias=c["dt_bias"], dt_softplus=True)
    assert R.rel_l2(o, c["ref64/out"]) <= TOL64 and R.rel_l2(f, c["ref64/final_kernel"]) <= TOL64
    c = F.case(SSD, "c3p")
    o, _, v = scan.ssd_scan(c["x"], c["dt"], c["A"], c["B"], c["C"], D=c["D"], dt_bias=c["dt_bias"],
                            dt_softplus=True, seq_idx=c["seq_idx"], cu_seqlens=c["cu_seqlens"])
    assert R.rel_l2(o, c["ref64/out"]) <= TOL64 and R.rel_l2(v, c["ref64/varlen_states"]) <= TOL64


def test_recurrent_scan_oracle_matches_chunked_oracle_with_resets():
    """The recurrence and the chunked restatement agree on packed rows whose first id is
    not 0 (the initial state is then dropped), with z, D per (head, column) and a head
    subset."""
    from oracle import scan
    from mamba2_b200 import synthetic as S
    cfg = S.SsdConfig("r", 2, 200, 4, 16, 2, 32, 64, "f32", has_z=True, has_init=True, return_final=True)
    inp = S.make_ssd_inputs(cfg, 3)
    D2 = np.random.default_rng(4).standard_normal((4, 16)).astype(np.float32)
    seq = np.zeros((2, 200), np.int32)
    seq[0, 70:] = 1
    seq[0, 71:] = 2
    seq[1] = 5
    seq[1, 130:] = 6
    kw = dict(D=D2, z=inp["z"], dt_bias=inp["dt_bias"], initial_states=inp["initial_states"], seq_idx=seq,
              dt_softplus=True)
    o_ref, f_ref = R.ssd_combined(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], 64,
                                  return_final_states=True, **kw)
    o, f, _ = scan.ssd_scan(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], heads=(2, 4), **kw)
    assert R.rel_l2(o[:, :, 2:], o_ref[:, :, 2:]) <= 1e-10
    assert R.rel_l2(f[:, 2:], f_ref[:, 2:]) <= 1e-10
    assert not o[:, :, :2].any()
