"""CPU checks of the oracle (oracle/ssd_ref.py) against the reference's own known-answer
procedures, restated, and against size-independent properties of the recurrence.

The reference ships no golden vectors and cannot run here (no JAX), so these pins are
procedural: each test names the reference test it restates.
"""
import math

import numpy as np
import pytest

from oracle import ssd_ref as R
from mamba2_b200 import synthetic as S


def _rng(seed):
    return np.random.default_rng(seed)


# ---- tests/test_mamba2_ops.py:25-65 (basic step, no softplus) -----------------------
def test_ssu_known_answer_basic():
    rng = _rng(42)
    b, H, P, N, G = 2, 4, 8, 16, 2
    state = rng.standard_normal((b, H, P, N))
    x = rng.standard_normal((b, H, P))
    dt = rng.uniform(0.01, 0.1, (b, H))
    A = -np.abs(rng.standard_normal(H))
    B = rng.standard_normal((b, G, N))
    C = rng.standard_normal((b, G, N))
    new, out = R.selective_state_update(state, x, dt, A, B, C)
    Be, Ce = np.repeat(B, H // G, 1), np.repeat(C, H // G, 1)
    dA = np.exp(dt[:, :, None, None] * A[None, :, None, None])
    ref = state * dA + dt[:, :, None, None] * Be[:, :, None, :] * x[..., None]
    assert np.max(np.abs(new - ref)) < 1e-12
    assert np.max(np.abs(out - (ref * Ce[:, :, None, :]).sum(-1))) < 1e-12


# ---- tests/test_mamba2_ops.py:68-112 (D, z, dt_bias, softplus) ------------------------
def test_ssu_known_answer_full():
    rng = _rng(123)
    b, H, P, N, G = 2, 4, 8, 16, 1
    state = rng.standard_normal((b, H, P, N))
    x = rng.standard_normal((b, H, P))
    dt = rng.standard_normal((b, H))
    A = -np.abs(rng.standard_normal(H))
    B, C = rng.standard_normal((b, G, N)), rng.standard_normal((b, G, N))
    D, z, bias = rng.standard_normal(H), rng.standard_normal((b, H, P)), rng.standard_normal(H)
    new, out = R.selective_state_update(state, x, dt, A, B, C, D=D, z=z, dt_bias=bias, dt_softplus=True)
    dtr = np.log1p(np.exp(dt + bias))
    Be, Ce = np.repeat(B, H, 1), np.repeat(C, H, 1)
    ref = state * np.exp(dtr[:, :, None, None] * A[None, :, None, None]) \
        + dtr[:, :, None, None] * Be[:, :, None, :] * x[..., None]
    o = (ref * Ce[:, :, None, :]).sum(-1) + D[None, :, None] * x
    o = o * (z / (1 + np.exp(-z)))
    assert np.max(np.abs(new - ref)) < 1e-12
    assert np.max(np.abs(out - o)) < 1e-12


# ---- state passing: sequential loop (tests/test_state_passing_and_bmm.py:92-138)
#      == pairwise-decay form (ssd_naive.py:135-182) ------------------------------------
@pytest.mark.parametrize("b,nc,H,D,init", [(1, 4, 1, 128, False), (2, 8, 4, 128, True),
                                           (1, 4, 2, 200, True), (2, 8, 4, 300, True)])
def test_state_passing_forms_agree(b, nc, H, D, init):
    rng = _rng(7)
    st = rng.standard_normal((b, nc, H, D))
    dA = -rng.uniform(0.0, 3.0, (b, H, nc))
    ini = rng.standard_normal((b, H, D)) if init else None
    o1, f1 = R.state_passing(st, dA, ini)
    o2, f2 = R.state_passing_pairwise(st, dA, ini)
    np.testing.assert_allclose(o1, o2, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(f1, f2, rtol=1e-12, atol=1e-12)


def _small_inputs(seed=0, b=2, L=200, H=4, P=8, G=2, N=16, Q=64, dtype="f32", z=True, init=True):
    cfg = S.SsdConfig("t", b, L, H, P, G, N, Q, dtype, has_z=z, has_init=init, return_final=True)
    return cfg, S.make_ssd_inputs(cfg, seed)


def _run(inp, Q, **kw):
    return R.ssd_combined(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], Q, D=inp["D"],
                          z=kw.pop("z", inp["z"]), dt_bias=inp["dt_bias"],
                          initial_states=kw.pop("init", inp["initial_states"]),
                          dt_softplus=True, **kw)


# ---- prefill == decode loop (tests/test_mamba2_vs_torch.py:312-408, at the SSD level) ---
def test_prefill_final_state_equals_decode_loop():
    cfg, inp = _small_inputs(L=96, Q=32, z=False)
    out, final = _run(inp, 32, return_final_states=True)
    state = inp["initial_states"].astype(np.float64)
    outs = []
    for t in range(cfg.seqlen):
        state, o = R.selective_state_update(
            state, inp["x"][:, t], inp["dt"][:, t], inp["A"], inp["B"][:, t], inp["C"][:, t],
            D=inp["D"], dt_bias=inp["dt_bias"], dt_softplus=True)
        outs.append(o)
    # chunk_cumsum's thresholded softplus equals jax.nn.softplus below the threshold
    np.testing.assert_allclose(final, state, rtol=1e-9, atol=1e-9)
    np.testing.assert_allclose(out, np.stack(outs, 1), rtol=1e-9, atol=1e-9)


# ---- split-resume == full ------------------------------------------------------------
@pytest.mark.parametrize("split", [64, 100])
def test_split_resume(split):
    cfg, inp = _small_inputs(L=200, Q=64)
    out, final = _run(inp, 64, return_final_states=True)
    first = {k: (v[:, :split] if k in ("x", "dt", "B", "C", "z") else v) for k, v in inp.items()}
    second = {k: (v[:, split:] if k in ("x", "dt", "B", "C", "z") else v) for k, v in inp.items()}
    o1, f1 = _run(first, 64, return_final_states=True)
    o2, f2 = _run(second, 64, init=f1, return_final_states=True)
    np.testing.assert_allclose(np.concatenate([o1, o2], 1), out, rtol=1e-9, atol=1e-9)
    np.testing.assert_allclose(f2, final, rtol=1e-9, atol=1e-9)


# ---- packed varlen == per-sequence (the seq_idx rules A7-A9 compose correctly) --------
@pytest.mark.parametrize("lens,Q", [([200, 312], 64), ([64, 192, 256], 64), ([64, 64, 64, 64], 64),
                                    ([1, 70, 33, 152], 32), ([256], 64)])
def test_packed_equals_per_sequence(lens, Q):
    T = sum(lens)
    cfg, inp = _small_inputs(b=1, L=T, Q=Q, init=False)
    cu = np.concatenate([[0], np.cumsum(lens)])
    seq = np.repeat(np.arange(len(lens)), lens)[None]
    out, final, varlen = _run(inp, Q, seq_idx=seq, cu_seqlens=cu, return_final_states=True,
                              return_varlen_states=True)
    for s in range(len(lens)):
        a, e = cu[s], cu[s + 1]
        sub = {k: (v[:, a:e] if k in ("x", "dt", "B", "C", "z") else v) for k, v in inp.items()}
        o, f = _run(sub, Q, return_final_states=True)
        np.testing.assert_allclose(out[:, a:e], o, rtol=1e-9, atol=1e-9)
        np.testing.assert_allclose(varlen[s], f[0], rtol=1e-9, atol=1e-9)
    np.testing.assert_allclose(final[0], varlen[-1], rtol=1e-9, atol=1e-9)


# ---- mask rules: vectorised == literal per-element statement ---------------------------
def test_masks_literal():
    rng = _rng(3)
    b, L, Q = 2, 300, 64
    seq = np.sort(rng.integers(0, 5, (b, L)), axis=1)
    seq[1] += 1  # first id != 0 exercises the prev=0 quirk
    nc = math.ceil(L / Q)
    pad = lambda i, t: seq[i, t] if t < L else -1
    m7 = R.mask_chunk_state(seq, Q)
    m8 = R.mask_bmm(seq, Q)
    m9 = R.mask_scan_state(seq, Q)
    keep = R.state_passing_keep(seq, Q)
    for i in range(b):
        prev_end = 0
        for c in range(nc):
            last = seq[i, min((c + 1) * Q, L) - 1]
            prev = 0 if c == 0 else seq[i, c * Q - 1]
            assert keep[i, c] == (last == prev_end)
            prev_end = last
            for m in range(Q):
                assert m7[i, c, m] == (last >= 0 and pad(i, c * Q + m) == last)
                assert m9[i, c, m] == (pad(i, c * Q + m) == prev)
                for n in range(0, Q, 7):
                    assert m8[i, c, m, n] == (pad(i, c * Q + m) == pad(i, c * Q + n))


def test_pad_modes_differ_only_in_tail():
    cfg, inp = _small_inputs(L=200, Q=64)
    (o1, f1), i1 = _run(inp, 64, return_final_states=True, return_intermediates=True)
    (o2, f2), i2 = _run(inp, 64, return_final_states=True, return_intermediates=True, pad_mode="naive")
    np.testing.assert_allclose(o1, o2, rtol=1e-12, atol=1e-12)
    assert not np.allclose(f1, f2)
    np.testing.assert_array_equal(i1["dt_out"][:, :, :-1], i2["dt_out"][:, :, :-1])


def test_round_bf16():
    v = np.array([1.0, 1.00390625, 1.005859375, -3.14159, 65504.0, 1e-40], np.float32)
    r = R.round_bf16(v)
    assert r[0] == 1.0 and r[1] == 1.0  # tie to even
    assert r[2] == 1.0078125
    np.testing.assert_array_equal(r, S.round_to(v, "bf16").astype(np.float64))
