"""CPU restatement of the reference Mamba2 SSD forward and decode step (NumPy, float64).

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA path: only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference
arm may import it.  The product path (``mamba2_b200``) never calls it and has no
CPU fallback.

Parity status: pinned to the reference's own outputs.  JAX cannot be installed in this
environment, so ``tests/golden/make_fixtures.py`` runs the reference's unmodified
``ops/ssd_naive.py``, ``ops/selective_state_update.py``, ``ops/rms_norm.py`` and
``ops/causal_conv1d.py`` on a NumPy stand-in for ``jax`` (``tests/golden/jaxshim``) and
commits the results as fixtures; ``tests/test_golden.py`` checks this module against them
(rel-L2 <= 1e-6 against the reference's float64 run, 2e-5 against its float32 run).  The
seq_idx rules, which ``ssd_naive`` does not implement, are pinned through per-sequence
reference runs of a packed row and by restating the reference's known-answer procedures
(decode-step hand formula of ``tests/test_mamba2_ops.py:25-112``; the sequential
state-passing loop of ``tests/test_state_passing_and_bmm.py:92-138``; the per-sequence
varlen loop of ``tests/test_chunk_scan_and_varlen.py:504-589``), plus size-independent
properties (packed == per-sequence, prefill == decode loop, split-resume == full).

Every array is float64 unless noted.  Shapes follow the reference:
x (b,L,H,P), dt (b,L,H), A (H,), B/C (b,L,G,N), D (H,) or (H,P), z (b,L,H,P),
dt_bias (H,), initial_states (b,H,P,N), seq_idx (b,L) int, cu_seqlens (S+1,) int.
Head h uses group ``h // (H // G)`` (``src/mamba2_jax/ops/ssd_naive.py:96-99``).
"""

from __future__ import annotations

import math

import numpy as np

F64 = np.float64


def _f(a):
    return None if a is None else np.asarray(a, dtype=F64)


def softplus_thr20(v):
    """``chunk_cumsum_fwd.py:223-225``: v if v > 20 else log1p(exp(v))."""
    v = np.asarray(v, dtype=F64)
    safe = np.where(v <= 20.0, v, 0.0)
    return np.where(v <= 20.0, np.log1p(np.exp(safe)), v)


def softplus(v):
    """``jax.nn.softplus`` (``selective_state_update.py:76``): log(1 + exp(v)), stable form."""
    v = np.asarray(v, dtype=F64)
    return np.logaddexp(v, 0.0)


def silu(v):
    return v / (1.0 + np.exp(-v))


# ---------------------------------------------------------------------------
# A2  chunk_cumsum
# ---------------------------------------------------------------------------

def chunk_cumsum(dt, A, chunk_size, dt_bias=None, dt_softplus=False,
                 dt_limit=(0.0, math.inf), pad_mode="kernel"):
    """``ssd_naive.py:26-70`` (order: dt*A then cumsum, ``:67-68``) with the softplus of
    ``chunk_cumsum_fwd.py:223-225``.

    ``pad_mode="kernel"`` zero-pads *after* bias/softplus/clip, as the kernel path
    does (``chunk_cumsum_fwd.py:221-231``): padded positions get dt_out = 0.
    ``pad_mode="naive"`` pads raw dt with zeros *before* bias/softplus, as
    ``ssd_naive.py:46-64`` does, so padded positions get dt_out = softplus(bias).
    The two differ only when L % Q != 0, and then only in dt_out/dA_cumsum at the
    padded tail and in final_states.
    Returns dA_cumsum, dt_out: (b, H, nc, Q).
    """
    dt = _f(dt)
    A = _f(A)
    b, L, H = dt.shape
    nc = -(-L // chunk_size)
    pad = nc * chunk_size - L

    def proc(v):
        if dt_bias is not None:
            v = v + _f(dt_bias)[None, None, :]
        if dt_softplus:
            v = softplus_thr20(v)
        return np.clip(v, dt_limit[0], dt_limit[1])

    if pad_mode == "naive":
        dtp = proc(np.pad(dt, ((0, 0), (0, pad), (0, 0))))
    else:
        dtp = np.pad(proc(dt), ((0, 0), (0, pad), (0, 0)))
    dt_out = dtp.reshape(b, nc, chunk_size, H).transpose(0, 3, 1, 2)
    dA = dt_out * A[None, :, None, None]
    return np.cumsum(dA, axis=-1), dt_out


# ---------------------------------------------------------------------------
# seq_idx rules (A7-A9)
# ---------------------------------------------------------------------------

def _pad_seq(seq_idx, total):
    seq_idx = np.asarray(seq_idx, dtype=np.int64)
    L = seq_idx.shape[1]
    return np.pad(seq_idx, ((0, 0), (0, total - L)), constant_values=-1)


def chunk_end_seq(seq_idx, chunk_size):
    """seq id at the last valid position of each chunk: ``seq_idx[min((c+1)Q, L) - 1]``
    (``chunk_state_fwd.py:257-260``; ``state_passing_fwd.py:209-212``).  (b, nc)."""
    seq_idx = np.asarray(seq_idx, dtype=np.int64)
    L = seq_idx.shape[1]
    nc = -(-L // chunk_size)
    ends = np.minimum(np.arange(1, nc + 1) * chunk_size, L) - 1
    return seq_idx[:, ends]


def mask_chunk_state(seq_idx, chunk_size):
    """A7 (``chunk_state_fwd.py:246-269``): position k of chunk c contributes to the
    chunk state iff ``last_c >= 0 and seq[k] == last_c``; seq padded with -1.
    Returns bool (b, nc, Q)."""
    L = np.asarray(seq_idx).shape[1]
    nc = -(-L // chunk_size)
    sp = _pad_seq(seq_idx, nc * chunk_size).reshape(-1, nc, chunk_size)
    last = chunk_end_seq(seq_idx, chunk_size)
    return (last[:, :, None] >= 0) & (sp == last[:, :, None])


def mask_bmm(seq_idx, chunk_size):
    """A8 (``bmm_chunk_fwd.py:353-372``): CB[m, n] kept iff seq[m] == seq[n] with the
    -1 padding (two padded positions match).  Returns bool (b, nc, Q, Q)."""
    L = np.asarray(seq_idx).shape[1]
    nc = -(-L // chunk_size)
    sp = _pad_seq(seq_idx, nc * chunk_size).reshape(-1, nc, chunk_size)
    return sp[:, :, :, None] == sp[:, :, None, :]


def mask_scan_state(seq_idx, chunk_size):
    """A9, chunk_scan part (``chunk_scan_fwd.py:294-322``): row m of chunk c reads the
    passed state iff ``seq[m] == prev_c`` where ``prev_0 = 0`` and
    ``prev_c = seq[cQ - 1]``.  Returns bool (b, nc, Q)."""
    L = np.asarray(seq_idx).shape[1]
    nc = -(-L // chunk_size)
    sp = _pad_seq(seq_idx, nc * chunk_size)
    prev_pos = np.arange(nc) * chunk_size - 1
    prev = np.where(prev_pos >= 0, sp[:, np.maximum(prev_pos, 0)], 0)
    return sp.reshape(-1, nc, chunk_size) == prev[:, :, None]


def state_passing_keep(seq_idx, chunk_size):
    """A9, state_passing part (``state_passing_fwd.py:208-225``;
    ``tests/test_state_passing_and_bmm.py:113-131``): chunk c keeps the running
    state iff ``end_c == end_{c-1}`` with ``end_{-1} = 0``.  Returns bool (b, nc)."""
    ends = chunk_end_seq(seq_idx, chunk_size)
    prev = np.concatenate([np.zeros_like(ends[:, :1]), ends[:, :-1]], axis=1)
    return ends == prev


# ---------------------------------------------------------------------------
# A3  chunk_state
# ---------------------------------------------------------------------------

def chunk_state(B, x, dt, dA_cumsum, seq_idx=None):
    """``ssd_naive.py:77-128`` (decay ``exp(dA_last - dA_k)``, ``:115``) with the A7 mask.
    dt, dA_cumsum are (b,H,nc,Q).  Returns states (b, nc, H, P, N)."""
    B, x, dt, dA_cumsum = _f(B), _f(x), _f(dt), _f(dA_cumsum)
    b, L, H, P = x.shape
    G, N = B.shape[2], B.shape[3]
    nc, Q = dt.shape[2], dt.shape[3]
    pad = nc * Q - L
    xp = np.pad(x, ((0, 0), (0, pad), (0, 0), (0, 0))).reshape(b, nc, Q, H, P)
    Bp = np.pad(B, ((0, 0), (0, pad), (0, 0), (0, 0))).reshape(b, nc, Q, G, N)
    Bh = np.repeat(Bp, H // G, axis=3)
    scale = np.exp(dA_cumsum[..., -1:] - dA_cumsum) * dt            # (b,H,nc,Q)
    if seq_idx is not None:
        scale = np.where(mask_chunk_state(seq_idx, Q)[:, None], scale, 0.0)
    return np.einsum("bclhn,bhcl,bclhp->bchpn", Bh, scale, xp, optimize=True)


# ---------------------------------------------------------------------------
# A4  state_passing
# ---------------------------------------------------------------------------

def state_passing(states, dA_chunk_cumsum, initial_states=None, seq_idx=None,
                  chunk_size=None):
    """Sequential form (``tests/test_state_passing_and_bmm.py:92-138``): s_0 = init | 0,
    s_{c+1} = keep_c * exp(dA_chunk[c]) * s_c + states[c].
    states (b,nc,H,D), dA_chunk_cumsum (b,H,nc) -> out (b,nc,H,D), final (b,H,D)."""
    states, dA = _f(states), _f(dA_chunk_cumsum)
    b, nc, H, D = states.shape
    run = np.zeros((b, H, D)) if initial_states is None else _f(initial_states).reshape(b, H, D).copy()
    keep = np.ones((b, nc), bool) if seq_idx is None else state_passing_keep(seq_idx, chunk_size)
    out = np.empty_like(states)
    for c in range(nc):
        out[:, c] = run
        scale = np.exp(dA[:, :, c]) * keep[:, c][:, None]
        run = scale[:, :, None] * run + states[:, c]
    return out, run


def state_passing_pairwise(states, dA_chunk_cumsum, initial_states=None):
    """Vectorised pairwise-decay form of ``ssd_naive.py:135-182`` (no seq_idx); used to
    cross-check :func:`state_passing`."""
    states, dA = _f(states), _f(dA_chunk_cumsum)
    b, nc, H, D = states.shape
    init = np.zeros((b, H, D)) if initial_states is None else _f(initial_states).reshape(b, H, D)
    st = np.concatenate([init[:, None], states], axis=1)
    cs = np.cumsum(np.pad(dA, ((0, 0), (0, 0), (1, 0))), axis=-1)
    n1 = nc + 1
    expo = cs[:, :, :, None] - cs[:, :, None, :]
    expo = np.where(np.tril(np.ones((n1, n1), bool))[None, None], expo, -np.inf)
    out = np.einsum("bhzc,bchd->bzhd", np.exp(expo), st, optimize=True)
    return out[:, :-1], out[:, -1]


# ---------------------------------------------------------------------------
# A5  bmm_chunk
# ---------------------------------------------------------------------------

def bmm_chunk(a, b_, chunk_size, seq_idx=None, causal=False):
    """``ssd_naive.py:189-216`` + the A8 mask and optional tril
    (``bmm_chunk_fwd.py:348-372``).  Returns (b, nc, G, Q, Q)."""
    a, b_ = _f(a), _f(b_)
    bs, L, G, K = a.shape
    nc = -(-L // chunk_size)
    pad = nc * chunk_size - L
    ac = np.pad(a, ((0, 0), (0, pad), (0, 0), (0, 0))).reshape(bs, nc, chunk_size, G, K)
    bc = np.pad(b_, ((0, 0), (0, pad), (0, 0), (0, 0))).reshape(bs, nc, chunk_size, G, K)
    out = np.einsum("bclgn,bcsgn->bcgls", ac, bc, optimize=True)
    if causal:
        out = np.where(np.tril(np.ones((chunk_size, chunk_size), bool)), out, 0.0)
    if seq_idx is not None:
        out = np.where(mask_bmm(seq_idx, chunk_size)[:, :, None], out, 0.0)
    return out


# ---------------------------------------------------------------------------
# A6  chunk_scan
# ---------------------------------------------------------------------------

def chunk_scan(CB, x, dt, dA_cumsum, C, prev_states, D=None, z=None, seq_idx=None):
    """``ssd_naive.py:223-318`` plus the seq_idx rules of
    ``tests/test_chunk_scan_and_varlen.py:133-255``: the CB term is masked by A8 and the
    state term row-masked by A9.  Returns out (b,L,H,P) and out_x (pre-gate, or None)."""
    CB, x, dt, dA, C, prev = _f(CB), _f(x), _f(dt), _f(dA_cumsum), _f(C), _f(prev_states)
    b, L, H, P = x.shape
    G, N = C.shape[2], C.shape[3]
    nc, Q = dt.shape[2], dt.shape[3]
    r = H // G
    pad = nc * Q - L
    xc = np.pad(x, ((0, 0), (0, pad), (0, 0), (0, 0))).reshape(b, nc, Q, H, P)
    Cc = np.pad(C, ((0, 0), (0, pad), (0, 0), (0, 0))).reshape(b, nc, Q, G, N)
    if seq_idx is not None:
        CB = np.where(mask_bmm(seq_idx, Q)[:, :, None], CB, 0.0)
    expo = dA[..., :, None] - dA[..., None, :]                       # (b,H,nc,Q,Q)
    expo = np.where(np.tril(np.ones((Q, Q), bool)), expo, -np.inf)
    decay = np.exp(expo)
    out = np.empty((b, nc, Q, H, P))
    sdec = np.exp(dA)                                                 # (b,H,nc,Q)
    if seq_idx is not None:
        sdec = np.where(mask_scan_state(seq_idx, Q)[:, None], sdec, 0.0)
    for h in range(H):
        g = h // r
        scores = CB[:, :, g] * decay[:, h] * dt[:, h][:, :, None, :]   # (b,nc,Q,Q)
        intra = np.einsum("bcls,bcsp->bclp", scores, xc[:, :, :, h], optimize=True)
        inter = np.einsum("bcln,bcpn->bclp", Cc[:, :, :, g], prev[:, :, h], optimize=True)
        out[:, :, :, h] = intra + inter * sdec[:, h][..., None]
    out = out.reshape(b, nc * Q, H, P)[:, :L]
    if D is not None:
        D = _f(D)
        out = out + x * (D[None, None, :, None] if D.ndim == 1 else D[None, None])
    out_x = None
    if z is not None:
        out_x = out
        out = out * silu(_f(z))
    return out, out_x


# ---------------------------------------------------------------------------
# A10  chunk_state_varlen
# ---------------------------------------------------------------------------

def chunk_state_varlen(B, x, dt, dA_cumsum, cu_seqlens, chunk_states):
    """Per-sequence loop of ``tests/test_chunk_scan_and_varlen.py:504-589``
    (kernel path ``chunk_state_fwd.py:448-597``).
    B (T,G,N), x (T,H,P), dt/dA_cumsum (H,nc,Q), chunk_states (nc,H,P,N) = passed
    states (state at the START of each chunk).  Returns (S, H, P, N)."""
    B, x, dt, dA, cs = _f(B), _f(x), _f(dt), _f(dA_cumsum), _f(chunk_states)
    T, H, P = x.shape
    G, N = B.shape[1], B.shape[2]
    Q = dt.shape[2]
    r = H // G
    cu = [int(v) for v in np.asarray(cu_seqlens)]
    res = np.zeros((len(cu) - 1, H, P, N))
    for s in range(len(cu) - 1):
        start, end = cu[s], cu[s + 1]
        lc = (end - 1) // Q
        c0 = lc * Q
        sic = max(start - c0, 0)
        lv = end - c0 - 1
        dlast = dA[:, lc, lv]
        scale = np.exp(dlast[:, None] - dA[:, lc]) * dt[:, lc]       # (H,Q)
        pos = np.arange(Q)
        valid = (pos >= sic) & (pos <= lv)
        scale = np.where(valid[None], scale, 0.0)
        n_ok = min(Q, T - c0)
        xs = np.zeros((Q, H, P))
        Bs = np.zeros((Q, G, N))
        xs[:n_ok] = x[c0:c0 + n_ok]
        Bs[:n_ok] = B[c0:c0 + n_ok]
        for h in range(H):
            res[s, h] = (xs[:, h] * scale[h][:, None]).T @ Bs[:, h // r]
        if start < c0:
            res[s] += cs[lc] * np.exp(dlast)[:, None, None]
    return res


# ---------------------------------------------------------------------------
# A1 / A12  combined forward
# ---------------------------------------------------------------------------

def ssd_combined(x, dt, A, B, C, chunk_size, D=None, z=None, dt_bias=None,
                 initial_states=None, seq_idx=None, cu_seqlens=None,
                 dt_softplus=False, dt_limit=(0.0, math.inf),
                 return_final_states=False, return_varlen_states=False,
                 pad_mode="kernel", state_round=None, return_intermediates=False):
    """``kernels/ssd_combined.py:46-203`` composed from the stages above (bmm with
    causal=False, masks in chunk_scan).  ``state_round`` optionally rounds the passed
    states before chunk_scan (the reference casts them to C's dtype,
    ``ssd_combined.py:140``); pass a function such as :func:`round_bf16`."""
    dA, dt_out = chunk_cumsum(dt, A, chunk_size, dt_bias, dt_softplus, dt_limit, pad_mode)
    states = chunk_state(B, x, dt_out, dA, seq_idx)
    b, nc, H, P, N = states.shape
    passed, final = state_passing(states.reshape(b, nc, H, P * N), dA[..., -1],
                                  initial_states, seq_idx, chunk_size)
    passed = passed.reshape(b, nc, H, P, N)
    final = final.reshape(b, H, P, N)
    if state_round is not None:
        passed = state_round(passed)
    CB = bmm_chunk(C, B, chunk_size, seq_idx)
    out, _ = chunk_scan(CB, x, dt_out, dA, C, passed, D, z, seq_idx)
    res = [out]
    if return_final_states:
        res.append(final)
    if return_varlen_states:
        assert cu_seqlens is not None and x.shape[0] == 1
        res.append(chunk_state_varlen(_f(B)[0], _f(x)[0], dt_out[0], dA[0],
                                      cu_seqlens, passed[0]))
    if return_intermediates:
        return tuple(res), dict(dA_cumsum=dA, dt_out=dt_out, states=states,
                                passed=passed, CB=CB)
    return res[0] if len(res) == 1 else tuple(res)


# ---------------------------------------------------------------------------
# A11  selective_state_update
# ---------------------------------------------------------------------------

def selective_state_update(state, x, dt, A, B, C, D=None, z=None, dt_bias=None,
                           dt_softplus=False):
    """``ops/selective_state_update.py:22-123``.  Returns (new_state, out)."""
    state, x, dt, A, B, C = map(_f, (state, x, dt, A, B, C))
    b, H, P, N = state.shape
    G = B.shape[1]
    r = H // G
    if dt_bias is not None:
        dt = dt + _f(dt_bias)
    if dt_softplus:
        dt = softplus(dt)
    if dt.ndim == 2:
        dt = dt[:, :, None]
    Bh = np.repeat(B, r, axis=1)
    Ch = np.repeat(C, r, axis=1)
    if A.ndim == 1:
        dA = np.exp(dt[..., None] * A[None, :, None, None])
    else:
        dA = np.exp(dt[..., None] * A[None])
    new = state * dA + dt[..., None] * Bh[:, :, None, :] * x[..., None]
    out = np.sum(new * Ch[:, :, None, :], axis=-1)
    if D is not None:
        D = _f(D)
        out = out + (D[None, :, None] if D.ndim == 1 else D[None]) * x
    if z is not None:
        out = out * silu(_f(z))
    return new, out


# ---------------------------------------------------------------------------
# F1  causal_conv1d (the step before the SSD)
# ---------------------------------------------------------------------------

def conv1d_keep(seq_idx, width):
    """``causal_conv1d.py:143-193`` (_mask_sequence_boundaries): the (b, L) 0/1 factor on x.

    boundary[t] = t == 0 or seq[t] != seq[t-1]; for each lag j in 1..width-1, x[t] is
    zeroed when boundary[t+j] (positions past the end count as no boundary).
    """
    seq = np.asarray(seq_idx)
    b, L = seq.shape
    boundary = np.concatenate([np.ones((b, 1), bool), seq[:, 1:] != seq[:, :-1]], axis=1)
    keep = np.ones((b, L), F64)
    for j in range(1, width):
        shifted = np.concatenate([boundary[:, j:], np.zeros((b, min(j, L)), bool)], axis=1)[:, :L]
        keep = keep * (1.0 - shifted)
    return keep


def causal_conv1d(x, weight, bias=None, activation=None, seq_idx=None):
    """``causal_conv1d.py:18-85``: x (b, d, L), weight (d, k) or (d, 1, k) -> (b, d, L).

    lax.conv_general_dilated is a cross-correlation over the left-padded input, so
    out[t] = sum_j w[j] x[t - (k-1) + j]: w[k-1] multiplies the newest input.
    """
    x, w = _f(x), _f(weight)
    if w.ndim == 3:
        w = w[:, 0, :]
    b, d, L = x.shape
    k = w.shape[1]
    if seq_idx is not None:
        x = x * conv1d_keep(seq_idx, k)[:, None, :]
    xp = np.concatenate([np.zeros((b, d, k - 1)), x], axis=2)
    out = np.zeros((b, d, L))
    for j in range(k):
        out += w[None, :, j:j + 1] * xp[:, :, j:j + L]
    if bias is not None:
        out = out + _f(bias)[None, :, None]
    if activation == "silu":
        out = silu(out)
    return out


def causal_conv1d_update(x_new, conv_state, weight, bias=None, activation=None):
    """``causal_conv1d.py:88-139``: returns (new_conv_state, out)."""
    s, w = _f(conv_state), _f(weight)
    if w.ndim == 3:
        w = w[:, 0, :]
    new = np.concatenate([s[:, :, 1:], _f(x_new)[:, :, None]], axis=-1)
    out = np.sum(new * w[None], axis=-1)
    if bias is not None:
        out = out + _f(bias)[None]
    if activation == "silu":
        out = silu(out)
    return new, out


# ---------------------------------------------------------------------------
# F2  rms_norm_gated (the step after the SSD)
# ---------------------------------------------------------------------------

def rms_norm_gated(x, weight, z=None, eps=1e-5, group_size=None, norm_before_gate=True):
    """``ops/rms_norm.py:15-92``: RMS over groups of ``group_size`` of the last axis.

    norm_before_gate: out = x / sqrt(mean_g(x^2) + eps) * weight * silu(z); otherwise x is
    multiplied by silu(z) first and the gate is not applied again (``:57-66``, ``:76-91``).
    """
    x, w = _f(x), _f(weight)
    hidden = x.shape[-1]
    gs = hidden if group_size is None else int(group_size)
    assert hidden % gs == 0
    if z is not None and not norm_before_gate:
        x = x * silu(_f(z))
    xg = x.reshape(*x.shape[:-1], hidden // gs, gs)
    rms = np.sqrt(np.mean(xg * xg, axis=-1, keepdims=True) + eps)
    out = (xg / rms).reshape(x.shape) * w
    if z is not None and norm_before_gate:
        out = out * silu(_f(z))
    return out


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def round_bf16(a):
    """Round-to-nearest-even to bfloat16, returned as float64."""
    a32 = np.asarray(a, dtype=np.float32)
    u = a32.view(np.uint32).astype(np.uint64)
    rnd = ((u >> 16) & 1) + 0x7FFF
    u = ((u + rnd) >> 16) << 16
    out = u.astype(np.uint32).view(np.float32)
    out = np.where(np.isnan(a32), a32, out)
    return out.astype(F64)


def rel_l2(got, ref):
    got = np.asarray(got, dtype=F64)
    ref = np.asarray(ref, dtype=F64)
    den = np.linalg.norm(ref.ravel())
    return float(np.linalg.norm((got - ref).ravel()) / (den if den > 0 else 1.0))
