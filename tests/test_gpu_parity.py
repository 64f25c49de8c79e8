"""GPU parity: every entry point of libssd_b200.so against the float64 oracle.

Tolerances (written here): rel-L2 <= 1e-4 for float32
inputs and <= 1e-2 for bf16 inputs with fp32 accumulation; mask / reset decisions and
chunk boundaries are compared bit-exactly (zero patterns of masked outputs).
"""
import math
import zlib

import numpy as np
import pytest
import torch

from oracle import ssd_ref as R
from mamba2_b200 import synthetic as S
from gpu_util import TOL, dev_inputs, rel_l2, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mamba2_b200._lib as L
    L.load()


def _combined_oracle(inp, Q, cfg, **kw):
    return R.ssd_combined(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], Q, D=inp["D"],
                          z=inp["z"], dt_bias=inp["dt_bias"], initial_states=inp["initial_states"],
                          seq_idx=inp["seq_idx"], cu_seqlens=inp["cu_seqlens"], dt_softplus=True,
                          return_final_states=True,
                          return_varlen_states=inp["cu_seqlens"] is not None, **kw)


# (name, cfg) — small versions of the BASELINE configs plus edge cases the reference tests
CASES = [
    ("c0-small", S.scaled(S.CONFIGS["c0"], seqlen=512)),
    ("c0-full", S.CONFIGS["c0"]),
    ("c1-small", S.scaled(S.CONFIGS["c1"], batch=2, seqlen=512, nheads=8)),
    ("c2-small", S.scaled(S.CONFIGS["c2"], seqlen=512, nheads=16)),
    ("c3-small", S.scaled(S.CONFIGS["c3"], seqlen=1024, nheads=16, varlen_seqs=5,
                          varlen_range=(32, 400))),
    ("ragged-L", S.SsdConfig("ragged", 2, 200, 4, 64, 2, 64, 64, "f32", has_z=True,
                             has_init=True, return_final=True)),
    ("ragged-bf16", S.SsdConfig("ragged16", 2, 333, 8, 64, 8, 128, 128, "bf16", has_z=True,
                                has_init=True, return_final=True)),
    ("tiny-P-N", S.SsdConfig("tiny", 1, 96, 3, 8, 1, 16, 32, "f32", has_init=True,
                             return_final=True)),
    ("odd-P", S.SsdConfig("oddP", 1, 256, 4, 80, 2, 96, 64, "f32", has_z=True, return_final=True)),
    ("one-token", S.SsdConfig("one", 1, 1, 2, 64, 1, 128, 64, "bf16", has_init=True,
                              return_final=True)),
    ("many-seqs", S.SsdConfig("manyseq", 1, 512, 4, 64, 2, 64, 64, "bf16", return_final=True,
                              varlen_seqs=24, varlen_range=(1, 40))),
]


@pytest.mark.parametrize("name,cfg", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("path", ["default", "simt"])
def test_combined_vs_oracle(name, cfg, path):
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    inp = S.make_ssd_inputs(cfg, 1000 + zlib.crc32(name.encode()) % 1000)
    d = dev_inputs(inp, cfg.dtype)
    varlen = inp["cu_seqlens"] is not None
    res = mamba_chunk_scan_combined_fwd(
        d["x"], d["dt"], d["A"], d["B"], d["C"], cfg.chunk_size, D=d["D"], z=d["z"],
        dt_bias=d["dt_bias"], initial_states=d["initial_states"], seq_idx=d["seq_idx"],
        cu_seqlens=d["cu_seqlens"], dt_softplus=True, return_final_states=True,
        return_varlen_states=varlen, force_simt=(path == "simt"))
    torch.cuda.synchronize()
    ref = _combined_oracle(inp, cfg.chunk_size, cfg)
    tol = TOL[cfg.dtype]
    for got, want, what in zip(res, ref, ("out", "final", "varlen")):
        assert torch.isfinite(got).all(), what
        e = rel_l2(got, want)
        assert e <= tol, f"{name}/{path} {what}: rel-L2 {e:.3e} > {tol}"


def test_combined_return_conventions():
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    cfg = S.SsdConfig("t", 1, 128, 2, 64, 1, 64, 64, "f32")
    inp = S.make_ssd_inputs(cfg, 5)
    d = dev_inputs(inp, "f32")
    a = (d["x"], d["dt"], d["A"], d["B"], d["C"], 64)
    out = mamba_chunk_scan_combined_fwd(*a)
    assert isinstance(out, torch.Tensor) and out.dtype == torch.float32
    o, f = mamba_chunk_scan_combined_fwd(*a, return_final_states=True)
    assert f.shape == (1, 2, 64, 64)
    cu = torch.tensor([0, 50, 128], dtype=torch.int32, device="cuda")
    seq = torch.repeat_interleave(torch.arange(2, device="cuda"), torch.tensor([50, 78], device="cuda"))[None]
    o, v = mamba_chunk_scan_combined_fwd(*a, seq_idx=seq.int(), cu_seqlens=cu, return_varlen_states=True)
    assert v.shape == (2, 2, 64, 64)
    o, f, v = mamba_chunk_scan_combined_fwd(*a, seq_idx=seq.int(), cu_seqlens=cu,
                                            return_final_states=True, return_varlen_states=True)
    # two different kernels reach the same state (fp32 contract: 1e-4)
    torch.testing.assert_close(f[0], v[1], rtol=1e-4, atol=1e-4)


# ---------------------------------------------------------------------------
# stages
# ---------------------------------------------------------------------------

def _stage_inputs(cfg, seed=11):
    inp = S.make_ssd_inputs(cfg, seed)
    dA, dto = R.chunk_cumsum(inp["dt"], inp["A"], cfg.chunk_size, inp["dt_bias"], True)
    return inp, dA, dto


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("L,Q", [(128, 64), (256, 256), (1000, 128), (77, 32)])
def test_chunk_cumsum(dtype, L, Q):
    from mamba2_b200 import chunk_cumsum_fwd
    cfg = S.SsdConfig("t", 2, L, 40, 8, 1, 8, Q, dtype)
    inp = S.make_ssd_inputs(cfg, 3)
    dA_ref, dt_ref = R.chunk_cumsum(inp["dt"], inp["A"], Q, inp["dt_bias"], True, (0.0, 0.5))
    dA, dto = chunk_cumsum_fwd(to_dev(inp["dt"], dtype), to_dev(inp["A"]), Q,
                               dt_bias=to_dev(inp["dt_bias"]), dt_softplus=True, dt_limit=(0.0, 0.5))
    np.testing.assert_allclose(dto.cpu().numpy(), dt_ref, rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(dA.cpu().numpy(), dA_ref, rtol=2e-5, atol=2e-5)
    # padded tail positions are exactly zero in dt_out
    if L % Q:
        assert (dto.reshape(2, 40, -1)[:, :, L:] == 0).all()


# fp32 stage kernels: "tc" = split-bf16 tcgen05 (default), "cuda" = fp32 FFMA.  bf16 inputs
# always take the CUDA-core stages, so they run once.  Tolerance: the FFMA stages are exact
# fp32 (1e-5); the split-bf16 products carry about 1e-5 relative error each (4e-5 here,
# inside the fp32 contract of 1e-4).
STAGE_PATHS = [("f32", "tc"), ("f32", "cuda"), ("bf16", "cuda")]
STAGE_TOL = {"tc": 4e-5, "cuda": 1e-5}


def _stage_path(path):
    import mamba2_b200._lib as L
    return L.fp32_stage_path(L.FP32_STAGES_TENSOR_CORES if path == "tc" else L.FP32_STAGES_CUDA_CORES)


SEQ_CFGS = [None, [[256]], [[128, 128]], [[200, 312], [100, 412]],
            [[64, 192, 256], [128, 128, 256]], [[64, 64, 64, 64]]]


def _seq_idx(batch, L, lens):
    out = np.zeros((batch, L), np.int32)
    for i in range(batch):
        ids = np.repeat(np.arange(len(lens[i])), lens[i])[:L]
        if len(ids) < L:
            ids = np.concatenate([ids, np.full(L - len(ids), ids[-1])])
        out[i] = ids
    return out


@pytest.mark.parametrize("dtype,path", STAGE_PATHS)
@pytest.mark.parametrize("lens", SEQ_CFGS)
def test_chunk_state(dtype, path, lens):
    from mamba2_b200 import chunk_state_fwd
    batch = 1 if lens is None else len(lens)
    L = 512 if lens is None else sum(lens[0])
    cfg = S.SsdConfig("t", batch, L, 8, 64, 2, 128, 64, dtype)
    inp, dA, dto = _stage_inputs(cfg)
    seq = None if lens is None else _seq_idx(batch, L, lens)
    ref = R.chunk_state(inp["B"], inp["x"], dto, dA, seq)
    with _stage_path(path):
        got = chunk_state_fwd(to_dev(inp["x"], dtype), to_dev(inp["B"], dtype), to_dev(dto), to_dev(dA),
                              seq_idx=to_dev(seq, int32=True))
    assert rel_l2(got, ref) <= STAGE_TOL[path]
    if seq is not None:
        # positions outside the chunk-end sequence contribute nothing (bit-exact mask):
        zero_chunks = ~R.mask_chunk_state(seq, 64).any(-1)
        assert (got.cpu().numpy()[zero_chunks] == 0).all()


@pytest.mark.parametrize("b,nc,H,dim,init,lens", [
    (1, 4, 1, 128, False, None), (2, 8, 4, 128, True, None), (2, 8, 16, 4096, True, None),
    (1, 8, 4, 16384, True, None), (1, 4, 2, 200, True, None), (2, 8, 4, 300, True, None),
    (1, 4, 4, 128, True, [[256]]), (1, 4, 4, 128, False, [[128, 128]]),
    (2, 8, 8, 128, True, [[200, 312], [100, 412]]), (2, 8, 4, 4096, True, [[64, 192, 256], [128, 128, 256]]),
    (1, 4, 4, 128, True, [[64, 64, 64, 64]]),
])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_state_passing(b, nc, H, dim, init, lens, out_dtype):
    """Configs of tests/test_state_passing_and_bmm.py:620-667."""
    from mamba2_b200 import state_passing_fwd
    rng = np.random.default_rng(nc * 100 + dim)
    st = rng.standard_normal((b, nc, H, dim)).astype(np.float32)
    dA = (-rng.uniform(0, 2, (b, H, nc))).astype(np.float32)
    ini = rng.standard_normal((b, H, dim)).astype(np.float32) if init else None
    seq = None if lens is None else _seq_idx(b, nc * 64, lens)
    o_ref, f_ref = R.state_passing(st, dA, ini, seq, 64)
    o, f = state_passing_fwd(to_dev(st), to_dev(dA), initial_states=to_dev(ini),
                             seq_idx=to_dev(seq, int32=True), chunk_size=64, out_dtype=out_dtype)
    tol = 1e-6 if out_dtype == torch.float32 else 4e-3
    assert rel_l2(o, o_ref) <= tol
    assert rel_l2(f, f_ref) <= 1e-6


@pytest.mark.parametrize("dtype,path", STAGE_PATHS)
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("lens,L,Q", [(None, 512, 64), (None, 300, 128), ([[200, 312], [100, 412]], 512, 64),
                                      ([[256, 256], [128, 384]], 512, 128), ([[3, 61, 100, 92]], 256, 256)])
def test_bmm_chunk(dtype, path, causal, lens, L, Q):
    from mamba2_b200 import bmm_chunk_fwd
    batch = 2 if lens is None else len(lens)
    rng = np.random.default_rng(L + Q)
    a = S.round_to(rng.standard_normal((batch, L, 2, 64)).astype(np.float32), dtype)
    bm = S.round_to(rng.standard_normal((batch, L, 2, 64)).astype(np.float32), dtype)
    seq = None if lens is None else _seq_idx(batch, L, lens)
    ref = R.bmm_chunk(a, bm, Q, seq, causal)
    with _stage_path(path):
        got = bmm_chunk_fwd(to_dev(a, dtype), to_dev(bm, dtype), Q, seq_idx=to_dev(seq, int32=True),
                            causal=causal).cpu().numpy()
    assert rel_l2(got, ref) <= STAGE_TOL[path]
    # bit-exact mask decisions: zero exactly where the oracle mask is false
    np.testing.assert_array_equal(got == 0, ref == 0)


@pytest.mark.parametrize("dtype,path", STAGE_PATHS)
@pytest.mark.parametrize("lens,G,Q,Dn,z", [(None, 1, 64, 1, True), (None, 8, 64, 0, False),
                                          ([[200, 312], [100, 412]], 1, 64, 1, False),
                                          ([[256, 256], [128, 384]], 4, 128, 2, True)])
def test_chunk_scan(dtype, path, lens, G, Q, Dn, z):
    """Configs of tests/test_chunk_scan_and_varlen.py:798-824."""
    from mamba2_b200 import chunk_scan_fwd
    L, H = 512, 8
    batch = 2
    cfg = S.SsdConfig("t", batch, L, H, 64, G, 64, Q, dtype, has_z=z)
    inp, dA, dto = _stage_inputs(cfg)
    seq = None if lens is None else _seq_idx(batch, L, lens)
    CB = R.bmm_chunk(inp["C"], inp["B"], Q, seq)
    rng = np.random.default_rng(9)
    prev = (0.3 * rng.standard_normal((batch, L // Q, H, 64, 64))).astype(np.float32)
    D = np.linspace(0.5, 1.5, H * 64).reshape(H, 64).astype(np.float32) if Dn == 2 else (
        inp["D"] if Dn == 1 else None)
    o_ref, ox_ref = R.chunk_scan(CB, inp["x"], dto, dA, inp["C"], prev, D, inp["z"], seq)
    with _stage_path(path):
        o, ox = chunk_scan_fwd(to_dev(CB), to_dev(inp["x"], dtype), to_dev(dto), to_dev(dA),
                               to_dev(inp["C"], dtype), to_dev(prev), D=to_dev(D),
                               z=to_dev(inp["z"], dtype), seq_idx=to_dev(seq, int32=True))
    assert rel_l2(o, o_ref) <= STAGE_TOL[path]
    if z:
        assert rel_l2(ox, ox_ref) <= STAGE_TOL[path]


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("S_,H,G,Q", [(10, 8, 1, 64), (5, 8, 8, 64), (7, 4, 2, 128)])
def test_chunk_state_varlen(dtype, S_, H, G, Q):
    """Pipeline of tests/test_chunk_scan_and_varlen.py:596-724 (chunk_state -> state_passing
    -> varlen)."""
    from mamba2_b200 import chunk_state_varlen_mosaic
    rng = np.random.default_rng(S_ * 10 + H)
    lens = rng.integers(1, 201, S_)
    T = int(lens.sum())
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    cfg = S.SsdConfig("t", 1, T, H, 64, G, 64, Q, dtype)
    inp, dA, dto = _stage_inputs(cfg)
    seq = np.repeat(np.arange(S_), lens)[None].astype(np.int32)
    st = R.chunk_state(inp["B"], inp["x"], dto, dA, seq)
    nc = st.shape[1]
    passed, _ = R.state_passing(st.reshape(1, nc, H, -1), dA[..., -1], None, seq, Q)
    passed = passed.reshape(nc, H, 64, 64)
    ref = R.chunk_state_varlen(inp["B"][0], inp["x"][0], dto[0], dA[0], cu, passed)
    got = chunk_state_varlen_mosaic(to_dev(inp["B"][0], dtype), to_dev(inp["x"][0], dtype),
                                    to_dev(dto[0]), to_dev(dA[0]), to_dev(cu, int32=True),
                                    to_dev(passed.astype(np.float32)))
    assert rel_l2(got, ref) <= 1e-5


# ---------------------------------------------------------------------------
# decode step
# ---------------------------------------------------------------------------

SSU_CASES = [
    # b, H, P, G, N, dtype, dt_ndim, A_ndim, D_ndim, bias_ndim, z, softplus
    (2, 4, 8, 2, 16, "f32", 2, 1, 0, 0, False, False),     # test_mamba2_ops.py:25-65
    (2, 4, 8, 1, 16, "f32", 2, 1, 1, 1, True, True),       # test_mamba2_ops.py:68-112
    (4, 16, 64, 8, 128, "bf16", 2, 1, 1, 1, True, True),   # c4-shaped
    (3, 6, 32, 3, 64, "f32", 3, 3, 2, 2, True, True),      # per-element dt/A/D/bias
    (2, 4, 16, 2, 18, "bf16", 2, 1, 1, 1, False, True),    # N % 4 != 0 (scalar path)
    (1, 8, 70, 4, 256, "bf16", 3, 1, 0, 0, True, False),   # P not a multiple of 8
    (3, 8, 64, 2, 256, "bf16", 2, 1, 1, 1, True, True),    # N=256 fast path
    (2, 4, 32, 4, 128, "f32", 2, 1, 0, 0, False, True),    # fast path, no D / z / bias
]


@pytest.mark.parametrize("case", SSU_CASES)
@pytest.mark.parametrize("inplace", [False, True])
def test_selective_state_update(case, inplace):
    from mamba2_b200 import selective_state_update
    b, H, P, G, N, dtype, dtn, An, Dn, bn, zz, sp = case
    rng = np.random.default_rng(b * 1000 + H * 10 + P)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)
    state = f(b, H, P, N)
    x = S.round_to(f(b, H, P), dtype)
    dt = S.round_to(f(b, H) if dtn == 2 else f(b, H, P), dtype)
    if not sp:
        dt = S.round_to(np.abs(dt) * 0.1, dtype)
    A = (-np.abs(f(H)) if An == 1 else -np.abs(f(H, P, N))).astype(np.float32)
    Bm, Cm = S.round_to(f(b, G, N), dtype), S.round_to(f(b, G, N), dtype)
    D = None if Dn == 0 else (f(H) if Dn == 1 else f(H, P))
    z = S.round_to(f(b, H, P), dtype) if zz else None
    bias = None if bn == 0 else (f(H) if bn == 1 else f(H, P))
    ns_ref, o_ref = R.selective_state_update(state, x, dt, A, Bm, Cm, D, z, bias, sp)
    st_dev = to_dev(state)
    ns, o = selective_state_update(st_dev, to_dev(x, dtype), to_dev(dt, dtype), to_dev(A),
                                   to_dev(Bm, dtype), to_dev(Cm, dtype), D=to_dev(D), z=to_dev(z, dtype),
                                   dt_bias=to_dev(bias), dt_softplus=sp, inplace=inplace)
    assert rel_l2(ns, ns_ref) <= 1e-6
    assert rel_l2(o, o_ref) <= 1e-5
    if inplace:
        assert ns.data_ptr() == st_dev.data_ptr()
    else:
        np.testing.assert_array_equal(st_dev.cpu().numpy(), state)


def test_ssu_decode_loop_matches_prefill():
    """SSD final state == L sequential decode steps (prefill == decode,
    tests/test_mamba2_vs_torch.py:312-408 at the SSD level)."""
    from mamba2_b200 import mamba_chunk_scan_combined_fwd, selective_state_update
    cfg = S.SsdConfig("t", 2, 100, 8, 64, 2, 64, 32, "f32", has_init=True, return_final=True)
    inp = S.make_ssd_inputs(cfg, 21)
    d = dev_inputs(inp, "f32")
    out, final = mamba_chunk_scan_combined_fwd(
        d["x"], d["dt"], d["A"], d["B"], d["C"], 32, D=d["D"], dt_bias=d["dt_bias"],
        initial_states=d["initial_states"], dt_softplus=True, return_final_states=True)
    state = d["initial_states"].clone()
    outs = []
    for t in range(cfg.seqlen):
        state, o = selective_state_update(state, d["x"][:, t], d["dt"][:, t], d["A"], d["B"][:, t],
                                          d["C"][:, t], D=d["D"], dt_bias=d["dt_bias"],
                                          dt_softplus=True, inplace=True)
        outs.append(o)
    assert rel_l2(state, final.double().cpu().numpy()) <= 1e-5
    assert rel_l2(torch.stack(outs, 1), out.double().cpu().numpy()) <= 1e-5


def test_tensor_core_path_selected():
    """bf16, P=64, N=128 runs the fused tcgen05 kernel (one launch); fp32 does not."""
    from mamba2_b200.runner import SsdForward
    for dtype, want in (("bf16", True), ("f32", False)):
        cfg = S.SsdConfig("t", 1, 256, 4, 64, 2, 128, 128, dtype)
        d = dev_inputs(S.make_ssd_inputs(cfg, 1), dtype)
        r = SsdForward(d["x"], d["dt"], d["A"], d["B"], d["C"], 128, dt_bias=d["dt_bias"], dt_softplus=True)
        assert r.uses_tc == want
        assert r.launches_per_step == (2 if want else 5)   # dt pre-pass + fused kernel
        r()
        torch.cuda.synchronize()
        if want:
            assert int(r.workspace[:4].view(torch.int32).item()) == 0  # device status word


@pytest.mark.parametrize("Dshape", ["head", "head-dim"])
def test_tensor_core_skip_term(Dshape):
    """D per head rides on the diagonal of the bf16 scores in the fused kernel; D per
    (head, head-dim column) cannot, and runs the stage pipeline.  Both within bf16 tolerance,
    with |D| large enough that the skip term dominates the output."""
    from mamba2_b200.runner import SsdForward
    cfg = S.SsdConfig("t", 2, 384, 8, 64, 2, 128, 128, "bf16", has_z=True, has_init=True, return_final=True)
    inp = S.make_ssd_inputs(cfg, 77)
    rng = np.random.default_rng(3)
    inp["D"] = (4.0 * rng.standard_normal((8,) if Dshape == "head" else (8, 64))).astype(np.float32)
    d = dev_inputs(inp, "bf16")
    r = SsdForward(d["x"], d["dt"], d["A"], d["B"], d["C"], 128, D=d["D"], z=d["z"], dt_bias=d["dt_bias"],
                   initial_states=d["initial_states"], dt_softplus=True, return_final_states=True)
    assert r.uses_tc == (Dshape == "head")
    out = r()
    torch.cuda.synchronize()
    ref_out, ref_final = _combined_oracle(inp, 128, cfg)[:2]
    assert rel_l2(out, ref_out) <= TOL["bf16"]
    assert rel_l2(r.final, ref_final) <= TOL["bf16"]


@pytest.mark.parametrize("N,lens", [(256, None), (256, [100, 300, 7, 233]), (128, [128, 1, 300, 211])],
                         ids=["n256", "n256-seq", "n128-seq"])
@pytest.mark.parametrize("z", [False, True])
def test_tensor_core_path_state_dims_and_seq_idx(N, lens, z):
    """The fused tcgen05 kernel at N=128 and N=256, with packed seq_idx (no varlen states
    requested, so the tensor-core path runs)."""
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    from mamba2_b200.runner import SsdForward
    L = 640 if lens is None else sum(lens)
    cfg = S.SsdConfig("t", 1 if lens else 2, L, 8, 64, 2, N, 128, "bf16", has_z=z, has_init=True,
                      return_final=True)
    inp = S.make_ssd_inputs(cfg, 31 + N)
    seq = None if lens is None else np.repeat(np.arange(len(lens)), lens)[None].astype(np.int32)
    d = dev_inputs(inp, "bf16")
    sd = to_dev(seq, int32=True)
    r = SsdForward(d["x"], d["dt"], d["A"], d["B"], d["C"], 128, D=d["D"], z=d["z"], dt_bias=d["dt_bias"],
                   initial_states=d["initial_states"], seq_idx=sd, dt_softplus=True, return_final_states=True)
    assert r.uses_tc
    out = r()
    torch.cuda.synchronize()
    assert int(r.workspace[:4].view(torch.int32).item()) == 0
    ref_out, ref_final = R.ssd_combined(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], 128, D=inp["D"],
                                        z=inp["z"], dt_bias=inp["dt_bias"], initial_states=inp["initial_states"],
                                        seq_idx=seq, dt_softplus=True, return_final_states=True)
    assert rel_l2(out, ref_out) <= TOL["bf16"]
    assert rel_l2(r.final, ref_final) <= TOL["bf16"]


@pytest.mark.parametrize("N,lens", [(128, [128, 1, 0, 300, 255, 44]), (256, [700, 3, 129, 127, 1]),
                                    (128, [256, 128, 384])],
                         ids=["n128-ragged", "n256-long", "n128-aligned"])
@pytest.mark.parametrize("z", [False, True])
def test_tensor_core_path_varlen_states(N, lens, z):
    """Varlen final states on the fused kernel: every packed sequence is tiled from its own
    start, so its state is read off the running state at its last chunk.  Covers an empty
    sequence, a one-token sequence, sequence ends on and off 128-token boundaries and a
    ragged last chunk; the outputs of rows stored twice (a short chunk's tail) must match."""
    from mamba2_b200.runner import SsdForward
    L = sum(lens)
    cfg = S.SsdConfig("t", 1, L, 8, 64, 2, N, 128, "bf16", has_z=z, return_final=True)
    inp = S.make_ssd_inputs(cfg, 7 + N + len(lens))
    seq = np.repeat(np.arange(len(lens)), lens)[None].astype(np.int32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    d = dev_inputs(inp, "bf16")
    r = SsdForward(d["x"], d["dt"], d["A"], d["B"], d["C"], 128, D=d["D"], z=d["z"], dt_bias=d["dt_bias"],
                   seq_idx=to_dev(seq, int32=True), cu_seqlens=to_dev(cu, int32=True), dt_softplus=True,
                   return_final_states=True)
    assert r.uses_tc and r.launches_per_step == 3   # schedule, dt pre-pass, fused kernel
    r.varlen.fill_(float("nan"))
    out = r()
    torch.cuda.synchronize()
    assert int(r.workspace[:4].view(torch.int32).item()) == 0
    ref_out, ref_final, ref_var = R.ssd_combined(
        inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], 128, D=inp["D"], z=inp["z"], dt_bias=inp["dt_bias"],
        seq_idx=seq, cu_seqlens=cu, dt_softplus=True, return_final_states=True, return_varlen_states=True)
    assert rel_l2(out, ref_out) <= TOL["bf16"]
    assert rel_l2(r.final, ref_final) <= TOL["bf16"]
    assert torch.isfinite(r.varlen).all()
    for k in range(len(lens)):
        if lens[k] == 0:
            assert (r.varlen[k] == 0).all()
        else:
            assert rel_l2(r.varlen[k], ref_var[k]) <= TOL["bf16"], k
    # deterministic: a second call writes the same bytes
    out1 = out.clone()
    r()
    torch.cuda.synchronize()
    assert torch.equal(out, out1)


@pytest.mark.parametrize("seq", [False, True])
def test_tensor_core_decay_paths(seq):
    """Score decays on the fused kernel take three forms per 32-token block: factored
    (dA non-increasing, block range <= 60), element by element because the range is larger
    (large |A| dt), and element by element because dA increases (A > 0).  One case mixes
    all three across heads and compares each with the oracle."""
    from mamba2_b200.runner import SsdForward
    lens = [200, 57, 383]
    L = sum(lens)
    cfg = S.SsdConfig("t", 1, L, 8, 64, 2, 128, 128, "bf16", has_init=True, return_final=True)
    inp = S.make_ssd_inputs(cfg, 404)
    A = np.array([-1.0, -3.0, -40.0, -90.0, 0.05, -0.5, -200.0, -8.0], np.float32)
    inp["A"] = A
    s_idx = np.repeat(np.arange(len(lens)), lens)[None].astype(np.int32) if seq else None
    d = dev_inputs(inp, "bf16")
    r = SsdForward(d["x"], d["dt"], d["A"], d["B"], d["C"], 128, D=d["D"], dt_bias=d["dt_bias"],
                   initial_states=d["initial_states"], seq_idx=to_dev(s_idx, int32=True), dt_softplus=True,
                   return_final_states=True)
    assert r.uses_tc
    out = r()
    torch.cuda.synchronize()
    assert int(r.workspace[:4].view(torch.int32).item()) == 0
    ref_out, ref_final = R.ssd_combined(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], 128, D=inp["D"],
                                        dt_bias=inp["dt_bias"], initial_states=inp["initial_states"],
                                        seq_idx=s_idx, dt_softplus=True, return_final_states=True)
    assert torch.isfinite(out).all()
    for h in range(cfg.nheads):
        assert rel_l2(out[:, :, h], ref_out[:, :, h]) <= TOL["bf16"], h
        assert rel_l2(r.final[:, h], ref_final[:, h]) <= TOL["bf16"], h


@pytest.mark.parametrize("z", [False, True])
def test_fp32_inputs_with_bf16_mma(z):
    """SSD_FLAG_BF16_MMA: fp32 inputs rounded to bf16 operands on the tensor-core path (the
    reference's Pallas behaviour for fp32 inputs), held to the bf16 tolerance; without the
    flag the same inputs take the exact fp32 path."""
    from mamba2_b200 import _lib
    from mamba2_b200.runner import SsdForward
    cfg = S.SsdConfig("f32mma", 1, 640, 8, 64, 1, 128, 256, "f32", has_z=z, has_init=True, return_final=True)
    inp = S.make_ssd_inputs(cfg, 51)
    d = dev_inputs(inp, "f32")
    kw = dict(D=d["D"], z=d["z"], dt_bias=d["dt_bias"], initial_states=d["initial_states"], dt_softplus=True,
              return_final_states=True)
    exact = SsdForward(d["x"], d["dt"], d["A"], d["B"], d["C"], 256, **kw)
    fast = SsdForward(d["x"], d["dt"], d["A"], d["B"], d["C"], 256, flags=_lib.SSD_FLAG_BF16_MMA, **kw)
    assert not exact.uses_tc and fast.uses_tc
    assert fast.launches_per_step == 3   # conversion, dt pre-pass, fused kernel
    out = fast()
    torch.cuda.synchronize()
    ref_out, ref_final = R.ssd_combined(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], 256, D=inp["D"],
                                        z=inp["z"], dt_bias=inp["dt_bias"], initial_states=inp["initial_states"],
                                        dt_softplus=True, return_final_states=True)
    assert rel_l2(out, ref_out) <= TOL["bf16"]
    assert rel_l2(fast.final, ref_final) <= TOL["bf16"]


@pytest.mark.parametrize("key", ["c2", "c3"])
def test_full_size_scaling_and_determinism(key):
    """At the full BASELINE sizes (too large for the oracle): without z the forward is linear
    in (x, initial state), and scaling both by 2 is exact at every rounding point (bf16
    operands, fp32 accumulation), so out(2x, 2 h0) must equal 2 out(x, h0) bit for bit, as
    must the final and varlen states.  A second run must also be bitwise identical."""
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    cfg = S.CONFIGS[key]
    inp = S.make_ssd_inputs(cfg, 4242)
    d = dev_inputs(inp, cfg.dtype)
    varlen = d["cu_seqlens"] is not None
    init = d["initial_states"] if d["initial_states"] is not None else None

    def run(scale):
        return mamba_chunk_scan_combined_fwd(
            d["x"] * scale, d["dt"], d["A"], d["B"], d["C"], cfg.chunk_size, D=d["D"], dt_bias=d["dt_bias"],
            initial_states=None if init is None else init * scale, seq_idx=d["seq_idx"],
            cu_seqlens=d["cu_seqlens"], dt_softplus=True, return_final_states=True,
            return_varlen_states=varlen)

    r1, r1b, r2 = run(1.0), run(1.0), run(2.0)
    torch.cuda.synchronize()
    for a_, b_, c_ in zip(r1, r1b, r2):
        assert torch.isfinite(a_).all()
        assert torch.equal(a_, b_)
        assert torch.equal(c_, 2 * a_)
