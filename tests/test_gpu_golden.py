"""The CUDA path against golden outputs of the REFERENCE's own code (tests/golden/*.npz,
made by tests/golden/make_fixtures.py from the reference's unmodified pure-JAX ops).

Bounds: rel-L2 <= 1e-4 for float32 inputs, <= 1e-2 for bf16
inputs with fp32 accumulation.  The comparison is against the reference's float64 run
(``ref64``) and, for float32 cases, also against its float32 run (``ref32``).
"""
import numpy as np
import pytest
import torch

import fixtures as F
from gpu_util import TOL, rel_l2, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mamba2_b200._lib as L
    L.load()


SSD = F.load("ssd")


def _ssd_dev(c, dtype):
    d = {k: to_dev(c.get(k), dtype) for k in ("x", "dt", "B", "C", "z")}
    d.update({k: to_dev(c.get(k), "f32") for k in ("A", "D", "dt_bias", "initial_states")})
    d["seq_idx"] = to_dev(c.get("seq_idx"), int32=True)
    d["cu_seqlens"] = to_dev(c.get("cu_seqlens"), int32=True)
    return d


@pytest.mark.parametrize("name", ["c0s", "c1s", "c2s", "c0r"])
@pytest.mark.parametrize("path", ["default", "simt"])
def test_combined_vs_reference_fixture(name, path):
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    c = F.case(SSD, name)
    Q, is_bf16 = int(c["meta"][0]), bool(c["meta"][1])
    dtype = "bf16" if is_bf16 else "f32"
    d = _ssd_dev(c, dtype)
    out, final = mamba_chunk_scan_combined_fwd(
        d["x"], d["dt"], d["A"], d["B"], d["C"], Q, D=d["D"], z=d["z"], dt_bias=d["dt_bias"],
        initial_states=d["initial_states"], dt_softplus=True, return_final_states=True,
        force_simt=(path == "simt"))
    torch.cuda.synchronize()
    tol = TOL[dtype]
    # the kernel path's final state (no padded positions) for the ragged case
    fkey = "final_kernel" if name == "c0r" else "final"
    for tag in ("ref64", "ref32"):
        if f"{tag}/out" not in c:
            continue
        e_out, e_fin = rel_l2(out, c[f"{tag}/out"]), rel_l2(final, c[f"{tag}/{fkey}"])
        assert e_out <= tol, f"{name}/{path}/{tag} out rel-L2 {e_out:.3e}"
        assert e_fin <= tol, f"{name}/{path}/{tag} final rel-L2 {e_fin:.3e}"


@pytest.mark.parametrize("path", ["default", "simt"])
def test_packed_varlen_vs_reference_fixture(path):
    """Packed row (sequences of 150, 57 and 177 tokens, N=256): outputs and per-sequence
    final states equal the reference run on each sequence alone."""
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    c = F.case(SSD, "c3p")
    d = _ssd_dev(c, "bf16")
    out, vs = mamba_chunk_scan_combined_fwd(
        d["x"], d["dt"], d["A"], d["B"], d["C"], int(c["meta"][0]), D=d["D"], dt_bias=d["dt_bias"],
        seq_idx=d["seq_idx"], cu_seqlens=d["cu_seqlens"], dt_softplus=True, return_varlen_states=True,
        force_simt=(path == "simt"))
    torch.cuda.synchronize()
    assert rel_l2(out, c["ref64/out"]) <= TOL["bf16"]
    assert rel_l2(vs, c["ref64/varlen_states"]) <= TOL["bf16"]
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("name", ["c4s", "c4v"])
def test_selective_state_update_vs_reference_fixture(name):
    from mamba2_b200 import selective_state_update
    d = F.load("ssu")
    c = F.case(d, name)
    st = torch.from_numpy(d["c4s/state"]).cuda()
    args = [to_dev(c[k], "bf16") for k in ("x", "dt")] + [to_dev(c["A"])] + \
        [to_dev(c[k], "bf16") for k in ("B", "C")]
    ns, out = selective_state_update(st, *args, D=to_dev(c["D"]), z=to_dev(c["z"], "bf16"),
                                     dt_bias=to_dev(c["dt_bias"]), dt_softplus=True)
    torch.cuda.synchronize()
    for tag in ("ref64", "ref32"):
        assert rel_l2(ns, c[f"{tag}/state"]) <= 1e-5
        assert rel_l2(out, c[f"{tag}/out"]) <= 1e-4


@pytest.mark.parametrize("case,gs,nbg,usez", [("g256", 256, True, True), ("g256_gate_first", 256, False, True),
                                              ("full", None, True, True), ("g1024_noz", 1024, True, False)])
def test_rms_norm_gated_vs_reference_fixture(case, gs, nbg, usez):
    from mamba2_b200 import rms_norm_gated
    d = F.load("norm")
    o = rms_norm_gated(to_dev(d["y"]), to_dev(d["w"]), z=to_dev(d["z"], "bf16") if usez else None,
                       eps=1e-5, group_size=gs, norm_before_gate=nbg)
    torch.cuda.synchronize()
    # the reference's own f32 bound for this op (tests/test_mamba2_ops.py:258-259): max-abs 1e-5
    # against its float64 run, on outputs of order one
    err = float(np.max(np.abs(o.double().cpu().numpy() - d[f"{case}/ref64/out"].astype(np.float64))))
    assert err <= 1e-5 + 1e-6 * float(np.max(np.abs(d[f"{case}/ref64/out"]))), err


def test_causal_conv1d_vs_reference_fixture():
    from mamba2_b200 import causal_conv1d, causal_conv1d_update
    d = F.load("conv")
    x = to_dev(d["x"], "bf16")
    w, b = to_dev(d["w"], "bf16"), to_dev(d["bias"])
    seq = to_dev(d["seq_idx"], int32=True)
    for key, kw in (("plain", {}), ("silu_bias", dict(bias=b, activation="silu")),
                    ("seq", dict(bias=b, activation="silu", seq_idx=seq))):
        o = causal_conv1d(x, w, **kw)
        torch.cuda.synchronize()
        # without a float32 bias the output keeps x's dtype (bf16): one rounding, about 2e-3
        tol = 1e-5 if o.dtype == torch.float32 else 4e-3
        assert rel_l2(o, d[f"{key}/ref64/out"]) <= tol, key
    ns, o = causal_conv1d_update(to_dev(d["x_new"], "bf16"), to_dev(d["state"]), w, bias=b, activation="silu")
    torch.cuda.synchronize()
    assert rel_l2(ns, d["update/ref64/state"]) <= 1e-6
    assert rel_l2(o, d["update/ref64/out"]) <= 1e-5
