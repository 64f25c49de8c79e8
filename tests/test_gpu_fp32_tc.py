"""fp32 inputs on the tensor cores: the staged pipeline's chunk_state, bmm_chunk and
chunk_scan as split-bf16 tcgen05 kernels (csrc/ssd_x3.cu) against the float64 oracle.

The contract for fp32 inputs is rel-L2 <= 1e-4 (TOL["f32"]); the split-bf16 products carry
about 1e-5 relative error each.  Each case also checks that the tensor-core kernels are
what ran (kernel names from the CUDA profiler) and that the CUDA-core stages agree.
"""
import zlib

import pytest
import torch

from oracle import ssd_ref as R
from mamba2_b200 import synthetic as S
from gpu_util import TOL, dev_inputs, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import mamba2_b200._lib as L
    L.load()


F = "f32"
CASES = [
    ("c0-full", S.CONFIGS["c0"]),
    ("c0-init-z", S.scaled(S.CONFIGS["c0"], seqlen=1024, has_z=True, has_init=True, return_final=True)),
    ("Q32-G2", S.SsdConfig("q32", 2, 200, 4, 64, 2, 64, 32, F, has_z=True, has_init=True, return_final=True)),
    ("Q96-ragged", S.SsdConfig("q96", 1, 437, 6, 32, 3, 48, 96, F, return_final=True)),
    ("N256-P128", S.SsdConfig("n256", 1, 600, 2, 128, 1, 256, 128, F, has_init=True, return_final=True)),
    ("P256", S.SsdConfig("p256", 1, 300, 2, 256, 2, 64, 64, F, has_z=True, return_final=True)),
    ("seq_idx", S.SsdConfig("seq", 1, 1024, 4, 64, 2, 128, 256, F, has_init=True, return_final=True,
                            varlen_seqs=6, varlen_range=(1, 400))),
]

X3_KERNELS = ("x3_chunk_state_kernel", "x3_bmm_kernel", "x3_chunk_scan_kernel")


def _run(cfg, d, **kw):
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    return mamba_chunk_scan_combined_fwd(
        d["x"], d["dt"], d["A"], d["B"], d["C"], cfg.chunk_size, D=d["D"], z=d["z"],
        dt_bias=d["dt_bias"], initial_states=d["initial_states"], seq_idx=d["seq_idx"],
        cu_seqlens=d["cu_seqlens"], dt_softplus=True, return_final_states=True,
        return_varlen_states=d["cu_seqlens"] is not None, **kw)


def _kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        out = fn()
        torch.cuda.synchronize()
    return out, {e.name for e in prof.events()}


@pytest.mark.parametrize("name,cfg", CASES, ids=[c[0] for c in CASES])
def test_fp32_tensor_core_stages_vs_oracle(name, cfg):
    inp = S.make_ssd_inputs(cfg, 3000 + zlib.crc32(name.encode()) % 1000)
    d = dev_inputs(inp, F)
    res, names = _kernel_names(lambda: _run(cfg, d))
    for k in X3_KERNELS:
        assert any(k in n for n in names), f"{k} did not run: {sorted(names)}"
    ref = R.ssd_combined(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], cfg.chunk_size, D=inp["D"],
                         z=inp["z"], dt_bias=inp["dt_bias"], initial_states=inp["initial_states"],
                         seq_idx=inp["seq_idx"], cu_seqlens=inp["cu_seqlens"], dt_softplus=True,
                         return_final_states=True, return_varlen_states=inp["cu_seqlens"] is not None)
    for got, want, what in zip(res, ref, ("out", "final", "varlen")):
        assert torch.isfinite(got).all(), what
        e = rel_l2(got, want)
        assert e <= TOL[F], f"{name} {what}: rel-L2 {e:.3e} > {TOL[F]}"
    # the exact fp32 CUDA-core stages on the same inputs agree to the same bound
    simt = _run(cfg, d, force_simt=True)
    torch.cuda.synchronize()
    assert rel_l2(res[0], simt[0].double().cpu().numpy()) <= TOL[F]


def test_fp32_stage_path_switch_selects_cuda_cores():
    import mamba2_b200._lib as L
    cfg = S.scaled(S.CONFIGS["c0"], seqlen=512)
    inp = S.make_ssd_inputs(cfg, 7)
    d = dev_inputs(inp, F)
    with L.fp32_stage_path(L.FP32_STAGES_CUDA_CORES):
        _, names = _kernel_names(lambda: _run(cfg, d))
    assert not any(k in n for n in names for k in X3_KERNELS)
    assert any("chunk_scan_kernel" in n for n in names)
    with pytest.raises(L.SsdError):
        with L.fp32_stage_path(7):
            pass
