"""GPU check of ssd_combined_fwd_noalloc, the combined forward that takes no workspace.

It exists for callers that cannot allocate device memory where they run the SSD forward
(a handler given only input/output buffers and a stream, or code running where
cudaMalloc is not allowed).  Its scratch is a 16 MiB static device array inside the
library.  This test calls it through the C ABI twice in a row on the same shapes and
compares both results with the workspace entry point ssd_combined_fwd, within the
parity tolerances of the other GPU tests; it also checks that oversized requests are
refused.  The file sorts last so a run that stops at the first failure has already run
every other test.
"""
import ctypes

import pytest
import torch

from mamba2_b200 import _lib
from mamba2_b200 import synthetic as S
from mamba2_b200.kernels.ssd_combined import _fwd_params
from gpu_util import TOL, dev_inputs, rel_l2

pytestmark = pytest.mark.gpu


def _params(cfg, d):
    p, keep = _fwd_params(d["x"], d["dt"], d["A"], d["B"], d["C"], cfg.chunk_size, d["D"], d["z"],
                          d["dt_bias"], d["initial_states"], d["seq_idx"], None, True, (0.0, float("inf")), 0)
    b, L, H, P = d["x"].shape
    N = d["B"].shape[3]
    out = torch.empty((b, L, H, P), device="cuda", dtype=torch.float32)
    final = torch.empty((b, H, P, N), device="cuda", dtype=torch.float32)
    p.out, p.final_states = out.data_ptr(), final.data_ptr()
    return p, keep, out, final


CASES = [
    # bf16, P=64, N=128: the fused tensor-core path (256 bytes of scratch)
    S.scaled(S.CONFIGS["c2"], seqlen=640, nheads=16),
    # fp32: the CUDA-core pipeline, whose chunk states and CB use several MiB of scratch
    S.SsdConfig("f32", 1, 512, 8, 64, 2, 64, 128, "f32", has_z=True, has_init=True, return_final=True),
]


@pytest.mark.parametrize("cfg", CASES, ids=["tensor-core", "cuda-core"])
def test_noalloc_matches_workspace_entry_point(cfg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    d = dev_inputs(S.make_ssd_inputs(cfg, 77), cfg.dtype)
    stream = torch.cuda.current_stream().cuda_stream

    p_ref, keep_ref, out_ref, fin_ref = _params(cfg, d)
    need = lib.ssd_combined_workspace_bytes(p_ref)
    assert need <= _lib.SSD_NOALLOC_SCRATCH_BYTES
    ws = torch.empty(max(need, 1), device="cuda", dtype=torch.uint8)
    _lib.check(lib.ssd_combined_fwd(p_ref, ws.data_ptr(), ws.numel(), stream))

    p, keep, out, fin = _params(cfg, d)
    tol = TOL[cfg.dtype]
    for _ in range(2):   # the second call sees the first call's leftovers in the scratch
        out.fill_(float("nan"))
        fin.fill_(float("nan"))
        _lib.check(lib.ssd_combined_fwd_noalloc(p, stream))
        torch.cuda.synchronize()
        assert torch.isfinite(out).all() and torch.isfinite(fin).all()
        assert rel_l2(out, out_ref.double().cpu().numpy()) <= tol
        assert rel_l2(fin, fin_ref.double().cpu().numpy()) <= tol
        # same kernels, same inputs: the results are in fact bit-identical
        assert torch.equal(out, out_ref) and torch.equal(fin, fin_ref)


def test_noalloc_rejects_oversized_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    cfg = S.SsdConfig("big", 1, 8192, 64, 64, 1, 128, 256, "f32")   # CUDA-core path, > 16 MiB scratch
    d = dev_inputs(S.make_ssd_inputs(cfg, 1), "f32")
    p, keep, out, fin = _params(cfg, d)
    assert lib.ssd_combined_workspace_bytes(p) > _lib.SSD_NOALLOC_SCRATCH_BYTES
    rc = lib.ssd_combined_fwd_noalloc(p, torch.cuda.current_stream().cuda_stream)
    assert rc == 4  # SSD_ERR_WORKSPACE
    assert b"static scratch" in lib.ssd_last_error()
