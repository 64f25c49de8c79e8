"""The SSD_DEBUG build (libssd_b200_debug.so, `build.py --debug`): every global index the
fused kernel computes is checked against its tensor's extent, and an out-of-range index is
skipped and reported through the device status word instead of being accessed.  On shapes
that reach every checked access (ragged lengths, z and out_x, initial and final states,
packed varlen states, the sequence split) the debug build must report nothing and give
bit-identical results to the release build."""
import ctypes

import pytest
import torch

from gpu_util import dev_inputs
from mamba2_b200 import _lib
from mamba2_b200 import synthetic as S
from mamba2_b200.kernels.ssd_combined import _fwd_params

pytestmark = pytest.mark.gpu


def _open(path):
    lib = ctypes.CDLL(str(path))
    P = ctypes.POINTER
    lib.ssd_combined_workspace_bytes.argtypes = [P(_lib.SsdFwdParams)]
    lib.ssd_combined_workspace_bytes.restype = ctypes.c_size_t
    lib.ssd_combined_fwd.argtypes = [P(_lib.SsdFwdParams), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.ssd_status_copy_async.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.ssd_status_decode.argtypes = [ctypes.c_uint32]
    lib.ssd_last_error.restype = ctypes.c_char_p
    lib.ssd_abi_version.restype = ctypes.c_int
    assert lib.ssd_abi_version() == _lib.ABI_VERSION
    return lib


CASES = [
    ("c2-small", S.scaled(S.CONFIGS["c2"], seqlen=640, nheads=16)),
    ("ragged-z", S.SsdConfig("rz", 2, 333, 8, 64, 8, 128, 128, "bf16", has_z=True, has_init=True, return_final=True)),
    ("varlen-n256", S.scaled(S.CONFIGS["c3"], seqlen=1024, nheads=16, varlen_seqs=5, varlen_range=(32, 400))),
    ("split", S.scaled(S.CONFIGS["c2"], nheads=16, ngroups=1)),
]


@pytest.mark.parametrize("name,cfg", CASES, ids=[c[0] for c in CASES])
def test_debug_build_reports_nothing_and_matches(name, cfg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not _lib.LIB_PATH.with_name("libssd_b200_debug.so").exists():
        pytest.fail("libssd_b200_debug.so missing: build it with `python mamba2-jax-pallas_b200/build.py --debug`")
    rel, dbg = _open(_lib.LIB_PATH), _open(_lib.LIB_PATH.with_name("libssd_b200_debug.so"))
    d = dev_inputs(S.make_ssd_inputs(cfg, 5), cfg.dtype)
    stream = torch.cuda.current_stream().cuda_stream
    results = []
    for lib in (rel, dbg):
        p, keep = _fwd_params(d["x"], d["dt"], d["A"], d["B"], d["C"], cfg.chunk_size, d["D"], d["z"], d["dt_bias"],
                              d["initial_states"], d["seq_idx"], d["cu_seqlens"], True, (0.0, float("inf")), 0)
        b, L, H, P = d["x"].shape
        N = d["B"].shape[3]
        out = torch.full((b, L, H, P), float("nan"), device="cuda")
        fin = torch.full((b, H, P, N), float("nan"), device="cuda")
        p.out, p.final_states = out.data_ptr(), fin.data_ptr()
        outs = [out, fin]
        if d["z"] is not None:
            out_x = torch.full_like(out, float("nan"))
            p.out_x = out_x.data_ptr()
            outs.append(out_x)
        if d["cu_seqlens"] is not None:
            vs = torch.full((p.num_seqs, H, P, N), float("nan"), device="cuda")
            p.varlen_states = vs.data_ptr()
            outs.append(vs)
        n = lib.ssd_combined_workspace_bytes(p)
        ws = torch.empty(n, device="cuda", dtype=torch.uint8)
        assert lib.ssd_combined_fwd(p, ws.data_ptr(), n, stream) == 0, lib.ssd_last_error()
        word = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert lib.ssd_status_copy_async(ws.data_ptr(), word.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        rc = lib.ssd_status_decode(int(word.item()) & 0xFFFFFFFF)
        assert rc == 0, (name, hex(int(word.item())), lib.ssd_last_error())
        results.append(outs)
    for a, b_ in zip(*results):
        assert torch.equal(a, b_), name
