"""GPU checks of the failure reporting and of the drop-in call:

- a bounded wait inside the fused kernel that gives up is reported to the caller
  (SSD_FLAG_TEST_WAIT_TIMEOUT makes every CTA wait on a barrier that nothing arrives on,
  with a short limit, before it issues any copy or MMA), and the context stays usable;
- the reference module's keyword call (modules/mamba2.py:377-389) through
  mamba2_b200.dispatch._ssd_combined_fwd;
- one process driving the fused kernel on two GPUs (the per-device kernel attribute).
"""
import pytest
import torch

from gpu_util import dev_inputs, rel_l2
from mamba2_b200 import _lib
from mamba2_b200 import synthetic as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _lib.load()


CFG = S.scaled(S.CONFIGS["c2"], seqlen=384, nheads=16)


def _run(d, flags=0, device="cuda"):
    from mamba2_b200.runner import SsdForward
    r = SsdForward(d["x"], d["dt"], d["A"], d["B"], d["C"], CFG.chunk_size, D=d["D"], dt_bias=d["dt_bias"],
                   initial_states=d["initial_states"], dt_softplus=True, return_final_states=True, flags=flags)
    assert r.uses_tc
    r()
    return r


def test_timeout_is_reported_and_context_survives():
    d = dev_inputs(S.make_ssd_inputs(CFG, 3), "bf16")
    ok = _run(d)
    _lib.check_device_status(ok.workspace)          # a normal launch leaves the word at 0
    want = ok.out.clone()
    bad = _run(d, flags=_lib.SSD_FLAG_TEST_WAIT_TIMEOUT)
    with pytest.raises(_lib.SsdError) as ei:
        _lib.check_device_status(bad.workspace)
    assert ei.value.code == 6 and "bounded wait" in str(ei.value)
    # the context is still usable and the next launch clears the word
    again = _run(d)
    _lib.check_device_status(again.workspace)
    torch.cuda.synchronize()
    assert torch.equal(again.out, want)


def test_check_status_keyword():
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    d = dev_inputs(S.make_ssd_inputs(CFG, 4), "bf16")
    out = mamba_chunk_scan_combined_fwd(d["x"], d["dt"], d["A"], d["B"], d["C"], CFG.chunk_size, D=d["D"],
                                        dt_bias=d["dt_bias"], dt_softplus=True, check_status=True)
    assert torch.isfinite(out).all()


def test_dispatch_reference_keyword_call():
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    from mamba2_b200.dispatch import _ssd_combined_fwd
    cfg = S.scaled(S.CONFIGS["c2"], seqlen=256, nheads=16, has_z=True)
    d = dev_inputs(S.make_ssd_inputs(cfg, 5), "bf16")
    y, fin = _ssd_combined_fwd(
        x=d["x"], dt=d["dt"], A=d["A"], B=d["B"], C=d["C"], chunk_size=cfg.chunk_size, D=d["D"], z=d["z"],
        dt_bias=d["dt_bias"], dt_softplus=True, dt_limit=(0.0, float("inf")), seq_idx=None, cu_seqlens=None,
        return_final_states=True, return_varlen_states=False)
    y2, fin2 = mamba_chunk_scan_combined_fwd(d["x"], d["dt"], d["A"], d["B"], d["C"], cfg.chunk_size, D=d["D"],
                                             z=d["z"], dt_bias=d["dt_bias"], dt_softplus=True,
                                             return_final_states=True)
    torch.cuda.synchronize()
    assert torch.equal(y, y2) and torch.equal(fin, fin2)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_one_process_two_devices():
    """The fused kernel's shared-memory attribute is set per device: the same process runs it
    on GPU 0, then GPU 1, then GPU 0 again, with identical results."""
    inp = S.make_ssd_inputs(CFG, 6)
    outs = []
    for dev in (0, 1, 0):
        with torch.cuda.device(dev):
            d = {k: (None if v is None else v.to(f"cuda:{dev}")) for k, v in dev_inputs(inp, "bf16").items()}
            r = _run(d)
            torch.cuda.synchronize()
            _lib.check_device_status(r.workspace)
            outs.append(r.out.cpu())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
