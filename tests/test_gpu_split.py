"""Sequence split of the tensor-core forward: with few (batch, head) walks per GPU (one
head-sharded rank of a layer) each sequence is cut into chunk-aligned segments whose entry
states come from a segment-state pass.  Checked against the float64 recurrence
(oracle/ssd_scan.c) with the bf16 bound of the other tests; the number of launches shows
the split ran."""
import pytest
import torch

from gpu_util import TOL
from mamba2_b200 import _lib
from mamba2_b200 import synthetic as S
from test_gpu_fullsize import check_by_group, gpu_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _lib.load()


CASES = [
    # one rank of c2 head-sharded over 8 GPUs: 16 heads, 2 groups -> 8 segments of 512 tokens
    ("c2-rank-of-8", S.scaled(S.CONFIGS["c2"], nheads=16, ngroups=2), 3),
    # one rank of c2 over 4 GPUs, with the z gate
    ("c2-rank-of-4-z", S.scaled(S.CONFIGS["c2"], nheads=32, ngroups=2, has_z=True), 3),
    # N = 256, two batch rows, no initial state
    ("n256-b2", S.SsdConfig("n256", 2, 2048, 8, 64, 1, 256, 128, "bf16", return_final=True), 3),
]


@pytest.mark.parametrize("name,cfg,launches", CASES, ids=[c[0] for c in CASES])
def test_split_walk_vs_recurrence(name, cfg, launches):
    from mamba2_b200.runner import SsdForward
    d = gpu_inputs(cfg, 91)
    r = SsdForward(d["x"], d["dt"], d["A"], d["B"], d["C"], cfg.chunk_size, D=d["D"], z=d["z"],
                   dt_bias=d["dt_bias"], initial_states=d["initial_states"], dt_softplus=True,
                   return_final_states=True)
    assert r.uses_tc and r.launches_per_step == launches
    r()
    torch.cuda.synchronize()
    _lib.check_device_status(r.workspace)
    worst = check_by_group(cfg, d, (r.out, r.final), False)
    print(f"{name}: worst rel-L2 {worst:.3e} (bound {TOL['bf16']})")
