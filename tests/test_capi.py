"""CPU checks of the C ABI library: it loads without a GPU, exports every symbol the
header declares, and rejects bad arguments before touching the device."""
import ctypes
import math
import os
import re

import pytest
import torch

from mamba2_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "ssd_b200.h")


def _header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(ssd_\w+)\s*\(", src, flags=re.M)))


def test_header_symbols_exported():
    lib = _lib.load()
    names = _header_functions()
    assert len(names) >= 11, names
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(names) == sorted(_lib.EXPORTED)


def test_abi_version():
    assert _lib.load().ssd_abi_version() == _lib.ABI_VERSION == 2


def _params(**kw):
    p = _lib.SsdFwdParams(batch=1, seqlen=256, nheads=8, headdim=64, ngroups=2, dstate=128,
                          chunk_size=128, dtype=1, dt_dtype=1, dt_softplus=1, D_ndim=0,
                          dt_min=0.0, dt_max=math.inf)
    for k in ("x", "dt", "A", "B", "C", "out"):
        setattr(p, k, 4096)
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("kw,code", [
    (dict(nheads=7), 1),            # H % G
    (dict(chunk_size=48), 2),       # unsupported Q
    (dict(chunk_size=512), 2),
    (dict(out=None), 1),
    (dict(dtype=5), 1),
    (dict(D_ndim=1), 1),            # D missing
    (dict(seqlen=0), 1),
    (dict(dt_min=2.0, dt_max=1.0), 1),
])
def test_combined_rejects(kw, code):
    lib = _lib.load()
    p = _params(**kw)
    rc = lib.ssd_combined_fwd(p, 256, 1 << 40, None)
    assert rc == code
    assert len(lib.ssd_last_error()) > 0


def test_workspace_checks():
    lib = _lib.load()
    p = _params()
    need = lib.ssd_combined_workspace_bytes(p)
    assert need > 0
    assert lib.ssd_combined_fwd(p, None, need, None) == 4
    assert lib.ssd_combined_fwd(p, 256, need - 1, None) == 4
    assert lib.ssd_combined_fwd(p, 257, need, None) == 3


def test_varlen_requires_batch1():
    lib = _lib.load()
    p = _params(batch=2, varlen_states=4096, cu_seqlens=4096, num_seqs=3)
    assert lib.ssd_combined_fwd(p, 256, 1 << 40, None) == 1
    assert b"batch=1" in lib.ssd_last_error()


def test_ssu_rejects():
    lib = _lib.load()
    p = _lib.SsuParams(batch=2, nheads=4, headdim=8, ngroups=3, dstate=16, dt_ndim=2, A_ndim=1)
    assert lib.ssd_selective_state_update(p, None) == 1
    p.ngroups = 2
    assert lib.ssd_selective_state_update(p, None) == 1  # null pointers


def test_python_api_refuses_cpu_tensors():
    from mamba2_b200 import mamba_chunk_scan_combined_fwd, selective_state_update
    x = torch.zeros(1, 64, 2, 8)
    dt = torch.zeros(1, 64, 2)
    A = -torch.ones(2)
    B = torch.zeros(1, 64, 1, 16)
    with pytest.raises(ValueError, match="CUDA"):
        mamba_chunk_scan_combined_fwd(x, dt, A, B, B, 64)
    with pytest.raises(ValueError, match="CUDA"):
        selective_state_update(torch.zeros(1, 2, 8, 16), x[:, 0], dt[:, 0], A, B[:, 0], B[:, 0])


@pytest.mark.parametrize("kw", [dict(chunk_size=0), dict(batch=-1), dict(seqlen=-5), dict(nheads=0),
                                dict(dstate=-128)])
def test_invalid_dims_rejected_before_sizing(kw):
    """Sizing returns 0 for invalid params (no division by a zero chunk size), and both
    entry points report SSD_ERR_INVALID_ARG without touching a device."""
    lib = _lib.load()
    p = _params(**kw)
    assert lib.ssd_combined_workspace_bytes(p) == 0
    assert lib.ssd_combined_fwd_noalloc(p, None) == 1
    assert b"positive" in lib.ssd_last_error()
    assert lib.ssd_combined_fwd(p, 256, 1 << 40, None) == 1


def test_status_decode():
    lib = _lib.load()
    assert lib.ssd_status_decode(0) == 0
    assert lib.ssd_status_decode(0x100 | 7) == 6          # SSD_ERR_TIMEOUT
    assert b"bounded wait" in lib.ssd_last_error()
    assert lib.ssd_status_decode(0x200) == 3              # SSD_ERR_ALIGNMENT
    assert lib.ssd_status_decode(0xdead) == 5
    assert lib.ssd_status_copy_async(None, 4096, None) == 1


def test_dispatch_is_the_reference_keyword_call():
    """mamba2_b200.dispatch._ssd_combined_fwd takes the reference module's keyword-only call
    (src/mamba2_jax/modules/mamba2.py:377-389) and has no fallback: CPU tensors raise."""
    import inspect
    from mamba2_b200 import dispatch
    from mamba2_b200.kernels.ssd_combined import mamba_chunk_scan_combined_fwd
    params = inspect.signature(mamba_chunk_scan_combined_fwd).parameters
    for k in ("x", "dt", "A", "B", "C", "chunk_size", "D", "z", "dt_bias", "initial_states", "seq_idx",
              "cu_seqlens", "dt_softplus", "dt_limit", "return_final_states", "return_varlen_states"):
        assert k in params, k
    x = torch.zeros(1, 64, 2, 8)
    with pytest.raises(ValueError, match="CUDA"):
        dispatch._ssd_combined_fwd(use_pallas=True, x=x, dt=torch.zeros(1, 64, 2), A=-torch.ones(2),
                                   B=torch.zeros(1, 64, 1, 16), C=torch.zeros(1, 64, 1, 16), chunk_size=64,
                                   D=torch.ones(2), z=None, dt_bias=torch.zeros(2), initial_states=None,
                                   seq_idx=None, dt_softplus=True, dt_limit=(0.0, float("inf")),
                                   return_final_states=True)
