"""rms_norm_gated (the step after the SSD, ops/rms_norm.py).

CPU: the oracle against the reference's own test procedures (tests/test_mamba2_ops.py:
205-290: plain RMSNorm by hand, the gate before and after the norm, grouped RMS by a
reshape), and the C-ABI rejects bad arguments before touching the device.
GPU: the CUDA kernels against the oracle for f32/bf16 inputs, gate on/off and both gate
orders, group sizes on the register-cached path (256..2048) and on the general path (odd
sizes, unaligned rows), and the layer's full-size call (group = d_ssm / G = 1024).
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import ssd_ref as R
from mamba2_b200 import _lib


def _silu(v):
    return v / (1.0 + np.exp(-v))


def test_oracle_basic_matches_hand_formula():
    """tests/test_mamba2_ops.py:205-227: weight = 1, no gate."""
    rng = np.random.default_rng(42)
    x = rng.standard_normal((2, 8, 16))
    ref = x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + 1e-5)
    assert np.max(np.abs(R.rms_norm_gated(x, np.ones(16)) - ref)) < 1e-12


def test_oracle_gate_orders():
    """tests/test_mamba2_ops.py:230-261: norm(x)*w*silu(z) and norm(x*silu(z))*w."""
    rng = np.random.default_rng(43)
    x, z, w = rng.standard_normal((2, 16)), rng.standard_normal((2, 16)), rng.standard_normal(16)
    rms = np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + 1e-5)
    np.testing.assert_allclose(R.rms_norm_gated(x, w, z=z), x / rms * w * _silu(z), rtol=1e-12)
    xz = x * _silu(z)
    rms2 = np.sqrt(np.mean(xz * xz, axis=-1, keepdims=True) + 1e-5)
    np.testing.assert_allclose(R.rms_norm_gated(x, w, z=z, norm_before_gate=False), xz / rms2 * w,
                               rtol=1e-12)


def test_oracle_grouped():
    """tests/test_mamba2_ops.py:264-290: group_size 8 of hidden 32 by reshape."""
    rng = np.random.default_rng(44)
    x = rng.standard_normal((2, 32))
    xg = x.reshape(2, 4, 8)
    ref = (xg / np.sqrt(np.mean(xg * xg, axis=-1, keepdims=True) + 1e-5)).reshape(2, 32)
    np.testing.assert_allclose(R.rms_norm_gated(x, np.ones(32), group_size=8), ref, rtol=1e-12)
    # group_size == hidden is the ungrouped form
    np.testing.assert_allclose(R.rms_norm_gated(x, np.ones(32), group_size=32), R.rms_norm_gated(x, np.ones(32)))


def test_capi_rms_norm_rejects_bad_args():
    lib = _lib.load()
    p = _lib.RmsNormParams(rows=4, hidden=64, group_size=16, x_stride_row=64, z_stride_row=64,
                           out_stride_row=64, eps=1e-5, norm_before_gate=1)
    assert lib.ssd_rms_norm_gated(ctypes.byref(p), None) == 1          # x, weight, out missing
    p.x, p.weight, p.out = 256, 512, 1024
    p.group_size = 24
    assert lib.ssd_rms_norm_gated(ctypes.byref(p), None) == 1          # 64 % 24 != 0
    assert "multiple" in lib.ssd_last_error().decode()
    p.group_size, p.x_dtype = 16, 5
    assert lib.ssd_rms_norm_gated(ctypes.byref(p), None) == 1          # bad dtype enum
    p.x_dtype, p.out_stride_row = 0, 32
    assert lib.ssd_rms_norm_gated(ctypes.byref(p), None) == 1          # row stride < hidden
    p.out_stride_row, p.eps = 64, -1.0
    assert lib.ssd_rms_norm_gated(ctypes.byref(p), None) == 1          # negative eps
    assert lib.ssd_rms_norm_gated(None, None) == 1


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def _round(a, dtype):
    return R.round_bf16(a) if dtype == torch.bfloat16 else np.asarray(a, np.float32).astype(np.float64)


DT = {"f32": torch.float32, "bf16": torch.bfloat16}


@pytest.mark.gpu
@pytest.mark.parametrize("xdt,zdt,wdt", [("f32", "f32", "f32"), ("f32", "bf16", "f32"),
                                         ("bf16", "bf16", "bf16"), ("bf16", "bf16", "f32"),
                                         ("bf16", None, "bf16")])
@pytest.mark.parametrize("hidden,gs", [(1024, 256), (2048, 512), (8192, 1024), (4096, 2048),
                                       (96, 24), (16, None), (600, 200)])
@pytest.mark.parametrize("nbg", [True, False])
def test_rms_norm_vs_oracle(xdt, zdt, wdt, hidden, gs, nbg):
    from mamba2_b200 import rms_norm_gated
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if zdt is None and not nbg:
        pytest.skip("the gate order only matters with z")
    rng = np.random.default_rng(hidden + (gs or 0) + 7 * nbg)
    shape = (2, 37, hidden)
    x = _round(rng.standard_normal(shape), DT[xdt])
    z = None if zdt is None else _round(rng.standard_normal(shape), DT[zdt])
    w = _round(rng.standard_normal(hidden), DT[wdt])
    xt = torch.from_numpy(x).to(DT[xdt]).cuda()
    zt = None if z is None else torch.from_numpy(z).to(DT[zdt]).cuda()
    wt = torch.from_numpy(w).to(DT[wdt]).cuda()
    out = rms_norm_gated(xt, wt, z=zt, group_size=gs, norm_before_gate=nbg)
    torch.cuda.synchronize()
    ref = R.rms_norm_gated(x, w, z=z, group_size=gs, norm_before_gate=nbg)
    all_bf16 = xdt == "bf16" and wdt == "bf16" and zdt in (None, "bf16")
    assert out.dtype == (torch.bfloat16 if all_bf16 else torch.float32)
    assert out.shape == shape
    got = out.double().cpu().numpy()
    if out.dtype == torch.float32:
        # the reference's own bound for the gated forms (tests/test_mamba2_ops.py:258-259)
        assert np.max(np.abs(got - ref)) < 1e-5
    else:
        assert R.rel_l2(got, ref) <= 1e-2
        np.testing.assert_allclose(got, ref, rtol=1e-2, atol=1e-2)


@pytest.mark.gpu
def test_rms_norm_strided_rows_and_inplace():
    """Rows addressed by a stride (a column slice of a wider buffer) go through without a
    copy; an unaligned row start takes the general kernel; out values equal in both."""
    from mamba2_b200 import rms_norm_gated
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = torch.Generator(device="cuda").manual_seed(5)
    big = torch.randn((64, 2048 + 8), generator=g, device="cuda")
    w = torch.randn((1024,), generator=g, device="cuda")
    aligned = big[:, 8:8 + 1024]           # 32-byte aligned rows, stride 2056
    unaligned = big[:, 3:3 + 1024]         # 12-byte offset: general kernel
    for view in (aligned, unaligned):
        out = rms_norm_gated(view, w, group_size=256)
        ref = R.rms_norm_gated(view.double().cpu().numpy(), w.double().cpu().numpy(), group_size=256)
        assert np.max(np.abs(out.double().cpu().numpy() - ref)) < 1e-5


@pytest.mark.gpu
def test_rms_norm_layer_shape_full_size():
    """The c2 layer's norm: SSD output y (1, 4096, 8192) f32, z bf16, weight f32,
    group = d_ssm / G = 1024; oracle on a slice of rows, and the cached kernel equal to the
    general kernel (forced by an unaligned copy) to within rounding on the whole tensor."""
    from mamba2_b200 import rms_norm_gated
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = torch.Generator(device="cuda").manual_seed(9)
    b, L, d, G = 1, 4096, 8192, 8
    y = torch.randn((b, L, d), generator=g, device="cuda")
    z = torch.randn((b, L, d), generator=g, device="cuda").to(torch.bfloat16)
    w = 1.0 + 0.1 * torch.randn((d,), generator=g, device="cuda")
    out = rms_norm_gated(y, w, z=z, group_size=d // G)
    assert out.dtype == torch.float32
    rows = slice(1000, 1032)
    ref = R.rms_norm_gated(y[0, rows].double().cpu().numpy(), w.double().cpu().numpy(),
                           z=z[0, rows].double().cpu().numpy(), group_size=d // G)
    assert np.max(np.abs(out[0, rows].double().cpu().numpy() - ref)) < 1e-5
    buf = torch.empty((b * L * d + 1,), device="cuda")
    y_un = buf[1:].view(b, L, d)
    y_un.copy_(y)
    alt = rms_norm_gated(y_un, w, z=z, group_size=d // G)
    torch.testing.assert_close(out, alt, rtol=1e-6, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("nbg", [True, False])
def test_rms_norm_bf16_out_is_the_f32_result_rounded_once(nbg):
    """out_dtype=bfloat16 (the layer's out_proj input) gives the float32 result rounded once,
    from the same pass: bit-identical to casting the float32 output."""
    from mamba2_b200 import rms_norm_gated
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = torch.Generator(device="cuda").manual_seed(21)
    for hidden, gs in ((2048, 1024), (1200, 400)):   # register-cached kernel and the general one
        y = torch.randn((2, 300, hidden), generator=g, device="cuda")
        z = torch.randn((2, 300, hidden), generator=g, device="cuda").to(torch.bfloat16)
        w = 1.0 + 0.1 * torch.randn((hidden,), generator=g, device="cuda")
        o32 = rms_norm_gated(y, w, z=z, group_size=gs, norm_before_gate=nbg)
        o16 = rms_norm_gated(y, w, z=z, group_size=gs, norm_before_gate=nbg, out_dtype=torch.bfloat16)
        assert o32.dtype == torch.float32 and o16.dtype == torch.bfloat16
        assert torch.equal(o16, o32.to(torch.bfloat16))
    with pytest.raises(ValueError):
        rms_norm_gated(y, w, z=z, group_size=400, out_dtype=torch.float16)
