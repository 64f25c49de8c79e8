"""causal_conv1d / causal_conv1d_update (the step before the SSD, ops/causal_conv1d.py).

CPU: the oracle against the reference's own test procedures (tests/test_mamba2_ops.py:
115-200: a hand-written sliding-window conv, SiLU applied after the conv, the decode step
against the full conv at every position) and the boundary mask in its literal form
(causal_conv1d.py:143-193) against the "seq_idx constant on [t, t+width-1]" form the CUDA
kernels use.  The C-ABI rejects bad arguments before touching the device.
GPU: the CUDA kernels against the oracle in the layer's channels-last layout, contiguous
(batch, dim, seqlen) and odd strides; f32 and bf16; widths 1-5; packed seq_idx; decode loop.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import ssd_ref as R
from mamba2_b200 import _lib


def _manual_conv(x, w, bias):
    """tests/test_mamba2_ops.py:131-138: window sums over the left-padded input."""
    b, d, L = x.shape
    k = w.shape[1]
    xp = np.pad(x, ((0, 0), (0, 0), (k - 1, 0)))
    out = np.zeros_like(x)
    for t in range(L):
        out[:, :, t] = np.sum(xp[:, :, t:t + k] * w[None], axis=-1) + (0 if bias is None else bias[None])
    return out


def test_oracle_conv_matches_manual_window():
    rng = np.random.default_rng(42)
    x, w, bias = rng.standard_normal((2, 8, 16)), rng.standard_normal((8, 4)), rng.standard_normal(8)
    np.testing.assert_allclose(R.causal_conv1d(x, w, bias), _manual_conv(x, w, bias), rtol=0, atol=1e-12)
    # (d, 1, k) weights are the same conv
    np.testing.assert_allclose(R.causal_conv1d(x, w[:, None, :], bias), _manual_conv(x, w, bias), atol=1e-12)


def test_oracle_silu_after_conv():
    rng = np.random.default_rng(7)
    x, w = rng.standard_normal((1, 4, 8)), rng.standard_normal((4, 3))
    np.testing.assert_allclose(R.causal_conv1d(x, w, activation="silu"), R.silu(R.causal_conv1d(x, w)), atol=1e-15)


def test_oracle_update_matches_full_conv():
    """tests/test_mamba2_ops.py:169-200: decode steps from a zero state == the full conv."""
    rng = np.random.default_rng(99)
    x, w, bias = rng.standard_normal((2, 8, 10)), rng.standard_normal((8, 4)), rng.standard_normal(8)
    full = R.causal_conv1d(x, w, bias, activation="silu")
    state = np.zeros((2, 8, 4))
    for t in range(10):
        state, o = R.causal_conv1d_update(x[:, :, t], state, w, bias, activation="silu")
        np.testing.assert_allclose(o, full[:, :, t], atol=1e-12)


@pytest.mark.parametrize("width", [1, 2, 3, 4, 6])
def test_keep_mask_is_constant_run(width):
    """The literal boundary loop == 'seq_idx constant on [t, min(t+width-1, L-1)]'."""
    rng = np.random.default_rng(width)
    L = 57
    lens = [1, 2, 3, 1, 5, 9, 1, 20, 15]
    seq = np.repeat(np.arange(len(lens)), lens)[None].repeat(2, 0)
    seq[1] = np.sort(rng.integers(0, 6, L))
    keep = R.conv1d_keep(seq, width)
    for bi in range(2):
        for t in range(L):
            run = seq[bi, t:min(t + width, L)]
            assert keep[bi, t] == float(np.all(run == run[0])), (bi, t)
    # the quirk: the last width-1 inputs of a sequence are dropped from its own outputs too
    if width > 1:
        assert keep[0, 5] == 0.0 and keep[0, 7] == (1.0 if width <= 5 else 0.0)


def test_capi_conv_rejects_bad_args():
    lib = _lib.load()
    p = _lib.Conv1dParams(batch=1, dim=8, seqlen=16, x_stride_b=128, x_stride_d=16, x_stride_t=1,
                          out_stride_b=128, out_stride_d=16, out_stride_t=1, width=4, dtype=0, out_dtype=0,
                          silu=1)
    assert lib.ssd_causal_conv1d_fwd(ctypes.byref(p), None) == 1        # x, weight, out missing
    p.x, p.weight, p.out, p.width = 16, 32, 48, 9
    assert lib.ssd_causal_conv1d_fwd(ctypes.byref(p), None) == 2        # width 9 unsupported
    p.width, p.dtype = 4, 7
    assert lib.ssd_causal_conv1d_fwd(ctypes.byref(p), None) == 1        # bad dtype enum
    p.dtype, p.out = 0, 16
    assert lib.ssd_causal_conv1d_fwd(ctypes.byref(p), None) == 1        # out aliases x
    assert "alias" in lib.ssd_last_error().decode()
    u = _lib.Conv1dUpdateParams(batch=2, dim=8, state_stride_b=32, state_stride_d=4, width=0)
    assert lib.ssd_causal_conv1d_update(ctypes.byref(u), None) == 2
    assert lib.ssd_causal_conv1d_fwd(None, None) == 1


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def _round(a, dtype):
    return R.round_bf16(a) if dtype == torch.bfloat16 else np.asarray(a, np.float32).astype(np.float64)


def _seq(b, L, rng):
    cuts = np.sort(rng.choice(np.arange(1, L), size=min(L - 1, 7), replace=False))
    lens = np.diff(np.concatenate([[0], cuts, [L]]))
    return np.repeat(np.arange(len(lens)), lens)[None].repeat(b, 0).astype(np.int32)


LAYOUTS = ["channels-last", "contiguous", "strided"]


@pytest.mark.gpu
@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("width,L,seq,silu,bias", [
    (4, 300, False, True, True), (4, 300, True, True, True), (4, 2, False, True, True),
    (3, 129, True, False, False), (2, 64, True, True, True), (1, 77, False, True, True),
    (5, 200, True, True, True)])
def test_conv1d_vs_oracle(layout, dtype, width, L, seq, silu, bias):
    from mamba2_b200 import causal_conv1d
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rng = np.random.default_rng(width * 1000 + L)
    b, d = 2, 96
    xs = _round(rng.standard_normal((b, d, L)), dtype)
    w = _round(rng.standard_normal((d, width)) * 0.5, dtype)
    bs = rng.standard_normal(d).astype(np.float32) if bias else None
    sq = _seq(b, L, rng) if seq and L > 1 else None
    if layout == "channels-last":       # the layer's (b, L, d) activations, viewed (b, d, L)
        xt = torch.from_numpy(xs.transpose(0, 2, 1).copy()).to(dtype).cuda().transpose(1, 2)
    elif layout == "contiguous":
        xt = torch.from_numpy(xs).to(dtype).cuda()
    else:                               # every other channel of a wider buffer
        big = torch.zeros((b, 2 * d, L + 3), dtype=dtype, device="cuda")
        big[:, ::2, 3:] = torch.from_numpy(xs).to(dtype).cuda()
        xt = big[:, ::2, 3:]
    wt = torch.from_numpy(w).to(dtype).cuda()
    bt = None if bs is None else torch.from_numpy(bs).cuda()
    st = None if sq is None else torch.from_numpy(sq).cuda()
    out = causal_conv1d(xt, wt, bias=bt, activation="silu" if silu else None, seq_idx=st)
    torch.cuda.synchronize()
    ref = R.causal_conv1d(xs, w, bs, activation="silu" if silu else None, seq_idx=sq)
    assert out.shape == (b, d, L)
    assert out.dtype == (torch.float32 if (dtype == torch.float32 or bias) else torch.bfloat16)
    got = out.double().cpu().numpy()
    if out.dtype == torch.float32:
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)
    else:
        np.testing.assert_allclose(got, ref, rtol=1e-2, atol=1e-2)
    if sq is not None and width > 1:
        assert R.conv1d_keep(sq, width).min() == 0.0   # the case exercises the boundary mask


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("width", [4, 3])
def test_conv1d_update_loop_matches_full_conv(dtype, width):
    """The reference's decode-consistency procedure on the GPU, in place and functional."""
    from mamba2_b200 import causal_conv1d, causal_conv1d_update
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rng = np.random.default_rng(5 + width)
    b, d, L = 3, 200, 12
    xs = _round(rng.standard_normal((b, d, L)), dtype)
    w = _round(rng.standard_normal((d, width)) * 0.5, dtype)
    bs = rng.standard_normal(d).astype(np.float32)
    xt = torch.from_numpy(xs).to(dtype).cuda()
    wt = torch.from_numpy(w).to(dtype).cuda()
    bt = torch.from_numpy(bs).cuda()
    full = causal_conv1d(xt, wt, bias=bt, activation="silu")
    state = torch.zeros((b, d, width), dtype=dtype, device="cuda")
    ref_state = np.zeros((b, d, width))
    for t in range(L):
        before = state.clone()
        new, o = causal_conv1d_update(xt[:, :, t], state, wt, bias=bt, activation="silu", inplace=(t % 2 == 0))
        if t % 2 == 0:
            assert new.data_ptr() == state.data_ptr()
        else:
            assert torch.equal(state, before)     # functional: the input state is unchanged
        state = new
        ref_state, ref_o = R.causal_conv1d_update(xs[:, :, t], ref_state, w, bs, activation="silu")
        np.testing.assert_allclose(state.double().cpu().numpy(), ref_state, rtol=0, atol=0)
        tol = 1e-5 if dtype == torch.float32 else 1e-2
        np.testing.assert_allclose(o.double().cpu().numpy(), ref_o, rtol=tol, atol=tol)
        torch.testing.assert_close(o, full[:, :, t], rtol=tol, atol=tol)


@pytest.mark.gpu
def test_conv1d_layer_shape_full_size():
    """The c2 layer's conv (dim = d_ssm + 2 G N = 10240, L = 4096, width 4, bf16,
    channels-last): f32 output against the oracle on a slice of channels, and exactly the
    same values as the contiguous-layout kernel on the whole tensor."""
    from mamba2_b200 import causal_conv1d
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = torch.Generator(device="cuda").manual_seed(3)
    b, L, d, k = 1, 4096, 10240, 4
    xbc = torch.randn((b, L, d), generator=g, device="cuda").to(torch.bfloat16)
    w = (0.5 * torch.randn((d, k), generator=g, device="cuda")).to(torch.bfloat16)
    bias = torch.randn((d,), generator=g, device="cuda")
    out = causal_conv1d(xbc.transpose(1, 2), w, bias=bias, activation="silu")
    assert out.stride(1) == 1                      # channels-last in, channels-last out
    alt = causal_conv1d(xbc.transpose(1, 2).contiguous(), w, bias=bias, activation="silu")
    torch.testing.assert_close(out, alt, rtol=0, atol=0)
    sl = slice(1000, 1064)
    ref = R.causal_conv1d(xbc.transpose(1, 2)[:, sl].double().cpu().numpy(), w[sl].double().cpu().numpy(),
                          bias[sl].double().cpu().numpy(), activation="silu")
    np.testing.assert_allclose(out[:, sl].double().cpu().numpy(), ref, rtol=1e-5, atol=1e-5)


def _cl_tensor(xs, dtype, layout):
    b, d, L = xs.shape
    if layout == "channels-last":
        return torch.from_numpy(xs.transpose(0, 2, 1).copy()).to(dtype).cuda().transpose(1, 2)
    if layout == "contiguous":
        return torch.from_numpy(xs).to(dtype).cuda()
    big = torch.zeros((b, 2 * d, L + 3), dtype=dtype, device="cuda")
    big[:, ::2, 3:] = torch.from_numpy(xs).to(dtype).cuda()
    return big[:, ::2, 3:]


_TD = {"f32": torch.float32, "bf16": torch.bfloat16}


@pytest.mark.gpu
@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("xdt", ["f32", "bf16"])
@pytest.mark.parametrize("wdt", ["f32", "bf16"])
@pytest.mark.parametrize("bdt", ["f32", "bf16", None])
@pytest.mark.parametrize("width", [3, 4])
def test_conv1d_capi_independent_param_dtypes(layout, xdt, wdt, bdt, width):
    """The C ABI takes weight and bias in f32 or bf16 independently of x (converted on load):
    every combination, in the three layouts, against the oracle on the same (bf16-representable)
    values.  width 3 with f32 x puts the channels-last kernel's 8-byte weight loads at 24-byte
    offsets."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rng = np.random.default_rng(17 * width + len(layout))
    b, d, L = 2, 96, 150
    xs = _round(rng.standard_normal((b, d, L)), torch.bfloat16)
    w = _round(rng.standard_normal((d, width)) * 0.5, torch.bfloat16)
    bs = _round(rng.standard_normal(d), torch.bfloat16)
    sq = _seq(b, L, rng)
    xt = _cl_tensor(xs, _TD[xdt], layout)
    wt = torch.from_numpy(w).to(_TD[wdt]).cuda().contiguous()
    bt = None if bdt is None else torch.from_numpy(bs).to(_TD[bdt]).cuda()
    st = torch.from_numpy(sq).cuda()
    out = torch.empty((b, L, d), device="cuda").transpose(1, 2)
    p = _lib.Conv1dParams(batch=b, dim=d, seqlen=L, x_stride_b=xt.stride(0), x_stride_d=xt.stride(1),
                          x_stride_t=xt.stride(2), out_stride_b=out.stride(0), out_stride_d=out.stride(1),
                          out_stride_t=out.stride(2), width=width, dtype=_lib.dtype_code(xt),
                          out_dtype=0, silu=1)
    p.x, p.weight, p.bias, p.seq_idx, p.out = xt.data_ptr(), wt.data_ptr(), _lib.ptr(bt), st.data_ptr(), out.data_ptr()
    p.weight_dtype = _lib.dtype_code(wt)
    p.bias_dtype = 0 if bt is None else _lib.dtype_code(bt)
    _lib.check(_lib.load().ssd_causal_conv1d_fwd(p, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ref = R.causal_conv1d(xs, w, None if bdt is None else bs, activation="silu", seq_idx=sq)
    np.testing.assert_allclose(out.double().cpu().numpy(), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("wdt,bdt", [("bf16", "bf16"), ("bf16", "f32"), ("f32", "bf16")])
def test_conv1d_update_capi_param_dtypes(wdt, bdt):
    """Decode steps with an f32 state and bf16 x through the C ABI, weight and bias dtypes
    chosen independently, against the oracle's decode loop."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rng = np.random.default_rng(3)
    b, d, k, steps = 3, 200, 4, 6
    w = _round(rng.standard_normal((d, k)) * 0.5, torch.bfloat16)
    bs = _round(rng.standard_normal(d), torch.bfloat16)
    xs = _round(rng.standard_normal((steps, b, d)), torch.bfloat16)
    wt = torch.from_numpy(w).to(_TD[wdt]).cuda()
    bt = torch.from_numpy(bs).to(_TD[bdt]).cuda()
    state = torch.zeros((b, d, k), device="cuda")
    ref_state = np.zeros((b, d, k))
    lib = _lib.load()
    for t in range(steps):
        xt = torch.from_numpy(xs[t]).to(torch.bfloat16).cuda()
        out = torch.empty((b, d), device="cuda")
        p = _lib.Conv1dUpdateParams(batch=b, dim=d, state_stride_b=state.stride(0), state_stride_d=state.stride(1),
                                    width=k, x_dtype=1, state_dtype=0, out_dtype=0, silu=1)
        p.x_new, p.conv_state, p.weight, p.bias, p.out = (xt.data_ptr(), state.data_ptr(), wt.data_ptr(),
                                                          bt.data_ptr(), out.data_ptr())
        p.weight_dtype, p.bias_dtype = _lib.dtype_code(wt), _lib.dtype_code(bt)
        _lib.check(lib.ssd_causal_conv1d_update(p, torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        ref_state, ref_o = R.causal_conv1d_update(xs[t], ref_state, w, bs, activation="silu")
        np.testing.assert_allclose(state.double().cpu().numpy(), ref_state, rtol=0, atol=0)
        np.testing.assert_allclose(out.double().cpu().numpy(), ref_o, rtol=1e-5, atol=1e-5)
