"""The Mamba2 mixer layer wired from the B200 kernels (modules/mamba2.py:179-520 of the
reference) against the same layer composed from the float64 oracle with the same weights and
the same bf16 rounding points (projection outputs, conv output, the norm's output before
out_proj).  Bound: rel-L2 <= 2e-2 on the layer output (bf16 activations, 1e-2 per stage);
the decode step is checked against the chunked forward of the longer sequence."""
import numpy as np
import pytest
import torch

from oracle import ssd_ref as R
from gpu_util import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _np(t):
    return t.double().cpu().numpy()


def oracle_layer(m, u, seq_idx=None):
    """The reference's forward (modules/mamba2.py:313-425) in float64 with bf16 roundings."""
    b, L, _ = u.shape
    zx = R.round_bf16(u @ _np(m.in_proj_kernel))
    s = np.cumsum([m.d_mlp, m.d_mlp, m.d_ssm, m.conv_dim])
    z0, x0, z, xBC, dt = np.split(zx, s, axis=-1)
    conv = R.causal_conv1d(xBC.transpose(0, 2, 1), _np(m.conv1d_weight),
                           None if m.conv1d_bias is None else _np(m.conv1d_bias), activation="silu",
                           seq_idx=seq_idx)
    xBC = R.round_bf16(conv.transpose(0, 2, 1))
    GN = m.ngroups * m.d_state
    x = xBC[..., :m.d_ssm].reshape(b, L, m.nheads, m.headdim)
    B = xBC[..., m.d_ssm:m.d_ssm + GN].reshape(b, L, m.ngroups, m.d_state)
    C = xBC[..., m.d_ssm + GN:].reshape(b, L, m.ngroups, m.d_state)
    A = -np.exp(_np(m.A_log))
    y = R.ssd_combined(x, dt, A, B, C, m.chunk_size, D=_np(m.D), dt_bias=_np(m.dt_bias), seq_idx=seq_idx,
                       dt_softplus=True)
    y = R.rms_norm_gated(y.reshape(b, L, m.d_ssm), _np(m.norm_weight), z=z,
                         group_size=m.d_ssm // m.ngroups, norm_before_gate=m.norm_before_gate)
    y = R.round_bf16(y)
    if m.d_mlp:
        y = np.concatenate([R.round_bf16(R.silu(z0)) * x0, y], axis=-1)
    return y @ _np(m.out_proj_kernel)


@pytest.mark.parametrize("kw", [dict(d_model=512, ngroups=2, chunk_size=128),
                                dict(d_model=256, d_ssm=384, ngroups=1, chunk_size=256, norm_before_gate=True)],
                         ids=["nemotron-like", "mlp-bypass"])
def test_layer_forward_vs_oracle(kw):
    from mamba2_b200.modules import Mamba2
    m = Mamba2(**kw)
    g = torch.Generator(device="cuda").manual_seed(1)
    u = torch.randn((2, 320, m.d_model), generator=g, device="cuda").to(torch.bfloat16)
    out = m(u)
    torch.cuda.synchronize()
    assert out.shape == (2, 320, m.d_model)
    e = rel_l2(out, oracle_layer(m, _np(u)))
    assert e <= 2e-2, e


def test_layer_packed_sequences_vs_oracle():
    from mamba2_b200.modules import Mamba2
    m = Mamba2(d_model=512, ngroups=2, chunk_size=128)
    g = torch.Generator(device="cuda").manual_seed(2)
    u = torch.randn((1, 400, m.d_model), generator=g, device="cuda").to(torch.bfloat16)
    seq = torch.zeros((1, 400), dtype=torch.int32, device="cuda")
    seq[:, 150:] = 1
    seq[:, 290:] = 2
    out = m(u, seq_idx=seq)
    torch.cuda.synchronize()
    e = rel_l2(out, oracle_layer(m, _np(u), seq_idx=seq.cpu().numpy()))
    assert e <= 2e-2, e


def test_decode_steps_continue_the_prefill():
    """Prefill L tokens with inference_params, then decode 3 tokens one at a time: each step's
    output equals the chunked forward of the whole sequence at that position."""
    from mamba2_b200.modules import Mamba2, allocate_inference_cache
    m = Mamba2(d_model=512, ngroups=2, chunk_size=128)
    g = torch.Generator(device="cuda").manual_seed(3)
    u = torch.randn((2, 131, m.d_model), generator=g, device="cuda").to(torch.bfloat16)
    full = m(u)
    cache = allocate_inference_cache(2, m)
    _, cache = m(u[:, :128], inference_params=cache)
    assert cache["seqlen_offset"] == 128
    for t in range(128, 131):
        o, cache = m(u[:, t:t + 1], inference_params=cache)
        torch.cuda.synchronize()
        e = rel_l2(o[:, 0], _np(full[:, t]))
        assert e <= 2e-2, (t, e)
