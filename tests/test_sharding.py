"""Multi-GPU partitioning (mamba2_b200.sharding).

CPU: head ranges of every BASELINE shape at 1/2/4/8 ranks; the sequence-parallel state
exchange over 2 and 4 gloo ranks against a sequential scan; the sequence-parallel
algorithm (per-segment pass from a zero state, exclusive prefix, rerun with the received
state) against the float64 oracle of the whole sequence, with and without packed seq_idx.
GPU: the sequence-parallel forward through the CUDA path on two gloo ranks sharing cuda:0
(the ranks only exchange between launches, never inside a kernel).
"""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import ssd_ref as R
from mamba2_b200 import sharding as SH
from mamba2_b200 import synthetic as S


# ---------------------------------------------------------------------------
# head sharding
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("H,G", [(24, 1), (80, 1), (128, 8), (256, 8), (112, 8)])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_range_partitions(H, G, world):
    hpg = H // G
    ok = G % world == 0 or (world % G == 0 and hpg % (world // G) == 0)
    if not ok:
        with pytest.raises(ValueError):
            SH.head_range(H, G, world, 0)
        return
    ranges = [SH.head_range(H, G, world, r) for r in range(world)]
    assert [h for a, b in ranges for h in range(a, b)] == list(range(H))
    for r, (a, b) in enumerate(ranges):
        assert b - a == H // world
        g0, g1 = SH.group_range(H, G, world, r)
        assert all(g0 <= h // hpg < g1 for h in range(a, b))
        assert (g1 - g0) * hpg >= b - a


def test_shard_heads_slices():
    cfg = S.SsdConfig("s", 2, 96, 16, 8, 4, 16, 32, "f32", has_z=True, has_init=True)
    inp = {k: (torch.from_numpy(np.ascontiguousarray(v)) if isinstance(v, np.ndarray) else v)
           for k, v in S.make_ssd_inputs(cfg, 3).items()}
    parts = [SH.shard_heads(inp, 2, r) for r in range(2)]
    torch.testing.assert_close(torch.cat([p["x"] for p in parts], 2), inp["x"])
    torch.testing.assert_close(torch.cat([p["z"] for p in parts], 2), inp["z"])
    torch.testing.assert_close(torch.cat([p["initial_states"] for p in parts], 1), inp["initial_states"])
    torch.testing.assert_close(torch.cat([p["A"] for p in parts]), inp["A"])
    assert parts[0]["B"].shape[2] == 2 and parts[1]["C"].shape[2] == 2
    torch.testing.assert_close(parts[1]["B"], inp["B"][:, :, 2:4])


def test_seq_segments_are_chunk_aligned():
    for L, Q, world in [(32768, 128, 8), (1000, 64, 3), (640, 128, 2), (100, 128, 2)]:
        segs = [SH.seq_segment(L, Q, world, r) for r in range(world)]
        assert segs[0][0] == 0 and segs[-1][1] == L
        assert all(segs[r][1] == segs[r + 1][0] for r in range(world - 1))
        assert all(t0 % Q == 0 for t0, _ in segs)


# ---------------------------------------------------------------------------
# the exchange over gloo ranks
# ---------------------------------------------------------------------------
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _pair(rank):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.rand(2, 3, generator=g), torch.randn(2, 3, 4, 5, generator=g)


def _prefix_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    a, s = _pair(rank)
    ea, es = SH.exclusive_prefix(a, s)
    q.put((rank, ea.numpy(), es.numpy()))
    dist.destroy_process_group()


def _run_ranks(target, world, *args):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            item = q.get(timeout=240)
            res[item[0]] = item[1:]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    return res


@pytest.mark.parametrize("world", [2, 4])
def test_exclusive_prefix_gloo(world):
    res = _run_ranks(_prefix_worker, world)
    acc_a, acc_s = torch.ones(2, 3), torch.zeros(2, 3, 4, 5)
    for r in range(world):
        np.testing.assert_allclose(res[r][0], acc_a.numpy(), rtol=1e-6)
        np.testing.assert_allclose(res[r][1], acc_s.numpy(), rtol=1e-5, atol=1e-6)
        acc_a, acc_s = SH.combine(acc_a, acc_s, *_pair(r))


def _failing_prefix_worker(rank, world, port, q):
    """Rank 1 dies before the exchange; the others run it with a 5 s bound per round."""
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    if rank == 1:
        os._exit(3)
    a, s = _pair(rank)
    try:
        SH.exclusive_prefix(a, s, timeout=datetime.timedelta(seconds=5))
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001 - the failure is the point
        q.put((rank, f"error: {type(e).__name__}"))
    q.close()
    q.join_thread()      # flush the message before the hard exit
    os._exit(0)


def test_exclusive_prefix_peer_failure_is_detected():
    """A rank that exits instead of joining the exchange makes the rank that needs its
    partial (rank 2 receives from rank 1 in the first round) raise within the bound, with no
    hang; rank 0, which receives nothing, may finish."""
    import time
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 3
    procs = [ctx.Process(target=_failing_prefix_worker, args=(r, world, port, q)) for r in range(world)]
    t0 = time.time()
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world - 1):
            r, msg = q.get(timeout=120)
            res[r] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert procs[1].exitcode == 3
    assert res[2].startswith("error"), res
    assert time.time() - t0 < 110


# ---------------------------------------------------------------------------
# the algorithm against the oracle (float64)
# ---------------------------------------------------------------------------
def _segment_inputs(inp, t0, t1):
    out = dict(inp)
    for k in ("x", "dt", "B", "C", "z"):
        if inp.get(k) is not None:
            out[k] = inp[k][:, t0:t1]
    return out


def _oracle(inp, Q, init, seq):
    return R.ssd_combined(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], Q, D=inp["D"], z=inp["z"],
                          dt_bias=inp["dt_bias"], initial_states=init, seq_idx=seq, dt_softplus=True,
                          return_final_states=True)


@pytest.mark.parametrize("lens", [None, [100, 230, 60, 250], [320, 320]], ids=["one-seq", "packed", "cut-at-segment"])
@pytest.mark.parametrize("world", [2, 3])
def test_sequence_parallel_algorithm_matches_oracle(world, lens):
    L, Q = 640, 64
    cfg = S.SsdConfig("sp", 1, L, 4, 16, 2, 32, Q, "f32", has_z=True, has_init=True, return_final=True)
    inp = S.make_ssd_inputs(cfg, 7)
    seq = None if lens is None else np.repeat(np.arange(len(lens)), lens)[None].astype(np.int32)
    full_out, full_final = _oracle(inp, Q, inp["initial_states"], seq)
    acc_a, acc_s = np.ones((1, 4)), np.zeros_like(full_final)
    outs = []
    for r in range(world):
        t0, t1 = SH.seq_segment(L, Q, world, r)
        sin = _segment_inputs(inp, t0, t1)
        sq = None
        if seq is not None:
            sq = seq[:, t0:t1]
            if r > 0:
                sq = SH.relabel_seq_idx(torch.from_numpy(sq), torch.from_numpy(seq[:, t0 - 1])).numpy()
        out_loc, s_loc = _oracle(sin, Q, inp["initial_states"] if r == 0 else None, sq)
        dA, _ = R.chunk_cumsum(sin["dt"], inp["A"], Q, inp["dt_bias"], True)
        a = np.exp(dA[..., -1].sum(-1))
        if sq is not None:
            a = a * (sq[:, -1] == 0)[:, None]
        if r == 0:
            outs.append(out_loc)
            a = np.zeros_like(a)
        else:
            # fix-up: the received state's term on the carried tokens (what the CUDA fix-up does)
            clen = (t1 - t0) if sq is None else int(SH.carried_len(torch.from_numpy(sq))[0])
            o2 = out_loc.copy()
            seg_L = t1 - t0
            dt_full = R.chunk_cumsum(sin["dt"], inp["A"], seg_L, inp["dt_bias"], True)[0][..., 0, :seg_L]
            hpg = 4 // 2
            for t in range(clen):
                for h in range(4):
                    g = h // hpg
                    y = np.exp(dt_full[0, h, t]) * (acc_s[0, h] @ sin["C"][0, t, g])
                    o2[0, t, h] += y * R.silu(np.float64(sin["z"][0, t, h]))
            outs.append(o2)
            if clen == seg_L:
                s_loc = s_loc + np.exp(dt_full[0, :, seg_L - 1])[:, None, None] * acc_s[0][None]
        if r == 0:
            acc_a, acc_s = acc_a * a, a[..., None, None] * acc_s + s_loc
        else:
            acc_a, acc_s = acc_a * a, s_loc      # s_loc already carries the received state
    np.testing.assert_allclose(np.concatenate(outs, 1), full_out, rtol=1e-9, atol=1e-9)
    np.testing.assert_allclose(acc_s, full_final, rtol=1e-9, atol=1e-9)


# ---------------------------------------------------------------------------
# the CUDA path, two ranks on one GPU
# ---------------------------------------------------------------------------
def _sp_gpu_worker(rank, world, port, q, lens, backend="gloo"):
    import torch.distributed as dist
    from gpu_util import dev_inputs, rel_l2, to_dev
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if backend == "nccl":   # one GPU per rank, the exchange over NCCL
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    else:
        dist.init_process_group("gloo", rank=rank, world_size=world)
    L, Q = 1024, 128
    cfg = S.SsdConfig("sp", 1, L, 8, 64, 2, 128, Q, "bf16", has_z=True, has_init=True, return_final=True)
    inp = S.make_ssd_inputs(cfg, 21)
    seq = None if lens is None else np.repeat(np.arange(len(lens)), lens)[None].astype(np.int32)
    full_out, full_final = _oracle(inp, Q, inp["initial_states"], seq)
    t0, t1 = SH.seq_segment(L, Q, world, rank)
    d = dev_inputs(_segment_inputs(inp, t0, t1), "bf16")
    sq = None if seq is None else to_dev(seq[:, t0:t1], int32=True)
    prev = None if seq is None or rank == 0 else to_dev(seq[:, t0 - 1], int32=True)
    out, final = SH.ssd_forward_sequence_parallel(
        d["x"], d["dt"], d["A"], d["B"], d["C"], Q, D=d["D"], z=d["z"], dt_bias=d["dt_bias"],
        initial_states=d["initial_states"], seq_idx=sq, prev_seq=prev, dt_softplus=True)
    torch.cuda.synchronize()
    e_out = rel_l2(out, full_out[:, t0:t1])
    e_fin = rel_l2(final, full_final) if rank == world - 1 else 0.0
    q.put((rank, e_out, e_fin))
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("lens", [None, [300, 500, 224], [300, 212, 512]],
                         ids=["one-seq", "packed", "new-seq-at-segment"])
def test_sequence_parallel_forward_two_ranks_one_gpu(lens):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    res = _run_ranks(_sp_gpu_worker, 2, lens)
    for r in range(2):
        assert res[r][0] <= 1e-2, (r, res[r])
        assert res[r][1] <= 1e-2, (r, res[r])


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("lens", [None, [300, 212, 512]], ids=["one-seq", "new-seq-at-segment"])
def test_sequence_parallel_forward_two_gpus_nccl(lens):
    """The same check with one GPU per rank and the state exchange over NCCL."""
    res = _run_ranks(_sp_gpu_worker, 2, lens, "nccl")
    for r in range(2):
        assert res[r][0] <= 1e-2, (r, res[r])
        assert res[r][1] <= 1e-2, (r, res[r])


def test_carried_len():
    sq = torch.tensor([[0, 0, 0, 1, 1, 2, 2, 2], [0, 0, 0, 0, 0, 1, 1, 1]], dtype=torch.int32)
    assert SH.carried_len(sq).tolist() == [3, 5]
    assert SH.carried_len(torch.zeros((1, 8), dtype=torch.int32)).tolist() == [8]
    assert SH.carried_len(torch.ones((1, 8), dtype=torch.int32)).tolist() == [0]


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_sharded_outputs_bitwise_equal(world):
    """Each rank's head block, run alone, gives bit-identical outputs and final states to the
    same heads of the whole-layer run (per-head arithmetic does not depend on the others)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpu_util import dev_inputs
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    cfg = S.SsdConfig("hs", 1, 512, 16, 64, 8, 128, 128, "bf16", has_z=True, has_init=True, return_final=True)
    d = dev_inputs(S.make_ssd_inputs(cfg, 5), "bf16")

    def run(t):
        return mamba_chunk_scan_combined_fwd(t["x"], t["dt"], t["A"], t["B"], t["C"], 128, D=t["D"], z=t["z"],
                                             dt_bias=t["dt_bias"], initial_states=t["initial_states"],
                                             dt_softplus=True, return_final_states=True)

    out, fin = run(d)
    for r in range(world):
        h0, h1 = SH.head_range(16, 8, world, r)
        o, f = run(SH.shard_heads(d, world, r))
        assert torch.equal(o, out[:, :, h0:h1])
        assert torch.equal(f, fin[:, h0:h1])


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,N,Q,lens", [("bf16", 128, 128, None), ("bf16", 256, 128, [[700, 324], [100, 924]]),
                                            ("f32", 128, 64, [[1024], [333, 691]]), ("bf16", 128, 256, [[0, 1024], [512, 512]])],
                         ids=["one-seq", "n256-packed", "f32-q64", "new-seq-first"])
def test_sp_fixup_equals_forward_with_initial_state(dtype, N, Q, lens):
    """Zero-state forward + ssd_sp_state_fixup(S) equals the forward started from S, for
    out and final states; per batch row the carried sequence ends at a different token."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpu_util import TOL, dev_inputs, rel_l2, to_dev
    from mamba2_b200 import chunk_cumsum_fwd, mamba_chunk_scan_combined_fwd
    L, H, P, G = 1024, 8, 64, 2
    cfg = S.SsdConfig("fx", 2, L, H, P, G, N, Q, dtype, has_z=True, has_init=True, return_final=True)
    d = dev_inputs(S.make_ssd_inputs(cfg, 31), dtype)
    seq = None
    if lens is not None:
        seq = np.stack([np.repeat(np.arange(len(r)), r) for r in lens]).astype(np.int32)
        if lens[0][0] == 0:
            seq[0] += 1                       # row 0 holds no token of the carried sequence
        seq = to_dev(seq, int32=True)
    kw = dict(D=d["D"], z=d["z"], dt_bias=d["dt_bias"], dt_softplus=True, seq_idx=seq, return_final_states=True)
    ref_out, ref_fin = mamba_chunk_scan_combined_fwd(d["x"], d["dt"], d["A"], d["B"], d["C"], Q,
                                                     initial_states=d["initial_states"], **kw)
    out, fin = mamba_chunk_scan_combined_fwd(d["x"], d["dt"], d["A"], d["B"], d["C"], Q, **kw)
    dA, _ = chunk_cumsum_fwd(d["dt"], d["A"], Q, dt_bias=d["dt_bias"], dt_softplus=True)
    clen = None if seq is None else SH.carried_len(seq)
    SH.sp_state_fixup(out, d["C"], d["z"], dA, d["initial_states"], Q, carried=clen, final_states=fin)
    torch.cuda.synchronize()
    assert rel_l2(out, ref_out.double().cpu().numpy()) <= TOL[dtype]
    assert rel_l2(fin, ref_fin.double().cpu().numpy()) <= TOL[dtype]
    if seq is not None:                       # tokens after the carried sequence are untouched
        out0, _ = mamba_chunk_scan_combined_fwd(d["x"], d["dt"], d["A"], d["B"], d["C"], Q, **kw)
        for bi in range(2):
            c = int(clen[bi])
            assert torch.equal(out[bi, c:], out0[bi, c:])


def test_capi_sp_fixup_rejects_bad_args():
    import ctypes
    from mamba2_b200 import _lib
    lib = _lib.load()
    p = _lib.SpFixupParams(batch=1, seqlen=256, nheads=8, headdim=64, ngroups=2, dstate=128, chunk_size=128)
    assert lib.ssd_sp_state_fixup(ctypes.byref(p), None) == 1          # C, dA, state, out missing
    p.C, p.dA_cumsum, p.state_in, p.out = 256, 512, 1024, 2048
    p.headdim = 62
    assert lib.ssd_sp_state_fixup(ctypes.byref(p), None) == 2          # headdim % 4
    p.headdim, p.ngroups = 64, 3
    assert lib.ssd_sp_state_fixup(ctypes.byref(p), None) == 1          # H % G
    p.ngroups, p.dstate, p.headdim = 2, 1024, 128
    assert lib.ssd_sp_state_fixup(ctypes.byref(p), None) == 2          # shared memory budget
    assert "shared memory" in lib.ssd_last_error().decode()
    p.dstate, p.dtype = 128, 9
    assert lib.ssd_sp_state_fixup(ctypes.byref(p), None) == 1          # bad dtype enum
    assert lib.ssd_sp_state_fixup(None, None) == 1
