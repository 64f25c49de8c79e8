"""Benchmark: Mamba2 SSD layer forward tokens/s on B200 (one process per GPU).

python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

A "step" is one SSD layer forward over one synthetic batch of the config (default c2,
the nemotron-h-8b shape the north star targets: b=1, L=4096, H=128, P=64, G=8, N=128,
Q=128, bf16 inputs, initial states in, final states out).  At N GPUs every rank runs its
own batch (weak scaling, no data-path collective).  `value` is measured with inputs
resident in HBM (one CUDA graph per step, input sets rotated so consecutive steps share
no L2 lines); `e2e` goes through the public Python API with pinned host buffers and
host<->device copies inside the timed region (steps alternate between two streams, so one
step's result copy overlaps the next step's input copy).  `--impl reference` times the CPU
restatement of the reference algorithm (the reference itself needs JAX, absent here).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

_REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(_REPO, "mamba2-jax-pallas_b200"))
sys.path.insert(0, _REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from mamba2_b200 import _lib  # noqa: E402
from mamba2_b200 import synthetic as S  # noqa: E402

N_SETS = 4   # rotated input sets (each > L2 when combined with its output)


def _peaks():
    try:
        with open(os.path.join(_REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def measured_traffic(key):
    """DRAM bytes per launch from the committed ncu summary (profiles/traffic.json), or None."""
    try:
        with open(os.path.join(_REPO, "profiles", "traffic.json")) as f:
            return json.load(f)[key]["traffic_bytes"]
    except Exception:
        return None


def layer_work(cfg):
    """Algorithmic FLOPs and HBM bytes of one SSD layer forward (causal FLOPs; fp32 out)."""
    b, L, H, P, G, N, Q = (cfg.batch, cfg.seqlen, cfg.nheads, cfg.headdim, cfg.ngroups,
                           cfg.dstate, cfg.chunk_size)
    nc = cfg.nchunks
    tri = Q * (Q + 1) / 2
    flops = 2 * b * (nc * G * tri * N + L * H * P * N + nc * H * tri * P + L * H * N * P
                     + nc * H * P * N)
    isz = 2 if cfg.dtype == "bf16" else 4
    byts = b * L * (H * P + H + 2 * G * N) * isz + b * L * H * P * 4
    if cfg.has_z:
        byts += b * L * H * P * isz
    if cfg.has_init:
        byts += b * H * P * N * 4
    if cfg.return_final:
        byts += b * H * P * N * 4
    return flops, byts


class Clocks:
    """SM clock and throttle reasons sampled through NVML every ~2 ms on a background thread
    while the timed region runs (nvidia-smi's 100 ms floor misses short regions)."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, index):
        import threading
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = torch.cuda.get_device_properties(index).uuid
            h = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                hi = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(hi)
                u = u.decode() if isinstance(u, bytes) else u
                if str(uuid) in u:
                    h = hi
            h = h or pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self._nv, self._h = pynvml, h
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception:
            self._nv = None

    def _run(self):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.reasons.update(n for bit, n in self.REASONS.items() if mask & bit)
            except Exception:
                pass
            time.sleep(0.002)

    def stop(self):
        if self._nv is None:
            return None
        self._stop.set()
        self._t.join(1.0)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dev_inputs(inp, cfg, device):
    tdt = torch.bfloat16 if cfg.dtype == "bf16" else torch.float32
    d = {}
    for k in ("x", "dt", "B", "C", "z"):
        d[k] = None if inp[k] is None else torch.from_numpy(inp[k]).to(device=device, dtype=tdt)
    for k in ("A", "D", "dt_bias", "initial_states"):
        d[k] = None if inp[k] is None else torch.from_numpy(inp[k]).to(device)
    for k in ("seq_idx", "cu_seqlens"):
        d[k] = None if inp[k] is None else torch.from_numpy(inp[k]).to(device=device, dtype=torch.int32)
    return d


def fwd_kwargs(cfg, d):
    return dict(D=d["D"], z=d["z"], dt_bias=d["dt_bias"], initial_states=d["initial_states"],
                seq_idx=d["seq_idx"], cu_seqlens=d["cu_seqlens"], dt_softplus=True,
                return_final_states=cfg.return_final)


def time_region(fn, steps, stream, side=()):
    """Device time of `steps` calls of fn() between two events on `stream`.  Work that fn
    puts on the `side` streams starts after the first event and ends before the second."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for s in side:
        s.wait_event(e0)
    for i in range(steps):
        fn(i)
    for s in side:
        ev = torch.cuda.Event()
        ev.record(s)
        stream.wait_event(ev)
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1)


def time_kernel(fn, reps=20):
    """Average device time of one launch: a sleep kernel ahead of each start event keeps
    host launch overhead out of the event window."""
    s = torch.cuda.current_stream()
    for _ in range(3):
        fn()
    tot = 0.0
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(2_000_000)
        e0.record(s)
        fn()
        e1.record(s)
        e1.synchronize()
        tot += e0.elapsed_time(e1)
    return tot / reps


def kernel_breakdown(cfg, d, runner):
    """Per-kernel device times (ms), algorithmic bytes and FLOPs of one forward."""
    from mamba2_b200 import kernels as K
    b, L, H, P, G, N, Q = (cfg.batch, cfg.seqlen, cfg.nheads, cfg.headdim, cfg.ngroups,
                           cfg.dstate, cfg.chunk_size)
    nc = cfg.nchunks
    isz = 2 if cfg.dtype == "bf16" else 4
    res = []
    if runner.uses_tc:
        flops, byts = layer_work(cfg)
        ms = time_kernel(lambda: runner())
        res.append(("ssd_fused_tc", ms, byts, flops, "tensor" if flops / 1.6e15 > byts / 6.5e12 else "hbm"))
        return res
    dA, dto = K.chunk_cumsum_fwd(d["dt"], d["A"], Q, dt_bias=d["dt_bias"], dt_softplus=True)
    st = K.chunk_state_fwd(d["x"], d["B"], dto, dA, seq_idx=d["seq_idx"])
    cb = K.bmm_chunk_fwd(d["C"], d["B"], Q, seq_idx=d["seq_idx"])
    dAc = dA[..., -1].contiguous()
    csz = b * H * nc * Q * 4
    ssz = b * nc * H * P * N * 4
    res.append(("chunk_cumsum", time_kernel(lambda: K.chunk_cumsum_fwd(d["dt"], d["A"], Q, dt_bias=d["dt_bias"], dt_softplus=True)),
                b * L * H * isz + 2 * csz, 0, "hbm"))
    res.append(("chunk_state", time_kernel(lambda: K.chunk_state_fwd(d["x"], d["B"], dto, dA, seq_idx=d["seq_idx"])),
                b * L * (H * P + G * N) * isz + 2 * csz + ssz, 2 * b * L * H * P * N, "hbm"))
    res.append(("state_passing", time_kernel(lambda: K.state_passing_fwd(st.view(b, nc, H, P * N), dAc,
                                                                          seq_idx=d["seq_idx"], chunk_size=Q)),
                2 * ssz, 0, "hbm"))
    res.append(("bmm_chunk", time_kernel(lambda: K.bmm_chunk_fwd(d["C"], d["B"], Q, seq_idx=d["seq_idx"])),
                2 * b * L * G * N * isz + b * nc * G * Q * Q * 4, 2 * b * nc * G * Q * Q * N, "hbm"))
    res.append(("chunk_scan", time_kernel(lambda: K.chunk_scan_fwd(cb, d["x"], dto, dA, d["C"], st, D=d["D"], z=d["z"],
                                                                  seq_idx=d["seq_idx"])),
                b * nc * G * Q * Q * 4 + b * L * (H * P + G * N) * isz + 2 * csz + ssz + b * L * H * P * 4,
                2 * b * nc * H * (Q * (Q + 1) / 2 * P + Q * N * P), "hbm"))
    return res


def cpu_oracle_sample(cfg, budget_s=12.0, heads=None):
    """Time the CPU restatement (numpy float64, BLAS on all host threads) on a head slice of
    the workload; returns (tokens/s scaled to the full head count, description, threads)."""
    from oracle import ssd_ref as R
    threads = len(os.sched_getaffinity(0))
    hs = heads or max(cfg.ngroups, min(cfg.nheads, 16))
    hs -= hs % cfg.ngroups
    small = S.scaled(cfg, nheads=hs)
    inp = S.make_ssd_inputs(small, 99)
    reps, t_tot = 0, 0.0
    while reps == 0 or (t_tot < budget_s and reps < 50):
        t0 = time.perf_counter()
        R.ssd_combined(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], cfg.chunk_size,
                       D=inp["D"], z=inp["z"], dt_bias=inp["dt_bias"],
                       initial_states=inp["initial_states"], seq_idx=inp["seq_idx"],
                       dt_softplus=True, return_final_states=cfg.return_final)
        t_tot += time.perf_counter() - t0
        reps += 1
    t = t_tot / reps
    tok_s = cfg.tokens / (t * cfg.nheads / hs)
    desc = (f"oracle/ssd_ref.py (numpy float64 restatement of ops/ssd_naive.py) on {hs} of "
            f"{cfg.nheads} heads, {reps} reps x {t:.2f}s, scaled by heads")
    return tok_s, desc, threads


def run_reference(args, cfg, rank):
    """The reference arm: the reference's CPU algorithm (ssd_naive, restated in NumPy float64
    with BLAS on all host threads) on rank 0.  Each step runs the oracle on a bounded head
    slice of the configured layer at its full length; `ms_per_step` is that measured sample
    time, and `value` extrapolates it to the whole layer (heads are independent, so the
    cost is linear in the head count)."""
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_oracle_sample(cfg, budget_s=0.0)
    t_all, scale, desc, thr = 0.0, 1.0, "", 1
    for _ in range(args.steps):
        v, desc, thr = cpu_oracle_sample(cfg, budget_s=0.0)
        hs = cfg.tokens * 1.0 / v   # full-layer seconds
        t_all += hs
    hslice = max(cfg.ngroups, min(cfg.nheads, 16))
    hslice -= hslice % cfg.ngroups
    scale = cfg.nheads / hslice
    value = args.steps * cfg.tokens / t_all
    line = {"impl": "reference", "metric": "SSD layer fwd tokens/s", "value": value,
            "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t_all / args.steps / scale, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": cfg.name, "key": args.config, "batch": cfg.batch,
                       "seqlen": cfg.seqlen, "nheads": cfg.nheads, "headdim": cfg.headdim,
                       "ngroups": cfg.ngroups, "dstate": cfg.dstate, "chunk_size": cfg.chunk_size,
                       "input_dtype": cfg.dtype,
                       "sample": f"each step: {hslice} of {cfg.nheads} heads at full length; value scaled "
                                 f"by {scale:g} to the whole layer"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": thr, "kind": "port",
                             "sample": desc},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "JAX is not installable here, so the reference's ssd_naive algorithm is timed through "
                    "its float64 NumPy restatement (oracle/ssd_ref.py), which tests/test_golden.py pins to "
                    "the reference's own outputs"}
    print(json.dumps(line), flush=True)


def run_ours(args, cfg, rank, world, device):
    from mamba2_b200 import mamba_chunk_scan_combined_fwd
    from mamba2_b200.runner import SsdForward
    hbm, tfl, peak_kind = _peaks()
    replicas = world > 1 and args.replicas
    # default at N > 1: one layer, heads sharded over the ranks on group boundaries (strong
    # scaling); --replicas runs an independent full layer per rank instead
    inp = S.make_ssd_inputs(cfg, 1000 + 2 + (rank if replicas else 0))
    sets = [dev_inputs(inp, cfg, device) for _ in range(N_SETS)]
    head_share = 1.0
    if world > 1 and not replicas:
        from mamba2_b200 import sharding as SH
        h0, h1 = SH.head_range(cfg.nheads, cfg.ngroups, world, rank)
        head_share = (h1 - h0) / cfg.nheads
        sets = [SH.shard_heads(d, world, rank) for d in sets]
    flags = _lib.SSD_FLAG_BF16_MMA if args.bf16_mma else 0
    runners = [SsdForward(d["x"], d["dt"], d["A"], d["B"], d["C"], cfg.chunk_size, flags=flags, **fwd_kwargs(cfg, d))
               for d in sets]
    graphs = [r.graph() for r in runners]
    stream = torch.cuda.current_stream()
    for i in range(max(args.warmup, 3)):
        graphs[i % N_SETS].replay()
    clk = Clocks(device.index) if rank == 0 else None
    if world > 1:
        torch.distributed.barrier()
    ms = time_region(lambda i: graphs[i % N_SETS].replay(), args.steps, stream)
    if world > 1:
        torch.distributed.barrier()
    clocks = clk.stop() if clk else None
    t = torch.tensor([ms], device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    layers = world if replicas else 1
    value = args.steps * cfg.tokens * layers / (ms / 1e3)
    launches_per_step = runners[0].launches_per_step

    # end to end through the public API: pinned host inputs -> device -> forward -> host.
    # Consecutive steps alternate between two streams, each with its own workspace and
    # host result buffers, so one step's result copy (D2H) overlaps the next step's input
    # copy (H2D): the host link runs both directions at once, as a serving loop would.
    host = {k: (None if v is None else v.cpu().pin_memory()) for k, v in sets[0].items()}
    h2d = sum(v.numel() * v.element_size() for k, v in host.items() if v is not None)
    b, L, H, P, N = cfg.batch, cfg.seqlen, sets[0]["x"].shape[2], cfg.headdim, cfg.dstate
    n_lanes = 2
    lanes = []
    for _ in range(n_lanes):
        lanes.append({
            "stream": torch.cuda.Stream(device),
            "ws": torch.empty(runners[0].workspace.numel(), device=device, dtype=torch.uint8),
            "out": torch.empty((b, L, H, P), dtype=torch.float32).pin_memory(),
            "fin": torch.empty((b, H, P, N), dtype=torch.float32).pin_memory() if cfg.return_final else None})
    d2h = lanes[0]["out"].numel() * 4 + (lanes[0]["fin"].numel() * 4 if cfg.return_final else 0)

    def e2e_step(i):
        ln = lanes[i % n_lanes]
        with torch.cuda.stream(ln["stream"]):
            dd = {k: (None if v is None else v.to(device, non_blocking=True)) for k, v in host.items()}
            r = mamba_chunk_scan_combined_fwd(dd["x"], dd["dt"], dd["A"], dd["B"], dd["C"], cfg.chunk_size,
                                              workspace=ln["ws"], bf16_mma=args.bf16_mma, **fwd_kwargs(cfg, dd))
            if cfg.return_final:
                ln["out"].copy_(r[0], non_blocking=True)
                ln["fin"].copy_(r[1], non_blocking=True)
            else:
                ln["out"].copy_(r, non_blocking=True)
    for i in range(2 * n_lanes):
        e2e_step(i)
    if world > 1:
        torch.distributed.barrier()
    ms_e2e = time_region(e2e_step, args.steps, stream, side=[ln["stream"] for ln in lanes])
    t = torch.tensor([ms_e2e], device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    e2e_val = args.steps * cfg.tokens * layers / (float(t.item()) / 1e3)

    if rank != 0:
        return
    flops, byts = layer_work(cfg)
    flops, byts = flops * head_share, byts * head_share    # this GPU's share of the layer
    if runners[0].uses_tc:
        # the step's kernels (dt pre-pass, [segment-state pass, state combine,] fused walk)
        # timed on the device inside the CUDA-graph replays above: the fused kernel is
        # about 0.9 of it (profiles/launches_c2.md), so the step bounds the kernel
        kms = ms / args.steps
        name = "ssd_fused_tc_kernel + dt pre-pass (one graph-replayed step)"
        kbytes, kflops = byts, flops
        bound = "tensor" if flops / (tfl * 1e12) > byts / (hbm * 1e9) else "hbm"
        brk = [(name, kms, kbytes, kflops, bound)]
    else:
        brk = kernel_breakdown(cfg, sets[0], runners[0])
        name, kms, kbytes, kflops, bound = max(brk, key=lambda r: r[1])
    if bound == "tensor":
        ach, peak, unit = kflops / (kms / 1e3) / 1e12, tfl, "TFLOP/s"
    else:
        ach, peak, unit = kbytes / (kms / 1e3) / 1e9, hbm, "GB/s"
    t_roof = max(flops / (tfl * 1e12), byts / (hbm * 1e9))
    line = {"metric": "SSD layer fwd tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak" if (replicas or world == 1) else "strong",
            "vs_baseline": None, "dtype": "bf16" if (cfg.dtype == "bf16" or args.bf16_mma) else "f32",
            "data": "synthetic",
            "config": {"workload": cfg.name, "key": args.config, "batch": cfg.batch, "seqlen": cfg.seqlen,
                       "nheads": cfg.nheads, "headdim": cfg.headdim, "ngroups": cfg.ngroups,
                       "dstate": cfg.dstate, "chunk_size": cfg.chunk_size, "input_dtype": cfg.dtype,
                       "mma_operands": "bf16" if (cfg.dtype == "bf16" or args.bf16_mma) else
                       "split bf16 hi+lo, 3 products (tcgen05; CUDA-core cumsum and state passing)",
                       "parallelism": (f"replicas x{world}, no collective" if replicas else
                                       f"head-sharded x{world} on group boundaries, no collective"),
                       "heads_per_gpu": sets[0]["x"].shape[2],
                       "l2": f"{N_SETS} rotated input sets, each step's inputs+outputs > L2"},
            "roofline": {"kernel": name, "bound": bound, "achieved": ach, "peak": peak, "unit": unit,
                         "frac": ach / peak, "peak_kind": peak_kind,
                         "traffic": (measured_traffic(f"ssd_fused_tc/{args.config}")
                                     if (not args.override and world == 1) else None),
                         "algorithmic_bytes": kbytes, "kernel_ms": kms},
            "layer_roofline": {"t_roof_us": t_roof * 1e6, "t_step_us": 1e3 * ms / args.steps,
                               "frac": t_roof / (ms / args.steps / 1e3), "flops": flops, "bytes": byts},
            "kernels": {r[0]: round(r[1] * 1e3, 2) for r in brk},
            "e2e": {"value": e2e_val, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks}
    if world == 1 and not args.no_cpu_baseline:
        v, desc, thr = cpu_oracle_sample(cfg)
        line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": thr, "kind": "port",
                                "sample": desc}
    print(json.dumps(line), flush=True)


def run_sp(args, cfg, rank, world, device):
    """--sp: the sequence-parallel variant of a packed config (c3): rank r holds a
    chunk-aligned token segment of the packed row, runs it from a zero state, receives the
    state entering it by the recursive-doubling exchange over NCCL and adds it with the
    tensor-core fix-up (mamba2_b200.sharding.ssd_forward_sequence_parallel).  value = the
    row's tokens / the slowest rank's time per step.  Inputs are drawn on the device (seeded
    per rank) with the config's distributions; the packed lengths come from the config's
    seeded generator."""
    from mamba2_b200 import sharding as SH
    g = torch.Generator(device=device).manual_seed(5000 + rank)
    rng = np.random.default_rng(77)
    L, H, P, G, N, Q = cfg.seqlen, cfg.nheads, cfg.headdim, cfg.ngroups, cfg.dstate, cfg.chunk_size
    t0, t1 = SH.seq_segment(L, Q, world, rank)
    n = t1 - t0
    seq_full = np.zeros(L, np.int32)
    if cfg.varlen_seqs:
        lens = S.varlen_lengths(rng, cfg.varlen_seqs, L, *cfg.varlen_range)
        seq_full = np.repeat(np.arange(len(lens), dtype=np.int32), lens)
    rn = lambda *shape: torch.randn(shape, generator=g, device=device).to(torch.bfloat16)
    x, dt, B, C = rn(1, n, H, P), rn(1, n, H), rn(1, n, G, N), rn(1, n, G, N)
    dt0 = np.exp(rng.uniform(math.log(1e-3), math.log(0.1), size=H))
    dt_bias = torch.from_numpy((dt0 + np.log(-np.expm1(-dt0))).astype(np.float32)).to(device)
    A = torch.from_numpy((-np.exp(np.log(rng.uniform(1.0, 16.0, size=H)))).astype(np.float32)).to(device)
    D = torch.ones(H, device=device)
    seq = torch.from_numpy(seq_full[t0:t1][None].copy()).to(device)
    prev = torch.tensor([int(seq_full[t0 - 1]) if t0 > 0 else 0], dtype=torch.int32, device=device)

    from mamba2_b200.kernels.ssd_combined import _fwd_params
    pf, _keep = _fwd_params(x, dt, A, B, C, Q, D, None, dt_bias, None, seq, None, True, (0.0, math.inf), 0)
    fwd_launches = _lib.load().ssd_combined_num_launches(pf)

    def step(_i):
        return SH.ssd_forward_sequence_parallel(x, dt, A, B, C, Q, D=D, dt_bias=dt_bias, seq_idx=seq,
                                                prev_seq=prev, dt_softplus=True)
    for i in range(max(args.warmup, 3)):
        step(i)
    stream = torch.cuda.current_stream()
    clk = Clocks(device.index) if rank == 0 else None
    if world > 1:
        torch.distributed.barrier()
    ms = time_region(step, args.steps, stream)
    if world > 1:
        torch.distributed.barrier()
    clocks = clk.stop() if clk else None
    t = torch.tensor([ms], device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    if rank != 0:
        return
    line = {"metric": "SSD layer fwd tokens/s (sequence parallel)", "value": args.steps * L / (ms / 1e3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": cfg.name, "key": args.config, "seqlen": L, "nheads": H, "headdim": P,
                       "ngroups": G, "dstate": N, "chunk_size": Q, "packed_sequences": cfg.varlen_seqs,
                       "parallelism": f"sequence-parallel x{world}: zero-state segment forward, recursive-"
                                      f"doubling state exchange over NCCL, tensor-core fix-up"},
            # per step on a rank after the first: the forward, chunk_cumsum, the fix-up
            "gpu_launches": (fwd_launches + 2) * args.steps, "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_ssu(args, rank, world, device):
    """c4: selective_state_update decode steps, state updated in place (1000 steps timed as
    one region; tokens = batch x steps)."""
    from mamba2_b200 import _lib
    from mamba2_b200.ops.selective_state_update import selective_state_update
    cfg = S.CONFIGS["c4"]
    hbm, tfl, peak_kind = _peaks()
    u = S.make_ssu_inputs(cfg, 1004 + rank)
    tdt = torch.bfloat16
    st = torch.from_numpy(u["state"]).to(device)
    d = {k: torch.from_numpy(u[k]).to(device=device, dtype=(tdt if k in ("x", "z", "dt", "B", "C") else torch.float32))
         for k in ("x", "z", "dt", "B", "C", "A", "D", "dt_bias")}
    b, H, P, N, G = cfg.batch, cfg.nheads, cfg.headdim, cfg.dstate, cfg.ngroups
    out = torch.empty((b, H, P), device=device, dtype=torch.float32)
    p = _lib.SsuParams(batch=b, nheads=H, headdim=P, ngroups=G, dstate=N, dtype=1, dt_dtype=1, dt_ndim=2,
                       A_ndim=1, D_ndim=1, dt_bias_ndim=1, dt_softplus=1)
    p.state, p.x, p.dt, p.A = st.data_ptr(), d["x"].data_ptr(), d["dt"].data_ptr(), d["A"].data_ptr()
    p.B, p.C, p.D, p.z = d["B"].data_ptr(), d["C"].data_ptr(), d["D"].data_ptr(), d["z"].data_ptr()
    p.dt_bias, p.out = d["dt_bias"].data_ptr(), out.data_ptr()
    lib = _lib.load()
    stream = torch.cuda.current_stream()
    steps = args.steps if args.steps != 50 else cfg.steps
    g = torch.cuda.CUDAGraph()
    s2 = torch.cuda.Stream()
    s2.wait_stream(stream)
    with torch.cuda.stream(s2):
        _lib.check(lib.ssd_selective_state_update(p, s2.cuda_stream))
    stream.wait_stream(s2)
    with torch.cuda.graph(g):
        _lib.check(lib.ssd_selective_state_update(p, torch.cuda.current_stream().cuda_stream))
    for _ in range(max(args.warmup, 3)):
        g.replay()
    clk = Clocks(device.index) if rank == 0 else None
    if world > 1:
        torch.distributed.barrier()
    ms = time_region(lambda i: g.replay(), steps, stream)
    clocks = clk.stop() if clk else None
    t = torch.tensor([ms], device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    value = steps * b * world / (ms / 1e3)
    state_bytes = b * H * P * N * 4
    io = b * H * P * 2 * 2 + b * H * 2 + 2 * b * G * N * 2 + b * H * P * 4
    step_bytes = 2 * state_bytes + io
    # e2e: per step H2D of the token inputs, D2H of out; state stays resident (as in decode)
    host = {k: d[k].cpu().pin_memory() for k in ("x", "z", "dt", "B", "C")}
    out_h = torch.empty((b, H, P), dtype=torch.float32).pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in host.values())

    def e2e_step(_i):
        dd = {k: host[k].to(device, non_blocking=True) for k in host}
        _, o = selective_state_update(st, dd["x"], dd["dt"], d["A"], dd["B"], dd["C"], D=d["D"], z=dd["z"],
                                      dt_bias=d["dt_bias"], dt_softplus=True, inplace=True)
        out_h.copy_(o, non_blocking=True)
    for i in range(3):
        e2e_step(i)
    e2e_steps = min(steps, 200)
    ms_e2e = time_region(e2e_step, e2e_steps, stream)
    if rank != 0:
        return
    ach = step_bytes / (ms / steps / 1e3) / 1e9
    line = {"metric": "selective_state_update decode tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": ms / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": cfg.name, "key": "c4", "batch": b, "nheads": H, "headdim": P,
                       "ngroups": G, "dstate": N, "input_dtype": "bf16", "state": "f32 in place",
                       "l2": f"state {state_bytes / 1e9:.2f} GB > L2"},
            "roofline": {"kernel": "ssu_kernel", "bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                         "frac": ach / hbm, "peak_kind": peak_kind,
                         "traffic": measured_traffic("ssu_kernel/c4") if not args.override else None,
                         "algorithmic_bytes": step_bytes},
            "e2e": {"value": e2e_steps * b * world / (ms_e2e / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": out_h.numel() * 4},
            "gpu_launches": steps, "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_conv(args, rank, world, device):
    """conv: causal_conv1d of the c2 layer (nemotron-h-8b: dim = d_ssm + 2 G N = 10240,
    L = 4096, width 4, bf16 weights and bias, SiLU) on the layer's channels-last
    activations, 4 rotated input sets (each in + out 168 MB > L2)."""
    from mamba2_b200 import causal_conv1d
    hbm, _, peak_kind = _peaks()
    b, L, dim, k = 1, 4096, 128 * 64 + 2 * 8 * 128, 4
    for kv in args.override:
        key, v = kv.split("=", 1)
        if key in ("batch", "seqlen"):
            b, L = (int(v), L) if key == "batch" else (b, int(v))
    g = torch.Generator(device=device).manual_seed(2024 + rank)
    sets = [torch.randn((b, L, dim), generator=g, device=device).to(torch.bfloat16) for _ in range(4)]
    w = (0.5 * torch.randn((dim, k), generator=g, device=device)).to(torch.bfloat16)
    bias = torch.randn((dim,), generator=g, device=device).to(torch.bfloat16)

    def step(i):
        return causal_conv1d(sets[i % 4].transpose(1, 2), w, bias=bias, activation="silu")
    for i in range(max(args.warmup, 3)):
        step(i)
    stream = torch.cuda.current_stream()
    steps = args.steps
    clk = Clocks(device.index) if rank == 0 else None
    if world > 1:
        torch.distributed.barrier()
    ms = time_region(step, steps, stream)
    clocks = clk.stop() if clk else None
    t = torch.tensor([ms], device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    kernel_ms = time_kernel(lambda: step(1))
    byts = 2 * b * L * dim * 2
    # e2e: pinned host activations in, the conv output back, both copies timed
    host_in = sets[0].cpu().pin_memory()
    host_out = torch.empty((b, L, dim), dtype=torch.bfloat16).pin_memory()

    def e2e_step(_i):
        xd = host_in.to(device, non_blocking=True)
        o = causal_conv1d(xd.transpose(1, 2), w, bias=bias, activation="silu")
        host_out.copy_(o.transpose(1, 2), non_blocking=True)
    for i in range(3):
        e2e_step(i)
    ms_e2e = time_region(e2e_step, min(steps, 20), stream)
    if rank != 0:
        return
    ach = byts / (kernel_ms / 1e3) / 1e9
    line = {"metric": "causal_conv1d tokens/s", "value": steps * b * L * world / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": ms / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "nemotron-h-8b conv1d (F1)", "key": "conv", "batch": b, "seqlen": L,
                       "dim": dim, "width": k, "layout": "channels-last", "activation": "silu",
                       "l2": "4 rotated input sets, each input + output > L2"},
            "roofline": {"kernel": "conv1d_cl_kernel", "bound": "hbm", "achieved": ach, "peak": hbm,
                         "unit": "GB/s", "frac": ach / hbm, "peak_kind": peak_kind,
                         "traffic": measured_traffic("conv1d_cl_kernel/conv") if not args.override else None,
                         "algorithmic_bytes": byts, "kernel_ms": kernel_ms},
            "e2e": {"value": min(steps, 20) * b * L * world / (ms_e2e / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": host_in.numel() * 2, "d2h_bytes_per_step": host_out.numel() * 2},
            "gpu_launches": steps, "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_norm(args, rank, world, device):
    """norm: rms_norm_gated of the c2 layer (nemotron-h-8b: the SSD output y (1, 4096, 8192)
    f32, gate z bf16, weight f32, group = d_ssm / G = 1024, norm before gate), 4 rotated
    input sets (each y + z + out 335 MB > L2)."""
    from mamba2_b200 import rms_norm_gated
    hbm, _, peak_kind = _peaks()
    b, L, d, G = 1, 4096, 128 * 64, 8
    for kv in args.override:
        key, v = kv.split("=", 1)
        if key in ("batch", "seqlen"):
            b, L = (int(v), L) if key == "batch" else (b, int(v))
    g = torch.Generator(device=device).manual_seed(4048 + rank)
    ys = [torch.randn((b, L, d), generator=g, device=device) for _ in range(4)]
    zs = [torch.randn((b, L, d), generator=g, device=device).to(torch.bfloat16) for _ in range(4)]
    w = 1.0 + 0.1 * torch.randn((d,), generator=g, device=device)

    def step(i):
        return rms_norm_gated(ys[i % 4], w, z=zs[i % 4], group_size=d // G)
    for i in range(max(args.warmup, 3)):
        step(i)
    stream = torch.cuda.current_stream()
    steps = args.steps
    clk = Clocks(device.index) if rank == 0 else None
    if world > 1:
        torch.distributed.barrier()
    ms = time_region(step, steps, stream)
    clocks = clk.stop() if clk else None
    t = torch.tensor([ms], device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    kernel_ms = time_kernel(lambda: step(1))
    byts = b * L * d * (4 + 2 + 4) + d * 4
    host_y, host_z = ys[0].cpu().pin_memory(), zs[0].cpu().pin_memory()
    host_out = torch.empty((b, L, d)).pin_memory()

    def e2e_step(_i):
        o = rms_norm_gated(host_y.to(device, non_blocking=True), w,
                           z=host_z.to(device, non_blocking=True), group_size=d // G)
        host_out.copy_(o, non_blocking=True)
    for i in range(3):
        e2e_step(i)
    ms_e2e = time_region(e2e_step, min(steps, 20), stream)
    if rank != 0:
        return
    ach = byts / (kernel_ms / 1e3) / 1e9
    line = {"metric": "rms_norm_gated tokens/s", "value": steps * b * L * world / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": ms / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "nemotron-h-8b gated RMSNorm (F2)", "key": "norm", "batch": b, "seqlen": L,
                       "hidden": d, "group_size": d // G, "y": "f32", "z": "bf16", "norm_before_gate": True,
                       "l2": "4 rotated input sets, each y + z + out > L2"},
            "roofline": {"kernel": "rmsnorm_cached_kernel", "bound": "hbm", "achieved": ach, "peak": hbm,
                         "unit": "GB/s", "frac": ach / hbm, "peak_kind": peak_kind,
                         "traffic": measured_traffic("rmsnorm_cached_kernel/norm") if not args.override else None,
                         "algorithmic_bytes": byts, "kernel_ms": kernel_ms},
            "e2e": {"value": min(steps, 20) * b * L * world / (ms_e2e / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": host_y.numel() * 4 + host_z.numel() * 2,
                    "d2h_bytes_per_step": host_out.numel() * 4},
            "gpu_launches": steps, "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_tail(args, rank, world, device):
    """tail: the c2 layer's SSD forward plus its gated RMSNorm (norm_before_gate=False, group =
    d_ssm / G, modules/mamba2.py:395-406), ending in the bf16 tensor the layer's out_proj takes:
    SSD (2 launches), then rms_norm_gated writing bf16 from its own pass (1 launch).  Also
    timed in the same run: the same with the norm writing f32 and a separate cast to bf16.
    4 rotated input sets."""
    import dataclasses
    from mamba2_b200 import mamba_chunk_scan_combined_fwd, rms_norm_gated
    cfg = dataclasses.replace(S.CONFIGS["c2"], has_z=True, has_init=False, return_final=False)
    sets = []
    for i in range(4):
        inp = S.make_ssd_inputs(cfg, 100 + i + 10 * rank)
        sets.append({k: (None if v is None else torch.from_numpy(np.ascontiguousarray(v)).to(
            torch.bfloat16 if k in ("x", "dt", "B", "C", "z") else torch.float32).to(device))
            for k, v in inp.items() if k in ("x", "dt", "A", "B", "C", "D", "z", "dt_bias")})
    b, L, H, P = sets[0]["x"].shape
    d, gs = H * P, H // cfg.ngroups * P
    w = (1.0 + 0.1 * torch.randn(d, generator=torch.Generator().manual_seed(5))).to(device)

    def ssd(t):
        return mamba_chunk_scan_combined_fwd(t["x"], t["dt"], t["A"], t["B"], t["C"], cfg.chunk_size, D=t["D"],
                                             dt_bias=t["dt_bias"], dt_softplus=True).view(b, L, d)

    def one_pass(i):
        t = sets[i % 4]
        return rms_norm_gated(ssd(t), w, z=t["z"].view(b, L, d), group_size=gs, norm_before_gate=False,
                              out_dtype=torch.bfloat16)

    def with_cast(i):
        t = sets[i % 4]
        o = rms_norm_gated(ssd(t), w, z=t["z"].view(b, L, d), group_size=gs, norm_before_gate=False)
        return o.to(torch.bfloat16)
    for i in range(max(args.warmup, 3)):
        one_pass(i)
        with_cast(i)
    stream = torch.cuda.current_stream()
    steps = args.steps
    clk = Clocks(device.index) if rank == 0 else None
    if world > 1:
        torch.distributed.barrier()
    ms = time_region(one_pass, steps, stream)
    clocks = clk.stop() if clk else None
    ms2 = time_region(with_cast, steps, stream)
    t = torch.tensor([ms, ms2], device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, ms2 = (float(v) for v in t.tolist())
    if rank != 0:
        return
    line = {"metric": "SSD + gated RMSNorm tokens/s", "value": steps * b * L * world / (ms / 1e3),
            "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": ms / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "nemotron-h-8b SSD layer + gated RMSNorm, bf16 result", "key": "tail",
                       "batch": b, "seqlen": L, "nheads": H, "group_size": gs, "norm_before_gate": False,
                       "l2": "4 rotated input sets, each step's inputs+outputs > L2"},
            "with_cast_ms_per_step": ms2 / steps,
            "gpu_launches": 3 * steps, "clocks": clocks}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2", choices=["c0", "c1", "c2", "c3", "c4", "conv", "norm", "tail"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--bf16-mma", action="store_true",
                    help="fp32 configs: bf16 MMA operands on the tensor-core path (the reference's Pallas "
                         "behaviour for fp32 inputs) instead of exact fp32")
    ap.add_argument("--sp", action="store_true",
                    help="sequence-parallel variant of the config (c3): token segments over the ranks")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: one independent full layer per rank (weak scaling) instead of one layer "
                         "head-sharded over the ranks")
    ap.add_argument("--override", action="append", default=[],
                    help="key=value on the config (e.g. batch=32) for small profiling cases")
    args = ap.parse_args()
    cfg = S.CONFIGS.get(args.config)
    if args.override and cfg is not None:
        import dataclasses
        kv = dict(o.split("=", 1) for o in args.override)
        cfg = dataclasses.replace(cfg, **{k: type(getattr(cfg, k))(v) for k, v in kv.items()})
        S.CONFIGS[args.config] = cfg
    if args.impl == "reference" and args.config in ("c4", "conv", "norm", "tail"):
        raise SystemExit(f"reference arm for {args.config} not implemented")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, cfg, rank)
        return
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1 or args.sp:
        if world == 1:   # the sequence-parallel path runs its exchange even on one rank
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", "29533")
            os.environ.setdefault("RANK", "0")
            os.environ.setdefault("WORLD_SIZE", "1")
        torch.distributed.init_process_group("nccl", device_id=device)
    try:
        if args.config == "c4":
            run_ssu(args, rank, world, device)
        elif args.config == "conv":
            run_conv(args, rank, world, device)
        elif args.config == "norm":
            run_norm(args, rank, world, device)
        elif args.config == "tail":
            run_tail(args, rank, world, device)
        elif args.sp:
            run_sp(args, cfg, rank, world, device)
        else:
            run_ours(args, cfg, rank, world, device)
    finally:
        if world > 1 or args.sp:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
