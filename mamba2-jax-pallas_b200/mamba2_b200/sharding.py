"""Multi-GPU partitioning of the SSD forward (one process per GPU).

Head sharding (no collective).  Heads are independent given their group's B and C, so the
heads are split into contiguous blocks aligned to group boundaries.  Each rank runs the
unchanged single-GPU forward on its block; outputs stay head-sharded and are bitwise equal
to the same heads of a single-GPU run.  With fewer groups than ranks (ngroups = 1 models),
B and C are replicated.

Sequence parallel (optional, long sequences).  Rank r holds tokens [L_r, L_{r+1}) of every
sequence.  The state entering segment r is the combination of the segments before it:
for a segment with total decay a (exp of its summed dt*A, or 0 when a sequence boundary
inside it cuts the carried state) and state s computed from a zero initial state, the
combine (a1, s1) o (a2, s2) = (a1 a2, a2 s1 + s2) is associative, so each rank needs the
exclusive prefix of the pairs of the ranks before it.  That prefix is exchanged by
recursive doubling with point-to-point sends (log2(world) rounds of (b,H) + (b,H,P,N)
fp32 per rank).  The received state's contribution is then added by one fix-up launch
(exp(dA) C S^T on the carried sequence's tokens, exp(total dA) S on the final state)
instead of a second forward.  The exchange is the only collective of the path.
"""
from __future__ import annotations

import math

import torch


# ---------------------------------------------------------------------------
# head sharding
# ---------------------------------------------------------------------------
def head_range(nheads: int, ngroups: int, world: int, rank: int) -> tuple[int, int]:
    """Heads [h0, h1) of `rank`: contiguous, group-aligned blocks of equal size.

    Needs ngroups % world == 0 (each rank owns whole groups) or world % ngroups == 0 with
    the heads of a group divisible among the ranks sharing it.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if nheads % ngroups:
        raise ValueError(f"nheads {nheads} is not a multiple of ngroups {ngroups}")
    hpg = nheads // ngroups
    if ngroups % world == 0:
        per = ngroups // world * hpg
    elif world % ngroups == 0 and hpg % (world // ngroups) == 0:
        per = hpg // (world // ngroups)
    else:
        raise ValueError(f"cannot split {nheads} heads in {ngroups} groups over {world} ranks")
    return rank * per, (rank + 1) * per


def group_range(nheads: int, ngroups: int, world: int, rank: int) -> tuple[int, int]:
    """Groups [g0, g1) whose B and C rows the heads of `rank` read."""
    h0, h1 = head_range(nheads, ngroups, world, rank)
    hpg = nheads // ngroups
    return h0 // hpg, (h1 - 1) // hpg + 1


def shard_heads(inputs: dict, world: int, rank: int) -> dict:
    """Slice SSD inputs to the heads of `rank` (keys as in the forward's arguments).

    x, z (b,L,H,P); dt (b,L,H); A, dt_bias (H,); D (H,) or (H,P); initial_states
    (b,H,P,N) are cut along H; B, C (b,L,G,N) along G.  Other entries pass through.
    """
    H = inputs["x"].shape[2]
    G = inputs["B"].shape[2]
    h0, h1 = head_range(H, G, world, rank)
    g0, g1 = group_range(H, G, world, rank)
    out = dict(inputs)
    for k in ("x", "z"):
        if inputs.get(k) is not None:
            out[k] = inputs[k][:, :, h0:h1].contiguous()
    if inputs.get("dt") is not None:
        out["dt"] = inputs["dt"][:, :, h0:h1].contiguous()
    for k in ("A", "dt_bias", "D"):
        if inputs.get(k) is not None:
            out[k] = inputs[k][h0:h1].contiguous()
    if inputs.get("initial_states") is not None:
        out["initial_states"] = inputs["initial_states"][:, h0:h1].contiguous()
    for k in ("B", "C"):
        out[k] = inputs[k][:, :, g0:g1].contiguous()
    return out


# ---------------------------------------------------------------------------
# sequence parallel
# ---------------------------------------------------------------------------
def seq_segment(seqlen: int, chunk_size: int, world: int, rank: int) -> tuple[int, int]:
    """Tokens [t0, t1) of `rank`: chunk-aligned, as equal as the chunks allow."""
    nc = -(-seqlen // chunk_size)
    c0 = rank * nc // world
    c1 = (rank + 1) * nc // world
    return min(c0 * chunk_size, seqlen), min(c1 * chunk_size, seqlen)


def combine(a1, s1, a2, s2):
    """(a1, s1) o (a2, s2): the segment pair followed by the second one.
    a: (b,H) decay, s: (b,H,P,N) state."""
    return a1 * a2, a2[..., None, None] * s1 + s2


def exclusive_prefix(decay: torch.Tensor, state: torch.Tensor, group=None, timeout=None):
    """Exclusive scan of (decay, state) pairs over the ranks of `group` in rank order.

    Recursive doubling: in round k every rank sends its inclusive partial to rank+2^k and
    receives from rank-2^k.  Returns the combination of all lower ranks' pairs (decay 1 and
    state 0 on rank 0).  Works on the gloo (CPU tensors) and NCCL (CUDA tensors) backends.
    ``timeout`` (a ``datetime.timedelta``) bounds each round's wait: a peer that died or
    stalls makes this rank raise instead of waiting for the process group's own timeout.
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if decay.is_cuda and dist.get_backend(group) == "gloo":
        # gloo moves host tensors only: stage through host memory (tests of the path on one GPU)
        a, s = exclusive_prefix(decay.cpu(), state.cpu(), group, timeout)
        return a.to(decay.device), s.to(state.device)
    inc_a, inc_s = decay.clone(), state.clone()          # inclusive partial of this rank
    exc_a, exc_s = torch.ones_like(decay), torch.zeros_like(state)
    k = 1
    while k < world:
        ra, rs = torch.empty_like(inc_a), torch.empty_like(inc_s)
        ops = []
        if rank + k < world:
            ops += [dist.P2POp(dist.isend, inc_a, _peer(rank + k, group), group),
                    dist.P2POp(dist.isend, inc_s, _peer(rank + k, group), group)]
        if rank - k >= 0:
            ops += [dist.P2POp(dist.irecv, ra, _peer(rank - k, group), group),
                    dist.P2POp(dist.irecv, rs, _peer(rank - k, group), group)]
        if ops:
            for req in dist.batch_isend_irecv(ops):
                if timeout is None:
                    req.wait()
                elif not req.wait(timeout):
                    raise RuntimeError(f"exclusive_prefix: round {k} did not complete within {timeout}")
        if rank - k >= 0:
            # the received partial covers ranks just below this one's current span
            exc_a, exc_s = combine(ra, rs, exc_a, exc_s)
            inc_a, inc_s = combine(ra, rs, inc_a, inc_s)
        k *= 2
    return exc_a, exc_s


def _peer(r, group):
    import torch.distributed as dist
    return r if group is None else dist.get_global_rank(group, r)


def segment_decay(dt, A, chunk_size, dt_bias=None, dt_softplus=False, dt_limit=(0.0, math.inf),
                  seq_idx=None, carried_seq=None, dA_cumsum=None):
    """Total decay (b,H) of a token segment: exp(sum_t dt'_t A), or 0 for batch rows whose
    last token belongs to another sequence than the carried one (seq_idx given)."""
    from .kernels import chunk_cumsum_fwd
    dA = dA_cumsum
    if dA is None:
        dA, _ = chunk_cumsum_fwd(dt, A, chunk_size, dt_bias=dt_bias, dt_softplus=dt_softplus, dt_limit=dt_limit)
    a = torch.exp(dA[..., -1].sum(-1))
    if seq_idx is not None and carried_seq is not None:
        a = a * (seq_idx[:, -1] == carried_seq).to(a.dtype)[:, None]
    return a


def relabel_seq_idx(seq_idx: torch.Tensor, carried: torch.Tensor) -> torch.Tensor:
    """Ids of a segment relabelled so that the carried sequence (id `carried` per batch
    row) becomes 0, which is the id the forward applies its initial state to; other ids
    stay distinct and non-negative (|ids| < 2^30)."""
    d = seq_idx - carried[:, None]
    return torch.where(d >= 0, d, d + (1 << 30)).to(torch.int32)


def ssd_forward_sequence_parallel(x, dt, A, B, C, chunk_size, D=None, z=None, dt_bias=None,
                                  initial_states=None, seq_idx=None, prev_seq=None, dt_softplus=False,
                                  dt_limit=(0.0, math.inf), group=None):
    """Sequence-parallel SSD forward of this rank's token segment.

    Inputs are this rank's tokens (the segments of all ranks, in rank order, make the
    sequence).  `initial_states` is the sequence's initial state and is used on rank 0
    only.  With seq_idx, `prev_seq` (b,) is the id of the token before this segment (any
    value on rank 0).  Returns (out, final_states): out is this segment's output, final
    the state after this segment (the sequence's final state on the last rank).
    """
    import torch.distributed as dist
    from .kernels import mamba_chunk_scan_combined_fwd
    rank = dist.get_rank(group)
    b, L, H, P = x.shape
    N = B.shape[3]
    kw = dict(D=D, z=z, dt_bias=dt_bias, dt_softplus=dt_softplus, dt_limit=dt_limit)
    sq = seq_idx
    carried = None
    if seq_idx is not None:
        carried = (torch.zeros(b, dtype=torch.int32, device=x.device) if rank == 0 else prev_seq.to(torch.int32))
        sq = seq_idx.to(torch.int32) if rank == 0 else relabel_seq_idx(seq_idx, carried)
    # pass 1: this segment from a zero state, and its decay
    from .kernels import chunk_cumsum_fwd
    init0 = initial_states if rank == 0 else None
    out0, s_loc = mamba_chunk_scan_combined_fwd(x, dt, A, B, C, chunk_size, initial_states=init0, seq_idx=sq,
                                                return_final_states=True, **kw)
    dA, _ = chunk_cumsum_fwd(dt, A, chunk_size, dt_bias=dt_bias, dt_softplus=dt_softplus, dt_limit=dt_limit)
    a_loc = segment_decay(dt, A, chunk_size, seq_idx=sq,
                          carried_seq=None if sq is None else torch.zeros_like(carried), dA_cumsum=dA)
    if rank == 0:
        a_loc = torch.zeros_like(a_loc)   # rank 0's pair already holds the initial state
    # exchange: the state entering this segment
    _, s_in = exclusive_prefix(a_loc.float().contiguous(), s_loc.float().contiguous(), group)
    if rank == 0:
        return out0, s_loc   # pass 1 already started from the sequence's initial state
    # fix-up: add the received state's contribution to the carried sequence's tokens (and
    # to the final state when that sequence reaches the segment's end), in place
    clen = None if sq is None else carried_len(sq)
    sp_state_fixup(out0, C, z, dA, s_in, chunk_size, carried=clen, final_states=s_loc)
    return out0, s_loc


def carried_len(seq_idx: torch.Tensor) -> torch.Tensor:
    """(b,) int32: per batch row, the number of leading tokens of the carried sequence (id 0
    after relabel_seq_idx), i.e. the first position with another id, or the segment length."""
    b, L = seq_idx.shape
    other = seq_idx != 0
    first = torch.where(other.any(1), other.int().argmax(1), torch.full((b,), L, device=seq_idx.device))
    return first.to(torch.int32).contiguous()


def sp_state_fixup(out, C, z, dA_cumsum, state_in, chunk_size, carried=None, final_states=None):
    """In place: out[b,t,h] += exp(dA(t)) C[b,t,g] . state_in[b,h]^T (times silu(z)) for the
    carried tokens, and final_states += exp(dA(L-1)) state_in where the carried sequence
    reaches the segment's end.  One launch of ``ssd_sp_state_fixup``."""
    from . import _lib
    b, L, H, P = out.shape
    G, N = C.shape[2], C.shape[3]
    if out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be a contiguous float32 tensor")
    if final_states is not None and (final_states.dtype != torch.float32 or not final_states.is_contiguous()):
        raise ValueError("final_states must be a contiguous float32 tensor")
    Cc = _lib.dev(C, "C")
    zc = _lib.dev(z, "z", Cc.dtype)
    dAc = _lib.dev(dA_cumsum, "dA_cumsum", torch.float32)
    sc = _lib.dev(state_in, "state_in", torch.float32)
    cl = _lib.dev(carried, "carried", torch.int32)
    p = _lib.SpFixupParams(batch=b, seqlen=L, nheads=H, headdim=P, ngroups=G, dstate=N, chunk_size=chunk_size,
                           dtype=_lib.dtype_code(Cc))
    p.C, p.z, p.dA_cumsum, p.state_in = Cc.data_ptr(), _lib.ptr(zc), dAc.data_ptr(), sc.data_ptr()
    p.carried_len, p.out, p.final_states = _lib.ptr(cl), out.data_ptr(), _lib.ptr(final_states)
    _lib.check(_lib.load().ssd_sp_state_fixup(p, _lib.stream_of(out)))
