"""Module-level worker functions for the multi-process tests (spawned processes
import them by name).  CPU workers use the oracle as the per-rank compute; the
GPU workers use the CUDA kernels."""

import os
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from gdn_kernel_b200 import sharding as S, workloads as W  # noqa: E402

PREFILL_LENGTHS = [37, 0, 129, 1, 200, 64, 90]
DECODE_BATCH = 5


def oracle_prefill_dps(q, k, v, state, A_log, a, dt_bias, b, cu, scale, out, ns):
    from oracle import gdn_oracle as O
    o, s = O.prefill_chunked(q, k, v, state, A_log, a, dt_bias, b, cu, scale)
    out.copy_(o)
    ns.copy_(s)


def oracle_decode_dps(q, k, v, state, A_log, a, dt_bias, b, scale, out, ns):
    from oracle import gdn_oracle as O
    o, s = O.decode_step(q, k, v, state, A_log, a, dt_bias, b, scale)
    out.copy_(o)
    ns.copy_(s)


def _gather(obj, world):
    objs = [None] * world
    dist.all_gather_object(objs, obj)
    return objs


def sharded_prefill_worker(rank, world, device=None, compute=None):
    """Each rank runs its LPT shard; rank 0 reassembles and returns the result."""
    x = W.make_prefill_inputs(PREFILL_LENGTHS, seed=77, h_qk=2, h_v=4)
    shard, out, ns = S.run_prefill_shard(rank, world, x.q, x.k, x.v, x.state, x.A_log, x.a,
                                         x.dt_bias, x.b, x.cu_seqlens, x.scale,
                                         compute or oracle_prefill_dps, device=device)
    parts = _gather((shard, out.cpu(), ns.cpu()), world)
    if rank != 0:
        return None
    shards, outs, states = zip(*parts)
    return S.scatter_prefill_outputs(shards, outs, states, sum(PREFILL_LENGTHS),
                                     len(PREFILL_LENGTHS))


def sharded_decode_worker(rank, world, device=None, compute=None, steps=3):
    first, tokens = W.make_decode_run(DECODE_BATCH, steps, seed=12, h_qk=2, h_v=4)
    lo, hi = S.decode_shards(DECODE_BATCH, world)[rank]
    dev = device or "cpu"
    mv = lambda t: t[lo:hi].contiguous().to(dev)
    dec = S.ShardedDecoder(rank, world, DECODE_BATCH, mv(first.state),
                           compute or oracle_decode_dps)
    outs = []
    for (q, k, v, a, b) in tokens:
        o = dec.step(mv(q), mv(k), mv(v), first.A_log.to(dev), mv(a), first.dt_bias.to(dev),
                     mv(b), first.scale)
        outs.append(o.cpu())
    parts = _gather((lo, hi, torch.stack(outs), dec.state.cpu()), world)
    if rank != 0:
        return None
    parts.sort(key=lambda p: p[0])
    return torch.cat([p[2] for p in parts], dim=1), torch.cat([p[3] for p in parts], dim=0)


def gpu_prefill_worker(rank, world):
    from gdn_kernel_b200 import kernel as K
    torch.cuda.set_device(rank)
    return sharded_prefill_worker(rank, world, device=f"cuda:{rank}", compute=K.gdn_prefill)


def gpu_decode_worker(rank, world):
    from gdn_kernel_b200 import kernel as K
    torch.cuda.set_device(rank)
    return sharded_decode_worker(rank, world, device=f"cuda:{rank}", compute=K.gdn_decode)


def failing_worker(rank, world):
    """Rank 1 raises before any collective; rank 0 finishes its own shard."""
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    return "rank0 done"


def failing_before_barrier_worker(rank, world):
    """Rank 1 raises; rank 0 then waits at a barrier, which must time out."""
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    dist.barrier()
    return "unreachable"


def silent_worker(rank, world):
    """Rank 1 never reports (sleeps past the launcher's limit)."""
    if rank == 1:
        time.sleep(600)
    return rank


# ----------------------------------------------------------------------------- context parallel
CP_TOKENS = 333          # 6 chunks: 64 x 5 + 13 (ragged tail on the last rank)


def _cp_inputs():
    return W.make_prefill_inputs([CP_TOKENS], seed=91, h_qk=1, h_v=2)


def cp_worker(rank, world, device=None, kernels=False):
    """One context-parallel prefill of a single sequence split over the ranks
    (the oracle as compute on CPU; the CUDA kernels with ``kernels``); rank 0
    returns the reassembled outputs and the last rank's end state."""
    from gdn_kernel_b200 import context_parallel as CP
    x = _cp_inputs()
    lo, hi = CP.cp_segments(CP_TOKENS, world)[rank]
    dev = device or "cpu"
    seg = lambda t: t[lo:hi].contiguous().to(dev)
    state = x.state[0].to(dev)
    extra = {} if kernels else dict(
        prefill_fn=oracle_prefill_dps,
        affine_fn=lambda s, m, n: n if s is None else s @ m + n)
    out, end = CP.cp_prefill(rank, world, seg(x.q), seg(x.k), seg(x.v), state, x.A_log.to(dev),
                             seg(x.a), x.dt_bias.to(dev), seg(x.b), x.scale, **extra)
    parts = _gather((rank, out.cpu(), end.cpu()), world)
    if rank != 0:
        return None
    parts.sort(key=lambda p: p[0])
    return torch.cat([p[1] for p in parts], dim=0), parts[-1][2]


def gpu_cp_worker(rank, world):
    torch.cuda.set_device(rank)
    return cp_worker(rank, world, device=f"cuda:{rank}", kernels=True)
