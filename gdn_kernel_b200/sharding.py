"""Sequence-sharded multi-GPU driver for the GDN hot path.

Heads and sequences of Gated DeltaNet are independent: a decode step or a
prefill of one sequence touches only that sequence's state.  The driver
therefore partitions *sequences* (and their resident fp32 states) across the
GPUs of one node, one process per GPU, and runs the single-GPU kernels on each
shard.  No collective sits on the data path; ``torch.distributed`` is used only
for host-side coordination (barriers, timing max-reduction, and the gathers
that tests use to verify results).

* decode: contiguous batch blocks ``[start, end)`` of near-equal size;
* prefill: longest-processing-time greedy assignment of sequences to ranks by
  chunk count (the sequential work of a sequence is its number of 64-token
  chunks), each rank packing its own tokens with a local ``cu_seqlens``.

The reference is single-GPU (its harness requests one B200, ref
scripts/run_modal.py:36); this module is the one parallel strategy this build
adds.
"""

from __future__ import annotations

import dataclasses
import heapq
import io
import math
import multiprocessing as mp
import os
import queue as queue_mod
import traceback
from typing import Callable, List, Optional, Sequence, Tuple

import torch

CHUNK = 64


# ----------------------------------------------------------------------------- partitioning
def decode_shards(batch: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous [start, end) batch blocks; sizes differ by at most one."""
    if world <= 0:
        raise ValueError("world must be positive")
    base, extra = divmod(batch, world)
    out, s = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((s, s + n))
        s += n
    return out


def prefill_shards(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Assign sequence indices to ranks, longest first, each to the rank with the
    least total chunks so far (ties: lowest rank).  Each rank's list is in that
    same order, longest first (ties: lower index): packed that way, the chain
    kernel's first wave of CTAs takes the longest sequences, so the short ones
    fill in behind them.  On B200, for 64 sequences of 1,024-16,384 tokens over 8
    ranks, that cut the slowest rank from 1.69 to 1.50 ms (index order gave ranks
    1.50-1.69 ms).  The outputs go back by token and sequence index
    (scatter_prefill_outputs)."""
    if world <= 0:
        raise ValueError("world must be positive")
    cost = [max(1, math.ceil(int(L) / CHUNK)) if int(L) > 0 else 0 for L in lengths]
    order = sorted(range(len(lengths)), key=lambda i: (-cost[i], i))
    heap = [(0, r) for r in range(world)]
    assign = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        assign[r].append(i)
        heapq.heappush(heap, (load + cost[i], r))
    return assign


@dataclasses.dataclass
class PrefillShard:
    """One rank's packed slice of a varlen prefill batch."""
    seq_ids: List[int]            # global sequence indices, in packing order
    token_index: torch.Tensor     # [T_local] global token index of each local token (int64)
    cu_seqlens: torch.Tensor      # [N_local + 1] local offsets
    lengths: List[int]


def make_prefill_shard(cu_seqlens: torch.Tensor, seq_ids: Sequence[int],
                       cu_dtype=torch.int32) -> PrefillShard:
    cu = [int(x) for x in cu_seqlens.cpu().tolist()]
    idx, lens = [], []
    for i in seq_ids:
        idx.append(torch.arange(cu[i], cu[i + 1], dtype=torch.int64))
        lens.append(cu[i + 1] - cu[i])
    token_index = torch.cat(idx) if idx else torch.zeros(0, dtype=torch.int64)
    local_cu = torch.zeros(len(lens) + 1, dtype=torch.int64)
    if lens:
        local_cu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int64), 0)
    return PrefillShard(list(seq_ids), token_index, local_cu.to(cu_dtype), lens)


def gather_prefill_inputs(shard: PrefillShard, q, k, v, state, a, b):
    """Slice the global packed tensors down to one shard (host or device)."""
    ti = shard.token_index.to(q.device)
    sel = lambda t: t.index_select(0, ti).contiguous()
    st = None
    if state is not None:
        st = state.index_select(0, torch.tensor(shard.seq_ids, dtype=torch.int64,
                                                device=state.device)).contiguous()
    return sel(q), sel(k), sel(v), st, sel(a), sel(b)


def scatter_prefill_outputs(shards: Sequence[PrefillShard], outs, states, total_tokens,
                            num_seqs):
    """Reassemble per-rank (output, new_state) into global packed tensors (host)."""
    o0, s0 = outs[0], states[0]
    out = torch.zeros((total_tokens,) + tuple(o0.shape[1:]), dtype=o0.dtype)
    new_state = torch.zeros((num_seqs,) + tuple(s0.shape[1:]), dtype=s0.dtype)
    for sh, o, s in zip(shards, outs, states):
        if len(sh.token_index):
            out[sh.token_index] = o.cpu()
        if sh.seq_ids:
            new_state[torch.tensor(sh.seq_ids)] = s.cpu()
    return out, new_state


# ----------------------------------------------------------------------------- per-rank drivers
class ShardedDecoder:
    """Decode state shard resident on this rank's GPU; ``step`` runs one T=1
    step of the local sequences in place.  ``compute`` is the decode entry
    point (``gdn_kernel_b200.kernel.gdn_decode`` on a GPU)."""

    def __init__(self, rank: int, world: int, batch: int, state: torch.Tensor,
                 compute: Callable):
        self.rank, self.world = rank, world
        self.start, self.end = decode_shards(batch, world)[rank]
        self.state = state            # [end - start, H_v, V, K], resident
        self.compute = compute

    def step(self, q, k, v, A_log, a, dt_bias, b, scale, output=None):
        n = self.end - self.start
        if output is None:
            output = torch.empty((n, 1, v.shape[2], v.shape[3]), dtype=torch.bfloat16,
                                 device=q.device)
        self.compute(q, k, v, self.state, A_log, a, dt_bias, b, scale, output, self.state)
        return output


def run_prefill_shard(rank: int, world: int, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens,
                      scale, compute: Callable, device=None, cu_dtype=torch.int32):
    """Pack this rank's sequences (LPT assignment), run ``compute`` (the prefill
    entry point, DPS) on them, and return (shard, output, new_state)."""
    lengths = (cu_seqlens[1:] - cu_seqlens[:-1]).cpu().tolist()
    seq_ids = prefill_shards(lengths, world)[rank]
    shard = make_prefill_shard(cu_seqlens, seq_ids, cu_dtype)
    lq, lk, lv, ls, la, lb = gather_prefill_inputs(shard, q, k, v, state, a, b)
    dev = device if device is not None else q.device
    mv = lambda t: None if t is None else t.to(dev)
    lq, lk, lv, ls, la, lb = (mv(t) for t in (lq, lk, lv, ls, la, lb))
    T_local = lq.shape[0]
    out = torch.empty((T_local, v.shape[1], v.shape[2]), dtype=torch.bfloat16, device=dev)
    ns = torch.empty((len(seq_ids), v.shape[1], v.shape[2], v.shape[2]), dtype=torch.float32,
                     device=dev)
    if seq_ids:
        compute(lq, lk, lv, ls, mv(A_log), la, mv(dt_bias), lb, shard.cu_seqlens.to(dev), scale,
                out, ns)
    return shard, out, ns


# ----------------------------------------------------------------------------- host workers
@dataclasses.dataclass
class WorkerResult:
    rank: int
    ok: bool
    value: object = None
    error: Optional[str] = None


def _worker_main(fn, rank, world, port, backend, result_q, pg_timeout_s):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=pg_timeout_s))
        value = fn(rank, world)
        # Serialise by value: tensors put on a multiprocessing queue would
        # otherwise be shared through a file descriptor that this process's
        # resource sharer serves, which is gone once the process exits.
        buf = io.BytesIO()
        torch.save(value, buf)
        result_q.put(WorkerResult(rank, True, buf.getvalue()))
    except BaseException:  # noqa: BLE001 - reported to the parent, never swallowed
        result_q.put(WorkerResult(rank, False, error=traceback.format_exc()))
    finally:
        try:
            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def free_port() -> int:
    """A TCP port on 127.0.0.1 that is free right now (for the rendezvous store)."""
    import socket
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch_workers(fn: Callable[[int, int], object], world: int, port: Optional[int] = None,
                   backend: str = "gloo", timeout_s: float = 120.0,
                   pg_timeout_s: float = 30.0) -> List[WorkerResult]:
    """Run ``fn(rank, world)`` in ``world`` spawned processes joined by a process
    group; return one WorkerResult per rank.  A rank that raises is reported
    with its traceback; a rank that neither reports nor exits within
    ``timeout_s`` is terminated and reported as failed.  ``fn`` must be
    picklable (a module-level function)."""
    if port is None:
        port = free_port()
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    procs = [ctx.Process(target=_worker_main,
                         args=(fn, r, world, port, backend, result_q, pg_timeout_s),
                         daemon=False) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    import time
    deadline = time.monotonic() + timeout_s
    while len(results) < world and time.monotonic() < deadline:
        try:
            res = result_q.get(timeout=0.2)
            if res.ok:
                res.value = torch.load(io.BytesIO(res.value), weights_only=False)
            results[res.rank] = res
        except queue_mod.Empty:
            if all(not p.is_alive() for p in procs) and result_q.empty():
                break
    for r, p in enumerate(procs):
        p.join(timeout=max(0.0, deadline - time.monotonic()) if r not in results else 10.0)
        if p.is_alive():
            p.terminate()
            p.join(5.0)
        if r not in results:
            results[r] = WorkerResult(r, False, error=f"rank {r} did not report "
                                                      f"(exit code {p.exitcode})")
    return [results[r] for r in range(world)]
