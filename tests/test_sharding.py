"""Host-side logic of the sequence-sharded multi-GPU driver, on CPU: partitioning,
packing, 2-rank gloo runs (oracle as the per-rank compute) and failure reports."""

import random

import pytest
import torch

import dist_workers as DW
from gdn_kernel_b200 import sharding as S, workloads as W
from oracle import gdn_oracle as O


def test_decode_shards_cover_contiguously():
    for batch in (0, 1, 7, 64, 1024, 1023):
        for world in (1, 2, 3, 8):
            sh = S.decode_shards(batch, world)
            assert sh[0][0] == 0 and sh[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(sh, sh[1:]))
            sizes = [e - s for s, e in sh]
            assert max(sizes) - min(sizes) <= 1


def test_prefill_shards_partition_and_balance():
    rng = random.Random(0)
    for world in (1, 2, 4, 8):
        lengths = [rng.randint(0, 16384) for _ in range(64)]
        sh = S.prefill_shards(lengths, world)
        flat = sorted(i for s in sh for i in s)
        assert flat == list(range(len(lengths)))
        cost = [(L + 63) // 64 for L in lengths]
        loads = [sum(cost[i] for i in s) for s in sh]
        # LPT bound: max load <= 4/3 of the optimum; the optimum >= mean and >= the largest job
        lower = max(sum(cost) / world, max(cost))
        assert max(loads) <= 4 / 3 * lower + 1
        for sh_r in sh:   # each rank packs its sequences longest first
            assert [cost[i] for i in sh_r] == sorted((cost[i] for i in sh_r), reverse=True)


def test_pack_and_scatter_roundtrip():
    x = W.make_prefill_inputs([5, 0, 70, 3], seed=1, h_qk=1, h_v=2)
    shards = [S.make_prefill_shard(x.cu_seqlens, ids) for ids in S.prefill_shards([5, 0, 70, 3], 2)]
    outs, states = [], []
    for sh in shards:
        q, k, v, st, a, b = S.gather_prefill_inputs(sh, x.q, x.k, x.v, x.state, x.a, x.b)
        assert q.shape[0] == sum(sh.lengths) == int(sh.cu_seqlens[-1])
        outs.append(v)          # identity "compute": output = v
        states.append(st)
    out, ns = S.scatter_prefill_outputs(shards, outs, states, 78, 4)
    assert torch.equal(out, x.v) and torch.equal(ns, x.state)


def test_two_rank_prefill_matches_single_process():
    res = S.launch_workers(DW.sharded_prefill_worker, 2)
    assert all(r.ok for r in res), [r.error for r in res]
    out, ns = res[0].value
    x = W.make_prefill_inputs(DW.PREFILL_LENGTHS, seed=77, h_qk=2, h_v=4)
    ro, rs = O.prefill_chunked(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                               x.cu_seqlens, x.scale)
    torch.testing.assert_close(out.float(), ro.float(), atol=0, rtol=0)
    torch.testing.assert_close(ns, rs, atol=1e-6, rtol=1e-6)


def test_two_rank_decode_matches_single_process():
    res = S.launch_workers(DW.sharded_decode_worker, 2)
    assert all(r.ok for r in res), [r.error for r in res]
    outs, state = res[0].value
    first, tokens = W.make_decode_run(DW.DECODE_BATCH, 3, seed=12, h_qk=2, h_v=4)
    st = first.state
    ref = []
    for (q, k, v, a, b) in tokens:
        o, st = O.decode_step(q, k, v, st, first.A_log, a, first.dt_bias, b, first.scale)
        ref.append(o)
    torch.testing.assert_close(outs.float(), torch.stack(ref).float(), atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(state, st, atol=1e-6, rtol=1e-6)


def test_failed_rank_is_reported_and_others_finish():
    res = S.launch_workers(DW.failing_worker, 2)
    assert res[0].ok and res[0].value == "rank0 done"
    assert not res[1].ok and "injected failure on rank 1" in res[1].error


def test_peer_failure_ends_collective_with_error_not_hang():
    res = S.launch_workers(DW.failing_before_barrier_worker, 2, timeout_s=90,
                           pg_timeout_s=5)
    assert not res[1].ok and "injected failure" in res[1].error
    assert not res[0].ok        # its barrier failed instead of waiting forever


def test_silent_rank_is_terminated_at_the_deadline():
    res = S.launch_workers(DW.silent_worker, 2, timeout_s=20)
    assert res[0].ok and res[0].value == 0
    assert not res[1].ok and "did not report" in res[1].error
