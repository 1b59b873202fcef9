"""Sequence-sharded runs on 2, 4 and 8 GPUs (one process each) equal the single-GPU
run bitwise: every CTA of both kernels touches one sequence only.  Context-parallel
prefill at 4 GPUs also exercises the middle ranks (prepare + segment maps); at 8 the
333-token sequence leaves three ranks with empty segments (identity maps) and the
5-entry decode batch leaves three ranks with no entries."""

import pytest
import torch

import dist_workers as DW
from gdn_kernel_b200 import kernel as K, sharding as S, workloads as W

pytestmark = pytest.mark.gpu


WORLDS = pytest.mark.parametrize("world", [2, 4, 8])


def _need(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


@WORLDS
def test_multi_gpu_prefill_equals_one_gpu(world):
    _need(world)
    res = S.launch_workers(DW.gpu_prefill_worker, world, timeout_s=300)
    assert all(r.ok for r in res), [r.error for r in res]
    out, ns = res[0].value
    # the workers draw their inputs on the CPU (CPU and CUDA generators differ)
    x = W.make_prefill_inputs(DW.PREFILL_LENGTHS, seed=77, h_qk=2, h_v=4)
    c = lambda t: t.cuda()
    ro, rs = K.prefill(c(x.q), c(x.k), c(x.v), c(x.state), c(x.A_log), c(x.a), c(x.dt_bias),
                       c(x.b), c(x.cu_seqlens), x.scale)
    assert torch.equal(out, ro.cpu()) and torch.equal(ns, rs.cpu())


@WORLDS
def test_multi_gpu_decode_equals_one_gpu(world):
    _need(world)
    res = S.launch_workers(DW.gpu_decode_worker, world, timeout_s=300)
    assert all(r.ok for r in res), [r.error for r in res]
    outs, state = res[0].value
    first, tokens = W.make_decode_run(DW.DECODE_BATCH, 3, seed=12, h_qk=2, h_v=4)
    st = first.state.cuda()
    ref = []
    for (q, k, v, a, b) in tokens:
        o, _ = K.decode(q.cuda(), k.cuda(), v.cuda(), st, first.A_log.cuda(), a.cuda(),
                        first.dt_bias.cuda(), b.cuda(), first.scale, in_place=True)
        ref.append(o.cpu())
    assert torch.equal(outs, torch.stack(ref)) and torch.equal(state, st.cpu())


@WORLDS
def test_multi_gpu_context_parallel_prefill(world):
    """One 333-token sequence split over 2, 4 or 8 GPUs (NCCL all-gather of the
    segment maps) against the fp32 oracle of the whole sequence."""
    _need(world)
    from helpers import assert_prefill_close
    from oracle import gdn_oracle as O
    res = S.launch_workers(DW.gpu_cp_worker, world, backend="nccl", timeout_s=300)
    assert all(r.ok for r in res), [r.error for r in res]
    out, end = res[0].value
    x = DW._cp_inputs()
    ro, rs = O.prefill_chunked(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                               x.cu_seqlens, x.scale)
    assert_prefill_close(out, end[None], ro, rs)
