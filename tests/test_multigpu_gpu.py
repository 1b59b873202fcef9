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


def test_calls_on_another_device_make_it_current():
    """Tensors on cuda:1 while device 0 is current: the wrappers and the TVM-FFI
    exports make the tensors' device current for the call (the library launches
    on the current device) and restore device 0.  First the library must see
    torch's device switch at all (it links its own CUDA runtime, which follows
    the thread's current context); only then are kernels launched, and their
    results must equal the same calls made with device 1 current."""
    _need(2)
    from gdn_kernel_b200 import _lib
    lib = _lib.load()
    torch.cuda.set_device(0)
    assert lib.gdn_b200_current_device() == 0
    with torch.cuda.device(1):
        assert lib.gdn_b200_current_device() == 1
    assert lib.gdn_b200_current_device() == 0

    dev = torch.device("cuda", 1)
    xd = W.make_decode_inputs(4, seed=3, device=dev)
    xp = W.make_prefill_inputs([300, 0, 2000], seed=4, device=dev)

    def run():
        st = xd.state.clone()
        out = torch.empty(4, 1, 32, 128, dtype=torch.bfloat16, device=dev)
        K.gdn_decode(xd.q, xd.k, xd.v, st, xd.A_log, xd.a, xd.dt_bias, xd.b, xd.scale, out, st)
        res = [out, st]
        for path in ("split", "ring"):
            res += list(K.prefill(xp.q, xp.k, xp.v, xp.state, xp.A_log, xp.a, xp.dt_bias, xp.b,
                                  xp.cu_seqlens, xp.scale, path=path))
        tvm_dec, tvm_pre = K.load_tvm_kernel("decode"), K.load_tvm_kernel("prefill")
        o2, s2 = torch.empty_like(out), xd.state.clone()
        tvm_dec(xd.q, xd.k, xd.v, s2, xd.A_log, xd.a, xd.dt_bias, xd.b, xd.scale, o2, s2)
        o3 = torch.empty(2300, 32, 128, dtype=torch.bfloat16, device=dev)
        s3 = torch.empty_like(xp.state)
        tvm_pre(xp.q, xp.k, xp.v, xp.state, xp.A_log, xp.a, xp.dt_bias, xp.b, xp.cu_seqlens,
                xp.scale, o3, s3)
        torch.cuda.synchronize(dev)
        return res + [o2, s2, o3, s3]

    got = run()                      # device 0 current
    assert torch.cuda.current_device() == 0 and lib.gdn_b200_current_device() == 0
    assert _lib.device_status(1) == 0 and _lib.device_status(0) == 0
    with torch.cuda.device(1):
        ref = run()
    for a, b in zip(got, ref):
        assert a.device == dev and torch.equal(a, b)
