"""The TVM-FFI `kernel` exports (what the reference's harness binds) give the
same results as the C-ABI path, with the reference's argument order.  Both
launch the same kernels on the same inputs, so the results agree bit for bit."""

import pytest
import torch

from helpers import assert_prefill_close
from gdn_kernel_b200 import kernel as K, workloads as W

pytestmark = pytest.mark.gpu


def test_tvm_decode_kernel_matches_capi():
    tvm_kernel = K.load_tvm_kernel("decode")
    x = W.make_decode_inputs(8, seed=3, device="cuda")
    out = torch.empty(8, 1, 32, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty_like(x.state)
    tvm_kernel(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale, out, ns)
    ro, rs = K.decode(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    torch.cuda.synchronize()
    assert torch.equal(out, ro)
    assert torch.equal(ns, rs)


def test_tvm_prefill_kernel_matches_capi():
    tvm_kernel = K.load_tvm_kernel("prefill")
    lengths = [200, 0, 64, 7]
    x = W.make_prefill_inputs(lengths, seed=4, device="cuda", cu_dtype=torch.int64)
    T = sum(lengths)
    out = torch.empty(T, 32, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty_like(x.state)
    tvm_kernel(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale, out, ns)
    ro, rs = K.prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale)
    torch.cuda.synchronize()
    assert torch.equal(out, ro)
    assert torch.equal(ns, rs)
    assert_prefill_close(out.cpu(), ns.cpu(), ro.cpu(), rs.cpu(), lengths)


def test_tvm_prefill_kernel_allocates_nothing():
    """The drop-in `kernel` works in the library's static record ring: a call
    that needs several ring windows (one 50,000-token sequence) leaves torch's
    allocator and the device's free memory untouched and matches the workspace
    path bit for bit.  (A first call loads the library's device image, whose
    static arrays are allocated then, once per process and device.)"""
    tvm_kernel = K.load_tvm_kernel("prefill")
    T = 50000
    x = W.make_prefill_inputs([T], seed=5, device="cuda", cu_dtype=torch.int64)
    out = torch.empty(T, 32, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty_like(x.state)
    tvm_kernel(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale, out,
               torch.empty_like(x.state))
    torch.cuda.synchronize()
    before = torch.cuda.memory_stats()["allocation.all.allocated"]
    free0, _ = torch.cuda.mem_get_info()
    tvm_kernel(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale, out, ns)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_stats()["allocation.all.allocated"] == before
    assert free1 == free0
    ro, rs = K.prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale)
    torch.cuda.synchronize()
    assert torch.equal(out, ro)
    assert torch.equal(ns, rs)


def test_tvm_prefill_rejects_bad_dtype():
    tvm_kernel = K.load_tvm_kernel("prefill")
    x = W.make_prefill_inputs([10], seed=1, device="cuda")
    out = torch.empty(10, 32, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty_like(x.state)
    with pytest.raises(Exception):
        tvm_kernel(x.q.float(), x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                   x.scale, out, ns)
