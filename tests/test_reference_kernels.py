"""Pin the CPU oracle against the reference repository's own CUDA kernels.

oracle/build_ref.sh compiles ref solution/cuda/kernel.cu and kernel_prefill.cu
unmodified into oracle/_ref/ (TVM-FFI modules exporting `kernel`).  They hard-code
the qk4_v8 head layout, so the comparison runs there: reference kernel vs oracle,
and reference kernel vs this package's kernels on the same inputs.
"""

import os

import pytest
import torch

from conftest import ROOT
from helpers import (DECODE_OUT_TOL, DECODE_STATE_TOL, assert_prefill_close)
from gdn_kernel_b200 import kernel as K, workloads as W
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

REF_DIR = os.path.join(ROOT, "oracle", "_ref")


def _ref_kernel(name):
    path = os.path.join(REF_DIR, name)
    if not os.path.exists(path):
        pytest.skip(f"{path} not built (oracle/build_ref.sh needs the reference tree)")
    tvm_ffi = pytest.importorskip("tvm_ffi")
    return tvm_ffi.load_module(path)["kernel"]


def test_reference_decode_kernel_matches_oracle_and_ours():
    ref = _ref_kernel("ref_decode.so")
    x = W.make_decode_inputs(6, seed=31, h_qk=4, h_v=8, device="cuda")
    out = torch.empty(6, 1, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(6, 8, 128, 128, dtype=torch.float32, device="cuda")
    ref(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale, out, ns)
    torch.cuda.synchronize()
    cpu = lambda t: t.cpu()
    ro, rs = O.decode_step(*(cpu(t) for t in (x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias,
                                              x.b)), x.scale)
    torch.testing.assert_close(out.cpu().float(), ro.float(), **DECODE_OUT_TOL)
    torch.testing.assert_close(ns.cpu(), rs, **DECODE_STATE_TOL)
    mo, ms = K.decode(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    torch.cuda.synchronize()
    torch.testing.assert_close(mo.float(), out.float(), **DECODE_OUT_TOL)
    torch.testing.assert_close(ms, ns, **DECODE_STATE_TOL)


def test_reference_prefill_kernel_matches_oracle_and_ours():
    ref = _ref_kernel("ref_prefill.so")
    lengths = [37, 0, 129, 1, 300]
    x = W.make_prefill_inputs(lengths, seed=41, h_qk=4, h_v=8, device="cuda",
                              cu_dtype=torch.int64)   # the reference reads int64 only
    T = sum(lengths)
    out = torch.empty(T, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(len(lengths), 8, 128, 128, dtype=torch.float32, device="cuda")
    ref(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale, out, ns)
    torch.cuda.synchronize()
    c = {n: getattr(x, n).cpu() for n in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b",
                                          "cu_seqlens")}
    ro, rs = O.prefill_chunked(c["q"], c["k"], c["v"], c["state"], c["A_log"], c["a"],
                               c["dt_bias"], c["b"], c["cu_seqlens"], x.scale)
    # the reference is all-fp32: tight agreement with the fp32 oracle
    torch.testing.assert_close(out.cpu().float(), ro.float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(ns.cpu(), rs, atol=1e-4, rtol=1e-3)
    mo, ms = K.prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                       x.scale)
    torch.cuda.synchronize()
    assert_prefill_close(mo.cpu(), ms.cpu(), out.cpu(), ns.cpu(), lengths)
