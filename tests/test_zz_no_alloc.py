"""The allocation-free prefill entry point, gdn_b200_prefill_static.

Some callers cannot allocate device memory: hosts bound to the reference's
fixed `kernel` argument list (no slot for a workspace), plugin hosts whose
framework owns all device memory, and serving loops that cannot take an
allocation on the hot path.  For them the library keeps a fixed-size scratch
array in its own device image.  These tests call that entry point through the
C ABI and compare it with the workspace entry point on the same inputs, on
two calls in a row (the second call finds the first call's leftovers in the
shared scratch), and check that an oversized problem is refused.

This file is named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

from helpers import assert_prefill_close
from gdn_kernel_b200 import _lib, kernel as K, workloads as W

pytestmark = pytest.mark.gpu

STATIC_SCRATCH_BYTES = 64 << 20   # GDN_B200_PREFILL_STATIC_SCRATCH_BYTES


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _call_static(x, out, ns):
    lib = _lib.load()
    T, h_qk, D = x.q.shape
    h_v = x.v.shape[1]
    N = x.cu_seqlens.numel() - 1
    return lib.gdn_b200_prefill_static(
        _p(x.q), _p(x.k), _p(x.v), _p(x.state), _p(x.A_log), _p(x.a), _p(x.dt_bias), _p(x.b),
        _p(x.cu_seqlens), 1 if x.cu_seqlens.dtype == torch.int64 else 0, float(x.scale),
        _p(out), _p(ns), N, T, h_qk, h_v, D,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_static_scratch_prefill_matches_workspace_entry_point():
    # Calls in a row with different inputs: each later call runs on the scratch
    # contents the call before it left behind.  Both entry points launch the
    # same kernels on the same tiles, so the results agree bit for bit.  The
    # 1100-token single sequence takes the one-sequence path that runs in
    # overlapping pieces (at least 16 chunks).
    for lengths, seed in (([150, 0, 64, 33], 71), ([700, 1, 129], 72), ([1100], 73)):
        x = W.make_prefill_inputs(lengths, seed=seed, device="cuda")
        T = sum(lengths)
        assert K.prefill_workspace_bytes(len(lengths), T, 32) <= STATIC_SCRATCH_BYTES
        out = torch.full((T, 32, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
        ns = torch.full_like(x.state, float("nan"))
        rc = _call_static(x, out, ns)
        assert rc == _lib.GDN_B200_OK, _lib.load().gdn_b200_last_error()
        ro, rs = K.prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                           x.scale, path="split")
        torch.cuda.synchronize()
        assert _lib.device_status(torch.cuda.current_device()) == 0
        assert torch.equal(out, ro), lengths
        assert torch.equal(ns, rs), lengths
        assert_prefill_close(out.cpu(), ns.cpu(), ro.cpu(), rs.cpu(), lengths)


def test_static_scratch_refuses_oversized_problem():
    lib = _lib.load()
    z = ctypes.c_void_p(0)
    # one 8192-token sequence needs ~200 MB of workspace: over the 64 MiB limit
    rc = lib.gdn_b200_prefill_static(z, z, z, z, z, z, z, z, z, 0, 0.0, z, z, 1, 8192, 16, 32,
                                     128, z)
    assert rc == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert b"static prefill scratch" in lib.gdn_b200_last_error()
    # a bad extent is reported as such, before the size comparison
    rc = lib.gdn_b200_prefill_static(z, z, z, z, z, z, z, z, z, 0, 0.0, z, z, 70000, 100, 16, 32,
                                     128, z)
    assert rc == _lib.GDN_B200_ERR_INVALID_ARGUMENT
    assert b"num_seqs" in lib.gdn_b200_last_error()
