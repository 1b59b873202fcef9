"""Device-side failure detection without a GPU fault: a bounded mbarrier wait
that nothing satisfies runs out, the kernel records a status bit and returns,
and the context keeps working (the prefill kernels use the same wait)."""

import ctypes
import time

import pytest
import torch

from helpers import DECODE_OUT_TOL, assert_prefill_close
from gdn_kernel_b200 import _lib, kernel as K, workloads as W
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports():
    lib = _lib.load()
    dev = torch.cuda.current_device()
    assert _lib.device_status(dev) == 0
    t0 = time.monotonic()
    rc = lib.gdn_b200_selftest_wait_timeout(
        2_000_000, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))   # 2 ms
    assert rc == _lib.GDN_B200_OK
    status = _lib.device_status(dev)          # synchronises, reads and clears
    assert status == _lib.STATUS_SELFTEST_WAIT
    assert time.monotonic() - t0 < 30.0
    assert _lib.device_status(dev) == 0       # cleared
    # the context is still usable: a decode step matches the oracle
    x = W.make_decode_inputs(4, seed=9)
    c = lambda t: t.cuda()
    out, ns = K.decode(c(x.q), c(x.k), c(x.v), c(x.state), c(x.A_log), c(x.a), c(x.dt_bias),
                       c(x.b), x.scale)
    ro, rs = O.decode_step(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    torch.testing.assert_close(out.cpu().float(), ro.float(), **DECODE_OUT_TOL)



def test_chain_kernel_abort_path_exercised():
    """The chain kernel's multi-role abort path, run for real: a self-test call
    over a properly prepared workspace withholds each sequence's stage loads
    from its third chunk on and limits every wait to 1 ms.  The first wait on a
    withheld stage runs out, the CTA raises its abort flag, all twelve warps
    leave their loops, drain the copies and tensor-core operations they have
    in flight and the CTA frees its TMEM.  The call returns, the status word
    records the timeout, aborted CTAs leave new_state unwritten, and the next
    prefill (every SM's TMEM allocated again) and decode match the oracle."""
    lib = _lib.load()
    dev = torch.cuda.current_device()
    assert _lib.device_status(dev) == 0
    lengths = [600, 300]
    x = W.make_prefill_inputs(lengths, seed=81, device="cuda")
    T, N = sum(lengths), len(lengths)
    need = K.prefill_workspace_bytes(N, T, 32)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    K.gdn_prefill_prepare(x.q, x.k, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, ws)
    out = torch.zeros(T, 32, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.zeros_like(x.state)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    t0 = time.monotonic()
    rc = lib.gdn_b200_selftest_prefill_abort(
        1_000_000, p(x.k), p(x.v), p(x.state), p(out), p(ns), N, T, 16, 32, 128, p(ws), need,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.GDN_B200_OK, lib.gdn_b200_last_error()
    status = _lib.device_status(dev)          # synchronises, reads and clears
    timeouts = _lib.STATUS_TMA_TIMEOUT | _lib.STATUS_MMA_TIMEOUT
    assert status & timeouts and not status & ~timeouts, status
    assert time.monotonic() - t0 < 30.0
    assert torch.count_nonzero(ns) == 0
    # the context and every SM's TMEM are usable again
    xs = W.make_prefill_inputs([700, 0, 129], seed=82)
    c = lambda t: None if t is None else t.cuda()
    o2, s2 = K.prefill(*(c(getattr(xs, n)) for n in ("q", "k", "v", "state", "A_log", "a",
                                                    "dt_bias", "b", "cu_seqlens")), xs.scale)
    ro, rs = O.prefill_chunked(xs.q, xs.k, xs.v, xs.state, xs.A_log, xs.a, xs.dt_bias, xs.b,
                               xs.cu_seqlens, xs.scale)
    assert_prefill_close(o2.cpu(), s2.cpu(), ro, rs, [700, 0, 129])
    xd = W.make_decode_inputs(4, seed=83)
    od, sd = K.decode(*(c(getattr(xd, n)) for n in ("q", "k", "v", "state", "A_log", "a",
                                                   "dt_bias", "b")), xd.scale)
    rdo, rds = O.decode_step(xd.q, xd.k, xd.v, xd.state, xd.A_log, xd.a, xd.dt_bias, xd.b, xd.scale)
    torch.testing.assert_close(od.cpu().float(), rdo.float(), **DECODE_OUT_TOL)
    assert _lib.device_status(dev) == 0
