"""Device-side failure detection without a GPU fault: a bounded mbarrier wait
that nothing satisfies runs out, the kernel records a status bit and returns,
and the context keeps working (the prefill kernels use the same wait)."""

import ctypes
import time

import pytest
import torch

from helpers import DECODE_OUT_TOL
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

