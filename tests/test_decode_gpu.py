"""Decode kernel (T=1) against the CPU oracle and the golden fixtures, through
the C ABI (gdn_kernel_b200.kernel calls libgdn_b200.so)."""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from helpers import DECODE_OUT_TOL, DECODE_STATE_TOL, to_dev
from gdn_kernel_b200 import _lib, kernel as K, workloads as W
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu


def _run(x, in_place=False, scale=None):
    dev = "cuda"
    q, k, v, a, b = (to_dev(t) for t in (x.q, x.k, x.v, x.a, x.b))
    st = to_dev(x.state)
    out, ns = K.decode(q, k, v, st, to_dev(x.A_log), a, to_dev(x.dt_bias), b,
                       x.scale if scale is None else scale, in_place=in_place)
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
    return out.cpu(), ns.cpu()


@pytest.mark.parametrize("batch", [1, 3, 8, 64])
def test_decode_matches_oracle(batch):
    x = W.make_decode_inputs(batch, seed=100 + batch)
    out, ns = _run(x)
    ro, rs = O.decode_step(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    torch.testing.assert_close(out.float(), ro.float(), **DECODE_OUT_TOL)
    torch.testing.assert_close(ns, rs, **DECODE_STATE_TOL)


@pytest.mark.parametrize("h_qk,h_v", [(4, 8), (1, 2), (32, 32), (2, 16)])
def test_decode_head_layouts(h_qk, h_v):
    """qk4_v8 is the reference's hard-coded layout; others exercise GQA ratios 1 and 8."""
    x = W.make_decode_inputs(5, seed=7, h_qk=h_qk, h_v=h_v)
    out, ns = _run(x)
    ro, rs = O.decode_step(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    torch.testing.assert_close(out.float(), ro.float(), **DECODE_OUT_TOL)
    torch.testing.assert_close(ns, rs, **DECODE_STATE_TOL)


def test_decode_null_state_and_default_scale():
    x = W.make_decode_inputs(4, seed=3, with_state=False)
    out, ns = _run(x, scale=0.0)
    ro, rs = O.decode_step(x.q, x.k, x.v, None, x.A_log, x.a, x.dt_bias, x.b, 0.0)
    torch.testing.assert_close(out.float(), ro.float(), **DECODE_OUT_TOL)
    torch.testing.assert_close(ns, rs, **DECODE_STATE_TOL)


def test_decode_in_place_equals_out_of_place():
    x = W.make_decode_inputs(8, seed=5)
    o1, s1 = _run(x)
    o2, s2 = _run(x, in_place=True)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def _golden(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def _bf16(arr):
    return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)


def test_decode_config0_golden_16_steps_in_place():
    """16 in-place steps at B=4, qk16_v32, against the definition fixture."""
    g = _golden("decode_b4_qk16v32_16steps.npz")
    first, tokens = W.make_decode_run(4, 16, seed=0)
    state = first.state.cuda()
    A_log, dt_bias = first.A_log.cuda(), first.dt_bias.cuda()
    outs = []
    for (q, k, v, a, b) in tokens:
        o, _ = K.decode(q.cuda(), k.cuda(), v.cuda(), state, A_log, a.cuda(), dt_bias, b.cuda(),
                        first.scale, in_place=True)
        outs.append(o.cpu())
    torch.cuda.synchronize()
    out = torch.stack(outs).float()
    torch.testing.assert_close(out, _bf16(g["outputs"]).float(), **DECODE_OUT_TOL)
    s = state.cpu().double()
    np.testing.assert_allclose(s.sum(-1).numpy(), g["state_rowsum"], atol=1e-3)
    np.testing.assert_allclose(s[0, 0].numpy(), g["state_head_first"], **DECODE_STATE_TOL)
    np.testing.assert_allclose(s[-1, -1].numpy(), g["state_head_last"], **DECODE_STATE_TOL)


@pytest.mark.parametrize("tag", ["state", "nostate"])
def test_decode_small_golden(tag):
    g = _golden(f"decode_small_{tag}.npz")
    f = lambda n: torch.from_numpy(g[n].copy()) if g[n].dtype != np.uint16 else _bf16(g[n])
    st = f("state").cuda() if tag == "state" else None
    out, ns = K.decode(f("q").cuda(), f("k").cuda(), f("v").cuda(), st, f("A_log").cuda(),
                       f("a").cuda(), f("dt_bias").cuda(), f("b").cuda(), 0.0)
    torch.testing.assert_close(out.cpu().float(), f("output").float(), **DECODE_OUT_TOL)
    torch.testing.assert_close(ns.cpu(), f("new_state"), **DECODE_STATE_TOL)


def test_decode_large_batch_slices():
    """B=256 (1 GiB of state) on the GPU; the oracle checks a few batch rows."""
    x = W.make_decode_inputs(256, seed=11, device="cuda")
    out, ns = K.decode(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    torch.cuda.synchronize()
    for lo in (0, 131, 255):
        sl = slice(lo, lo + 1)
        ro, rs = O.decode_step(x.q[sl].cpu(), x.k[sl].cpu(), x.v[sl].cpu(), x.state[sl].cpu(),
                               x.A_log.cpu(), x.a[sl].cpu(), x.dt_bias.cpu(), x.b[sl].cpu(),
                               x.scale)
        torch.testing.assert_close(out[sl].cpu().float(), ro.float(), **DECODE_OUT_TOL)
        torch.testing.assert_close(ns[sl].cpu(), rs, **DECODE_STATE_TOL)


def test_decode_rejects_misuse():
    x = W.make_decode_inputs(2, seed=1, device="cuda")
    with pytest.raises(ValueError):   # wrong dtype
        K.decode(x.q.float(), x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    with pytest.raises(ValueError):   # non-contiguous
        K.gdn_decode(x.q, x.k, x.v, x.state.transpose(2, 3), x.A_log, x.a, x.dt_bias, x.b,
                     x.scale, torch.empty_like(x.v), torch.empty_like(x.state))
