"""A packed Solution loaded from its own sources alone (as the contest harness
would) runs the reference's `kernel` signatures at the contest's qk4_v8 head
layout: it matches the CPU oracle and, bit for bit, this package's C ABI."""

import importlib.util

import pytest
import torch

from helpers import DECODE_OUT_TOL, DECODE_STATE_TOL, assert_prefill_close
from gdn_kernel_b200 import _lib, kernel as K, pack, workloads as W
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu


def _load(kind, tmp_path):
    entry = pack.unpack(pack.solution(kind), str(tmp_path / kind))
    spec = importlib.util.spec_from_file_location(f"gdn_solution_{kind}_gpu", entry)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.kernel


def test_packed_decode_solution(tmp_path):
    kernel = _load("decode", tmp_path)
    x = W.make_decode_inputs(8, seed=61, h_qk=4, h_v=8)
    d = {n: getattr(x, n).cuda() for n in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")}
    out = torch.empty(8, 1, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty_like(d["state"])
    kernel(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"], x.scale,
           out, ns)
    ro, rs = O.decode_step(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    co, cs = K.decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                      d["b"], x.scale)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu().float(), ro.float(), **DECODE_OUT_TOL)
    torch.testing.assert_close(ns.cpu(), rs, **DECODE_STATE_TOL)
    assert torch.equal(out, co) and torch.equal(ns, cs)


def test_packed_prefill_solution(tmp_path):
    kernel = _load("prefill", tmp_path)
    lengths = [100, 0, 300, 1]
    x = W.make_prefill_inputs(lengths, seed=62, h_qk=4, h_v=8, cu_dtype=torch.int64)
    d = {n: getattr(x, n).cuda() for n in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b",
                                           "cu_seqlens")}
    T = sum(lengths)
    out = torch.empty(T, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty_like(d["state"])
    kernel(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"], d["b"],
           d["cu_seqlens"], x.scale, out, ns)
    co, cs = K.prefill(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                       d["b"], d["cu_seqlens"], x.scale)
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
    ro, rs = O.prefill_chunked(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                               x.cu_seqlens, x.scale)
    assert_prefill_close(out.cpu(), ns.cpu(), ro, rs, lengths)
    assert torch.equal(out, co) and torch.equal(ns, cs)
