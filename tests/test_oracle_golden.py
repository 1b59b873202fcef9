"""Pin the CPU oracle against the golden fixtures (tests/golden/make_golden.py),
which were produced by the published contest definition functions."""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from gdn_kernel_b200 import workloads as W
from oracle import gdn_oracle as O


def _load(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def _t(arr):
    if arr.dtype == np.uint16:
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(arr.copy())


def _checksum(t):
    f = t.double()
    return np.array([f.sum().item(), (f * f).sum().item()])


def test_decode_config0_16_steps():
    """B=4, qk16_v32, 16 consecutive decode steps from seed 0."""
    g = _load("decode_b4_qk16v32_16steps.npz")
    first, tokens = W.make_decode_run(4, 16, seed=0)
    # inputs regenerated from the seed must be the ones the fixture was made from
    np.testing.assert_allclose(_checksum(first.state), g["in_state"], rtol=1e-12)
    for s, (q, k, v, a, b) in enumerate(tokens):
        for name, t in (("q", q), ("k", k), ("v", v), ("a", a), ("b", b)):
            np.testing.assert_allclose(_checksum(t.float()), g[f"in_{name}_{s}"], rtol=1e-12)
    state = first.state
    outs = []
    for (q, k, v, a, b) in tokens:
        o, state = O.decode_step(q, k, v, state, first.A_log, a, first.dt_bias, b, first.scale)
        outs.append(o)
    out = torch.stack(outs).float()
    ref = _t(g["outputs"]).float()
    torch.testing.assert_close(out, ref, atol=1e-2, rtol=1e-2)
    # a few bf16 ulps at most, not just within tolerance
    assert (out - ref).abs().max().item() < 4e-3
    np.testing.assert_allclose(state.double().sum(-1).numpy(), g["state_rowsum"], atol=1e-4)
    np.testing.assert_allclose((state.double() ** 2).sum(-1).numpy(), g["state_rowsq"],
                               rtol=1e-4, atol=1e-7)
    np.testing.assert_allclose(state[0, 0].numpy(), g["state_head_first"], atol=1e-5)
    np.testing.assert_allclose(state[-1, -1].numpy(), g["state_head_last"], atol=1e-5)


@pytest.mark.parametrize("tag", ["state", "nostate"])
def test_decode_small(tag):
    g = _load(f"decode_small_{tag}.npz")
    args = {n: _t(g[n]) for n in ("q", "k", "v", "A_log", "a", "dt_bias", "b")}
    state = _t(g["state"]) if tag == "state" else None
    o, ns = O.decode_step(args["q"], args["k"], args["v"], state, args["A_log"], args["a"],
                          args["dt_bias"], args["b"], 0.0)
    torch.testing.assert_close(o.float(), _t(g["output"]).float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(ns, _t(g["new_state"]), atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("fn", ["sequential", "chunked"])
@pytest.mark.parametrize("tag", ["state", "nostate"])
def test_prefill_small(tag, fn):
    g = _load(f"prefill_small_{tag}.npz")
    args = {n: _t(g[n]) for n in ("q", "k", "v", "A_log", "a", "dt_bias", "b", "cu_seqlens")}
    state = _t(g["state"]) if tag == "state" else None
    f = O.prefill_sequential if fn == "sequential" else O.prefill_chunked
    o, ns = f(args["q"], args["k"], args["v"], state, args["A_log"], args["a"], args["dt_bias"],
              args["b"], args["cu_seqlens"], 0.0)
    torch.testing.assert_close(o.float(), _t(g["output"]).float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(ns, _t(g["new_state"]), atol=1e-5, rtol=1e-4)


def test_prefill_full_heads_T150():
    g = _load("prefill_qk16v32_T150.npz")
    x = W.make_prefill_inputs([150], seed=3)
    for n in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b"):
        np.testing.assert_allclose(_checksum(getattr(x, n).float()), g[f"in_{n}"], rtol=1e-12)
    for f in (O.prefill_sequential, O.prefill_chunked):
        o, ns = f(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale)
        torch.testing.assert_close(o.float(), _t(g["output"]).float(), atol=1e-2, rtol=1e-2)
        np.testing.assert_allclose(ns.double().sum(-1).numpy(), g["state_rowsum"], atol=1e-4)
        np.testing.assert_allclose(ns[0, 0].numpy(), g["state_head_first"], atol=1e-5)
        np.testing.assert_allclose(ns[-1, -1].numpy(), g["state_head_last"], atol=1e-5)


def test_oracle_flags_planted_mistake():
    """A mistake planted in the oracle (beta dropped) must be caught by the fixture."""
    g = _load("decode_small_state.npz")
    args = {n: _t(g[n]) for n in ("q", "k", "v", "A_log", "a", "dt_bias", "b")}
    bad_b = torch.full_like(args["b"], 30.0)   # sigmoid(30) == 1: beta removed
    o, _ = O.decode_step(args["q"], args["k"], args["v"], _t(g["state"]), args["A_log"],
                         args["a"], args["dt_bias"], bad_b, 0.0)
    assert (o.float() - _t(g["output"]).float()).abs().max().item() > 1e-2


def test_gate_softplus_threshold():
    """softplus(x) = x above 20 (ref kernel.cu:51) and log(1+e^x) below."""
    A_log = torch.zeros(2)
    a = torch.tensor([[25.0, -3.0]]).to(torch.bfloat16)
    lg, beta = O.log_gate_beta(A_log, a, torch.zeros(2), torch.zeros(1, 2).to(torch.bfloat16))
    assert lg[0, 0].item() == pytest.approx(-25.0)
    assert lg[0, 1].item() == pytest.approx(-float(np.log1p(np.exp(-3.0))), rel=1e-6)
    assert beta.eq(0.5).all()


def test_chunked_matches_sequential_ragged():
    """The chunked restatement equals the token recurrence on ragged lengths."""
    x = W.make_prefill_inputs([1, 63, 64, 65, 0, 130], seed=9, h_qk=2, h_v=4)
    o1, s1 = O.prefill_sequential(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                                  x.cu_seqlens, x.scale)
    o2, s2 = O.prefill_chunked(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                               x.cu_seqlens, x.scale)
    torch.testing.assert_close(o1.float(), o2.float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(s1, s2, atol=1e-5, rtol=1e-4)


def test_chunk_states_are_the_token_recurrence_at_chunk_ends():
    """The per-chunk states the chunked oracle reports (the state entering each
    chunk, ref prefill_design.md:600-606 asks tests to compare these) equal the
    token-by-token recurrence stopped at each chunk end."""
    x = W.make_prefill_inputs([200], seed=12, h_qk=2, h_v=4)
    _, fin, cs = O.prefill_chunked(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                                   x.cu_seqlens, x.scale, return_chunk_states=True)
    assert cs[0].shape[0] == 4   # chunks of 64, 64, 64, 8 tokens
    for j, end in enumerate((0, 64, 128, 192)):
        if end == 0:
            torch.testing.assert_close(cs[0][0], x.state[0])
            continue
        cu = torch.tensor([0, end], dtype=x.cu_seqlens.dtype)
        _, s_seq = O.prefill_sequential(x.q[:end], x.k[:end], x.v[:end], x.state, x.A_log,
                                        x.a[:end], x.dt_bias, x.b[:end], cu, x.scale)
        torch.testing.assert_close(cs[0][j], s_seq[0], atol=1e-5, rtol=1e-4)


def _mtp_fixture_inputs(g):
    x = W.make_pool_decode_inputs(3, 3, 5, seed=21, h_qk=1, h_v=2)
    for n in ("q", "k", "v", "pool", "A_log", "a", "dt_bias", "b"):
        np.testing.assert_allclose(_checksum(getattr(x, n).float()), g[f"in_{n}"], rtol=1e-12)
    return x, torch.from_numpy(g["indices"].copy())


def test_mtp_pool_matches_definition():
    """Multi-token decode against a state pool, with intermediate states: the
    oracle against the MTP definition function's fixture."""
    g = _load("mtp_b3_t3_qk1v2_pool5.npz")
    x, idx = _mtp_fixture_inputs(g)
    inter = torch.zeros(5, 3, 2, 128, 128)
    out, pool = O.decode_pool(x.q, x.k, x.v, x.pool, idx, x.A_log, x.a, x.dt_bias, x.b, 0.0,
                              inter=inter)
    ref = _t(g["output"]).float()
    assert (out.float() - ref).abs().max().item() < 4e-3
    np.testing.assert_allclose(pool.double().sum(-1).numpy(), g["pool_rowsum"], atol=1e-4)
    np.testing.assert_allclose((pool.double() ** 2).sum(-1).numpy(), g["pool_rowsq"],
                               rtol=1e-4, atol=1e-7)
    np.testing.assert_allclose(pool[2, 1].numpy(), g["pool_slot2_head1"], atol=1e-5)
    np.testing.assert_allclose(inter.double().sum(-1).numpy(), g["inter_rowsum"], atol=1e-4)
    np.testing.assert_allclose(inter[0, 1, 0].numpy(), g["inter_slot0_t1_head0"], atol=1e-5)
    # untouched slots are copied through
    assert torch.equal(pool[1], x.pool[1]) and torch.equal(pool[4], x.pool[4])


def test_pool_decode_padding_and_write_slots():
    """Host semantics of the pool addressing: a negative index is padding (zero
    output, no state traffic); write slots may differ from read slots; T=1 with
    identity slots is the plain decode step."""
    x = W.make_pool_decode_inputs(3, 1, 6, seed=4, h_qk=1, h_v=2)
    read = torch.tensor([4, -1, 0])
    write = torch.tensor([1, 3, 5])
    out, pool = O.decode_pool(x.q, x.k, x.v, x.pool, read, x.A_log, x.a, x.dt_bias, x.b, 0.0,
                              write_idx=write)
    assert out[1].abs().max().item() == 0.0
    for s in (0, 2, 3, 4):      # not written (3 belongs to the padding entry)
        assert torch.equal(pool[s], x.pool[s])
    o1, s1 = O.decode_step(x.q[[0]], x.k[[0]], x.v[[0]], x.pool[[4]], x.A_log, x.a[[0]],
                           x.dt_bias, x.b[[0]], 0.0)
    assert torch.equal(out[[0]], o1) and torch.equal(pool[1], s1[0])
