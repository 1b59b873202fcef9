"""Chunked prefill kernel (tcgen05) against the CPU oracle and the golden
fixtures, through the C ABI."""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from helpers import (PREFILL_OUT_TOL, PREFILL_STATE_REL_FRO, assert_prefill_close, rel_fro,
                     to_dev)
from gdn_kernel_b200 import _lib, kernel as K, workloads as W
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["split", "fused"])
def path(request):
    """Both prefill paths: the two-stage kernels (default) and the single kernel."""
    return request.param


def _run(x, path="split", in_place=False, cu_dtype=None, scale=None):
    cu = x.cu_seqlens if cu_dtype is None else x.cu_seqlens.to(cu_dtype)
    st = to_dev(x.state)
    out, ns = K.prefill(to_dev(x.q), to_dev(x.k), to_dev(x.v), st, to_dev(x.A_log), to_dev(x.a),
                        to_dev(x.dt_bias), to_dev(x.b), to_dev(cu),
                        x.scale if scale is None else scale, in_place=in_place, path=path)
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
    return out.cpu(), ns.cpu()


def _oracle(x):
    return O.prefill_chunked(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                             x.scale)


def _golden(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def _f(g, n):
    a = g[n]
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(a.copy())


@pytest.mark.parametrize("tag", ["state", "nostate"])
def test_prefill_small_golden(tag, path):
    """Ragged tails, an empty and a 1-token sequence, int64 cu_seqlens (qk1_v2)."""
    g = _golden(f"prefill_small_{tag}.npz")
    st = _f(g, "state").cuda() if tag == "state" else None
    out, ns = K.prefill(*(_f(g, n).cuda() for n in ("q", "k", "v")), st,
                        *(_f(g, n).cuda() for n in ("A_log", "a", "dt_bias", "b", "cu_seqlens")),
                        0.0, path=path)
    torch.cuda.synchronize()
    assert_prefill_close(out, ns, _f(g, "output"), _f(g, "new_state"), lengths=[37, 0, 129, 1])


def test_prefill_full_heads_T150_golden(path):
    g = _golden("prefill_qk16v32_T150.npz")
    x = W.make_prefill_inputs([150], seed=3)
    out, ns = _run(x, path)
    torch.testing.assert_close(out.float(), _f(g, "output").float(), **PREFILL_OUT_TOL)
    np.testing.assert_allclose(ns[0, 0].numpy(), g["state_head_first"], atol=2e-3, rtol=2e-2)
    np.testing.assert_allclose(ns[-1, -1].numpy(), g["state_head_last"], atol=2e-3, rtol=2e-2)


@pytest.mark.parametrize("lengths", [[64], [1], [63], [65], [200], [128, 1, 64, 0, 77]])
def test_prefill_ragged_lengths(lengths, path):
    x = W.make_prefill_inputs(lengths, seed=sum(lengths) + len(lengths))
    out, ns = _run(x, path)
    ro, rs = _oracle(x)
    assert_prefill_close(out, ns, ro, rs, lengths)


def test_prefill_varlen_int32_vs_int64_and_in_place(path):
    lengths = W.varlen_lengths(6, 128, 1024, seed=21)
    x = W.make_prefill_inputs(lengths, seed=21, cu_dtype=torch.int32)
    o32, s32 = _run(x, path)
    o64, s64 = _run(x, path, cu_dtype=torch.int64)
    assert torch.equal(o32, o64) and torch.equal(s32, s64)
    oi, si = _run(x, path, in_place=True)
    assert torch.equal(o32, oi) and torch.equal(s32, si)
    ro, rs = _oracle(x)
    assert_prefill_close(o32, s32, ro, rs, lengths)


def test_prefill_null_state_and_all_empty(path):
    x = W.make_prefill_inputs([100, 0, 30], seed=4, with_state=False)
    out, ns = _run(x, path, scale=0.0)
    ro, rs = _oracle(x)
    assert_prefill_close(out, ns, ro, rs, [100, 0, 30])
    assert ns[1].abs().max().item() == 0.0
    # every sequence empty: states pass through, nothing else is touched
    y = W.make_prefill_inputs([0, 0], seed=5)
    _, ns2 = _run(y, path)
    assert torch.equal(ns2, y.state)


@pytest.mark.parametrize("h_qk,h_v", [(4, 8), (2, 2), (1, 8)])
def test_prefill_head_layouts(h_qk, h_v, path):
    x = W.make_prefill_inputs([70, 190], seed=8, h_qk=h_qk, h_v=h_v)
    out, ns = _run(x, path)
    ro, rs = _oracle(x)
    assert_prefill_close(out, ns, ro, rs)


def test_prefill_config2_T8192_drift(path):
    """one sequence of 8192 tokens, zero initial state; reports drift."""
    x = W.make_prefill_inputs([8192], seed=2, with_state=False)
    out, ns = _run(x, path)
    ro, rs = _oracle(x)
    err = assert_prefill_close(out, ns, ro, rs)
    d = (out.float() - ro.float()).abs()
    print(f"\n[T=8192 drift, {path}] output max-abs {d.max().item():.3e} mean-abs {d.mean().item():.3e}; "
          f"final state rel-Frobenius max {err.max().item():.3e}")


def test_prefill_intermediate_chunk_states(path):
    """The state at every chunk boundary, as the reference's prefill design asks
    tests to compare (ref prefill_design.md:600-606).  One call whose sequences
    are prefixes of the same 500-token stream (1 to 7 whole chunks, a ragged
    100 tokens, and the whole stream), each from the same initial state, returns
    the state after every chunk; each is compared with the state the oracle
    carries into the next chunk of the whole stream.  The packed call's outputs
    and states are checked against the oracle too."""
    import types
    base = W.make_prefill_inputs([500], seed=81)
    ends = [64 * j for j in range(1, 8)] + [100, 500]
    cat = lambda t: torch.cat([t[:e] for e in ends])
    cu = torch.tensor([0] + [sum(ends[:i + 1]) for i in range(len(ends))], dtype=torch.int32)
    x = types.SimpleNamespace(q=cat(base.q), k=cat(base.k), v=cat(base.v),
                              state=base.state.expand(len(ends), -1, -1, -1).contiguous(),
                              A_log=base.A_log, a=cat(base.a), dt_bias=base.dt_bias,
                              b=cat(base.b), cu_seqlens=cu, scale=base.scale)
    out, ns = _run(x, path)
    ro, rs = _oracle(x)
    assert_prefill_close(out, ns, ro, rs, ends)
    _, fin, cs = O.prefill_chunked(base.q, base.k, base.v, base.state, base.A_log, base.a,
                                   base.dt_bias, base.b, base.cu_seqlens, base.scale,
                                   return_chunk_states=True)
    for j in range(1, 8):   # the prefix of j chunks ends where chunk j of the stream starts
        err = rel_fro(ns[j - 1:j], cs[0][j:j + 1])
        assert err.max().item() <= PREFILL_STATE_REL_FRO, (j, err.max().item())
    assert rel_fro(ns[-1:], fin).max().item() <= PREFILL_STATE_REL_FRO


def test_prefill_config3_varlen16(path):
    """16 sequences, lengths U[128, 8192], random initial states, int32."""
    lengths = W.varlen_lengths(16, 128, 8192, seed=3)
    x = W.make_prefill_inputs(lengths, seed=3, cu_dtype=torch.int32)
    out, ns = _run(x, path)
    ro, rs = _oracle(x)
    err = assert_prefill_close(out, ns, ro, rs, lengths)
    print(f"\n[varlen16 drift, {path}] per-seq state rel-Frobenius max "
          f"{[round(float(e), 6) for e in err.max(dim=1).values]}")


def test_prefill_rejects_misuse():
    x = W.make_prefill_inputs([10], seed=1, device="cuda")
    with pytest.raises(ValueError):
        K.prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                  x.cu_seqlens.to(torch.float32), x.scale)
    with pytest.raises(ValueError):
        K.prefill(x.q[:, :3], x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                  x.scale)


def test_split_and_fused_paths_agree():
    """The two paths compute the same products from the same operand tiles."""
    lengths = [300, 1, 64, 0, 129]
    x = W.make_prefill_inputs(lengths, seed=12)
    o1, s1 = _run(x, "split")
    o2, s2 = _run(x, "fused")
    assert (o1.float() - o2.float()).abs().max().item() <= 1e-2
    assert (s1 - s2).abs().max().item() <= 1e-4


def test_split_workspace_contract():
    x = W.make_prefill_inputs([100, 30], seed=6, device="cuda")
    need = K.prefill_workspace_bytes(2, 130, 32)
    assert need > 0
    out = torch.empty(130, 32, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(2, 32, 128, 128, device="cuda")
    with pytest.raises(ValueError):
        K.gdn_prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                      x.scale, out, ns, workspace=torch.empty(need - 1024, dtype=torch.uint8,
                                                             device="cuda"))
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    K.gdn_prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale,
                  out, ns, workspace=ws)
    ro, rs = O.prefill_chunked(*(t.cpu() for t in (x.q, x.k, x.v, x.state, x.A_log, x.a,
                                                  x.dt_bias, x.b, x.cu_seqlens)), x.scale)
    assert_prefill_close(out.cpu(), ns.cpu(), ro, rs)


@pytest.mark.parametrize("T,with_state,in_place", [(8192, True, True), (8192, False, False),
                                                    (1500, True, False), (24000, True, True)])
def test_one_sequence_pieces_bitwise(T, with_state, in_place):
    """One sequence runs in overlapping pieces of its chunks (the prep of a piece
    overlaps the previous piece's chain); the same sequence followed by an empty
    one runs in a single piece.  Every chunk computes the same products from the
    same tiles, so outputs and the final state agree bit for bit."""
    x = W.make_prefill_inputs([T], seed=21, with_state=with_state)
    dev = [to_dev(t) for t in (x.q, x.k, x.v, x.A_log, x.a, x.dt_bias, x.b)]
    q, k, v, A_log, a, dt_bias, b = dev
    st1 = to_dev(x.state).clone() if with_state else None
    o1, s1 = K.prefill(q, k, v, st1, A_log, a, dt_bias, b, to_dev(x.cu_seqlens), x.scale,
                       in_place=in_place)
    # the same tokens as sequence 0 of two, the second empty
    cu2 = torch.tensor([0, T, T], dtype=x.cu_seqlens.dtype, device="cuda")
    st2 = None
    if with_state:
        st2 = torch.cat([to_dev(x.state), torch.zeros_like(to_dev(x.state))]).contiguous()
    o2, s2 = K.prefill(q, k, v, st2, A_log, a, dt_bias, b, cu2, x.scale, in_place=in_place)
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
    assert torch.equal(o1, o2)
    assert torch.equal(s1[0], s2[0])
    # and both are the recurrence (the oracle check is kept to the short case)
    if T <= 1500:
        ro, rs = _oracle(x)
        assert_prefill_close(o1.cpu(), s1.cpu(), ro, rs)


def test_wide_chain_matches_per_sequence_calls():
    """Three or more sequences run one 128-column chain CTA per (sequence, head);
    a single sequence runs 64-column CTAs (and, long enough, in pieces).  The
    same chunks give the same bits either way."""
    lengths = [700, 4000, 1, 2500]
    x = W.make_prefill_inputs(lengths, seed=31)
    d = {n: to_dev(getattr(x, n)) for n in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")}
    out, ns = K.prefill(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                        d["b"], to_dev(x.cu_seqlens), x.scale)
    lo = 0
    for i, n in enumerate(lengths):
        cu = torch.tensor([0, n], dtype=torch.int32, device="cuda")
        o1, s1 = K.prefill(d["q"][lo:lo + n], d["k"][lo:lo + n], d["v"][lo:lo + n],
                           d["state"][i:i + 1].contiguous(), d["A_log"], d["a"][lo:lo + n],
                           d["dt_bias"], d["b"][lo:lo + n], cu, x.scale)
        assert torch.equal(o1, out[lo:lo + n]), i
        assert torch.equal(s1[0], ns[i]), i
        lo += n
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
    ro, rs = _oracle(x)
    assert_prefill_close(out.cpu(), ns.cpu(), ro, rs)


def test_unordered_cu_seqlens_flagged_and_bounded():
    """cu_seqlens whose entries are each in range but not ordered ([0, T, 0, T])
    describe overlapping sequences with more chunks than the table holds.  The
    split path sets the bad-seqlens status bit, treats every sequence as empty
    (each final state is its initial state) and writes nothing past its
    workspace; a descending pair alone is flagged too."""
    T = 1000
    x = W.make_prefill_inputs([T], seed=41, device="cuda")
    cu = torch.tensor([0, T, 0, T], dtype=torch.int32, device="cuda")
    state = torch.randn(3, 32, 128, 128, device="cuda") * 0.02
    need = K.prefill_workspace_bytes(3, T, 32)
    guard = 1 << 20
    buf = torch.full((need + guard,), 0x5A, dtype=torch.uint8, device="cuda")
    out = torch.zeros(T, 32, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty_like(state)
    K.gdn_prefill(x.q, x.k, x.v, state, x.A_log, x.a, x.dt_bias, x.b, cu, x.scale, out, ns,
                  workspace=buf[:need])
    torch.cuda.synchronize()
    status = _lib.device_status(torch.cuda.current_device())
    assert status & _lib.STATUS_BAD_SEQLENS
    assert status & ~_lib.STATUS_BAD_SEQLENS == 0
    assert torch.all(buf[need:] == 0x5A)
    assert torch.equal(ns, state)
    assert torch.count_nonzero(out) == 0
    # a descending pair within the table's capacity: flagged, the others still run
    cu2 = torch.tensor([0, 50, 20, 100], dtype=torch.int64, device="cuda")
    out2 = torch.empty(100, 32, 128, dtype=torch.bfloat16, device="cuda")
    x2 = W.make_prefill_inputs([100], seed=42, device="cuda")
    ns2 = torch.empty(3, 32, 128, 128, device="cuda")
    K.gdn_prefill(x2.q, x2.k, x2.v, None, x2.A_log, x2.a, x2.dt_bias, x2.b, cu2, x2.scale, out2,
                  ns2)
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == _lib.STATUS_BAD_SEQLENS
    assert torch.count_nonzero(ns2[1]) == 0


# The 1 GiB ring holds 668 record rows at qk16_v32: one sequence runs in
# windows of 334 chunks, several sequences in windows of 668.
RING_CASES = [
    ([150, 0, 64, 33], True, False),       # records fit the ring: one window
    ([8192], False, False),                # fits: the one-sequence pieces path
    ([50000], False, False),               # one sequence over three ring windows
    ([60000], True, True),                 # in place, three windows
    ([20000, 0, 15000, 12000, 1], True, False),   # windows that span sequence boundaries
    ([9000] * 6 + [300, 0, 2], True, False),      # sequence-major windows (short sequences)
    ([50000, 45000, 1000], True, False),          # long sequences: one interleaved group
]


@pytest.mark.parametrize("lengths,with_state,in_place", RING_CASES)
def test_ring_path_bitwise_equal_to_workspace(lengths, with_state, in_place):
    """gdn_b200_prefill works in the library's static record ring (no
    allocation), in windows of chunks when the records do not all fit.  Every
    chunk computes the same products from the same tiles as with a caller
    workspace, and the state crosses window boundaries in fp32, so the results
    are bit-identical."""
    x = W.make_prefill_inputs(lengths, seed=51, device="cuda", with_state=with_state)
    st1 = x.state.clone() if with_state else None
    st2 = x.state.clone() if with_state else None
    o1, s1 = K.prefill(x.q, x.k, x.v, st1, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale,
                       in_place=in_place, path="ring")
    o2, s2 = K.prefill(x.q, x.k, x.v, st2, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale,
                       in_place=in_place, path="split")
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
    assert torch.equal(o1, o2)
    assert torch.equal(s1, s2)


def test_ring_path_matches_oracle_over_windows():
    """Two ring windows (a 44,000-token sequence after a short one: 692 chunks
    against 668 record rows) against the fp32 oracle."""
    lengths = [100, 44000]
    x = W.make_prefill_inputs(lengths, seed=52)
    out, ns = _run(x, "ring")
    ro, rs = _oracle(x)
    assert_prefill_close(out, ns, ro, rs, lengths)


def test_ring_path_calls_on_two_streams():
    """Calls on two streams share the ring; the second call's stream waits for
    the first call's kernels on the GPU, so both results are right."""
    xa = W.make_prefill_inputs([7000], seed=53, device="cuda")
    xb = W.make_prefill_inputs([2000, 4500], seed=54, device="cuda")
    ref = [K.prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale,
                     path="split") for x in (xa, xb)]
    torch.cuda.synchronize()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    res = []
    for x, s in ((xa, s1), (xb, s2)):
        with torch.cuda.stream(s):
            res.append(K.prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                                 x.cu_seqlens, x.scale, path="ring"))
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
    for (o, s), (ro, rs) in zip(res, ref):
        assert torch.equal(o, ro)
        assert torch.equal(s, rs)


def test_ring_path_sequence_major_windows():
    """Several sequences whose records overflow the ring but are short next to a
    window: the table stays sequence-major and each window holds whole
    sequences (one split at each window edge).  Bit-identical to the workspace
    path, and within tolerance of the oracle."""
    lengths = [2100, 9000, 1, 7500, 12300, 0, 5400, 1920, 15000]   # 840 chunks, 668 rows
    x = W.make_prefill_inputs(lengths, seed=55)
    o1, s1 = _run(x, "ring")
    o2, s2 = _run(x, "split")
    assert torch.equal(o1, o2)
    assert torch.equal(s1, s2)
    ro, rs = _oracle(x)
    assert_prefill_close(o1, s1, ro, rs, lengths)


def test_ring_path_interleaved_groups():
    """Sequences long next to a window (17-30K tokens, 1,314 chunks
    against 668 record rows): the chunk table interleaves them in rounds, so
    that each ring window holds a run of chunks of every member.
    Bit-identical to the workspace path, and within tolerance of the oracle."""
    lengths = [30000, 29000, 8000, 0, 17000]
    x = W.make_prefill_inputs(lengths, seed=56)
    o1, s1 = _run(x, "ring")
    o2, s2 = _run(x, "split")
    assert torch.equal(o1, o2)
    assert torch.equal(s1, s2)
    ro, rs = _oracle(x)
    assert_prefill_close(o1, s1, ro, rs, lengths)


def test_configs4_scale_ring_equals_workspace_and_oracle_on_samples():
    """64 sequences of U[1024, 16384] tokens (about 552K, the multi-GPU
    benchmark's batch) in one packed call: the ring path (windows over the 1 GiB
    ring) equals the workspace path bit for bit, and two of the packed
    sequences equal the fp32 oracle run on those sequences alone (sequences
    are independent), to the prefill tolerance."""
    lengths = W.varlen_lengths(64, 1024, 16384, seed=4)
    x = W.make_prefill_inputs(lengths, seed=9, device="cuda")
    args = (x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale)
    o1, s1 = K.prefill(*args, path="split")
    o2, s2 = K.prefill(*args, path="ring")
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    cu = x.cu_seqlens.cpu().tolist()
    for n in (0, 37):
        lo, hi = cu[n], cu[n + 1]
        sl = lambda t: t[lo:hi].cpu()
        ro, rs = O.prefill_chunked(sl(x.q), sl(x.k), sl(x.v), x.state[n:n + 1].cpu(),
                                   x.A_log.cpu(), sl(x.a), x.dt_bias.cpu(), sl(x.b),
                                   torch.tensor([0, hi - lo], dtype=torch.int32), x.scale)
        assert_prefill_close(o1[lo:hi].cpu(), s1[n:n + 1].cpu(), ro, rs)


def test_long_sequence_ring_windows_equal_workspace():
    """One 65,536-token sequence (1,025 chunks over 334-chunk ring windows)
    equals the workspace path (eight overlapping pieces) bit for bit, in
    place, from a random initial state."""
    x = W.make_prefill_inputs([65536], seed=10, device="cuda", with_state=True)
    args = (x.q, x.k, x.v, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale)
    st1, st2 = x.state.clone(), x.state.clone()
    o1, s1 = K.prefill(x.q, x.k, x.v, st1, *args[3:], in_place=True, path="split")
    o2, s2 = K.prefill(x.q, x.k, x.v, st2, *args[3:], in_place=True, path="ring")
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def test_thousands_of_short_sequences():
    """3,000 sequences of 0-40 tokens (many empty): the chunk table is filled
    over several passes of its threads, each position's owner found among
    sequences that share a first chunk position.  Ring and workspace paths
    agree bit for bit, and sampled sequences match the oracle run on them
    alone."""
    g = torch.Generator().manual_seed(21)
    lengths = torch.randint(0, 41, (3000,), generator=g).tolist()
    lengths[0], lengths[-1] = 0, 0
    x = W.make_prefill_inputs(lengths, seed=22, device="cuda", h_qk=1, h_v=2)
    args = (x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale)
    o1, s1 = K.prefill(*args, path="split")
    o2, s2 = K.prefill(*args, path="ring")
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    cu = x.cu_seqlens.cpu().tolist()
    for n in (0, 1, 1500, 2998, 2999):
        lo, hi = cu[n], cu[n + 1]
        sl = lambda t: t[lo:hi].cpu()
        ro, rs = O.prefill_chunked(sl(x.q), sl(x.k), sl(x.v), x.state[n:n + 1].cpu(),
                                   x.A_log.cpu(), sl(x.a), x.dt_bias.cpu(), sl(x.b),
                                   torch.tensor([0, hi - lo], dtype=torch.int32), x.scale)
        assert_prefill_close(o1[lo:hi].cpu(), s1[n:n + 1].cpu(), ro, rs, [hi - lo])
