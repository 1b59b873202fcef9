"""Context-parallel prefill with the CUDA kernels: the affine combine kernel,
and the full protocol emulated on one GPU (every virtual rank's passes run in
turn; the all-gather becomes a list), checked against the fp32 oracle of the
whole sequence and against the single-call prefill."""

import pytest
import torch

from helpers import assert_prefill_close
from gdn_kernel_b200 import context_parallel as CP, kernel as K, workloads as W
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu


def test_state_affine_kernel_matches_fp32_matmul():
    g = torch.Generator(device="cuda").manual_seed(3)
    s, m, n = (torch.randn(5, 128, 128, device="cuda", generator=g) for _ in range(3))
    out = K.state_affine(s, m, n)
    ref = torch.matmul(s.double(), m.double()) + n.double()
    torch.testing.assert_close(out.double(), ref, atol=1e-4, rtol=1e-5)
    # no state: out = offset; out may alias the offset
    torch.testing.assert_close(K.state_affine(None, None, n), n, atol=0, rtol=0)
    n2 = n.clone()
    K.state_affine(s, m, n2, out=n2)
    torch.testing.assert_close(n2.double(), ref, atol=1e-4, rtol=1e-5)


@pytest.mark.parametrize("lengths", [[300, 0, 64, 1, 129], [300, 129]])
def test_prepare_then_recur_equals_prefill(lengths):
    """The two stages as separate calls give the single call's results bitwise;
    a null V equals an all-zero V; a null output changes nothing else.  Five
    sequences run 128-column chain CTAs (2 x 5 x 32 > SMs), two run 64-column
    ones."""
    x = W.make_prefill_inputs(lengths, seed=17, device="cuda")
    T, N = sum(lengths), len(lengths)
    ws = torch.empty(K.prefill_workspace_bytes(N, T, 32), dtype=torch.uint8, device="cuda")
    K.gdn_prefill_prepare(x.q, x.k, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, ws)
    out = torch.empty(T, 32, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty_like(x.state)
    K.gdn_prefill_recur(x.k, x.v, x.state, x.scale, out, ns, N, 32, ws)
    ro, rs = K.prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                       x.scale)
    assert torch.equal(out, ro) and torch.equal(ns, rs)
    # the workspace is read only: a second recurrence from it gives the same again
    ns2 = torch.empty_like(ns)
    K.gdn_prefill_recur(x.k, x.v, x.state, x.scale, None, ns2, N, 32, ws)
    assert torch.equal(ns2, rs)
    zo, zs = (torch.empty_like(out), torch.empty_like(ns))
    K.gdn_prefill_recur(x.k, torch.zeros_like(x.v), x.state, x.scale, zo, zs, N, 32, ws)
    no = torch.full_like(out, 7.0)
    nz = torch.empty_like(ns)
    K.gdn_prefill_recur(x.k, None, x.state, x.scale, no, nz, N, 32, ws)
    torch.cuda.synchronize()
    assert torch.equal(nz, zs) and torch.equal(no, zo)


def test_kernel_segment_maps_match_function_maps():
    """Pass A through prepare + two concurrent recurrences equals pass A
    through one packed prefill call, and both are the segment's affine map."""
    x = W.make_prefill_inputs([700], seed=23, device="cuda")
    args = (x.q, x.k, x.v, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    seg = CP._KernelSegment(*args)
    m1, n1 = seg.pass_a()
    m2, n2, o2, q2 = CP.segment_pass_a(*args)
    torch.cuda.synchronize()
    torch.testing.assert_close(m1, m2, atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(n1, n2, atol=1e-6, rtol=1e-5)
    # the same kernels on the same records: the outputs agree bitwise
    assert torch.equal(seg.out0, o2) and torch.equal(seg.qt, q2)
    s0 = x.state[0]
    _, ref = K.prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                       x.scale)
    from helpers import rel_fro
    err = rel_fro((s0 @ m1 + n1)[None].cpu(), ref.cpu())
    assert err.max().item() < 1e-2
    # outputs from s0 by the correction equal a run from s0 to the prefill tolerance
    ref_o = K.prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                      x.scale)[0]
    out, end = seg.finish(s0, CP._default_affine())
    torch.cuda.synchronize()
    assert_prefill_close(out.cpu(), end[None].cpu(), ref_o.cpu(), ref.cpu())


def _emulate(x, world, first_weight=1.0):
    """cp_prefill's steps for every virtual rank in turn: rank 0 runs its
    segment outright, the others run pass A; then each folds the maps before it
    and finishes (output correction and end state)."""
    T = x.q.shape[0]
    segs = CP.cp_segments(T, world, first_weight)
    maps, runs = [], []
    for r, (lo, hi) in enumerate(segs):
        sl = lambda t: t[lo:hi].contiguous()
        args = (sl(x.q), sl(x.k), sl(x.v))
        gates = (x.A_log, sl(x.a), x.dt_bias, sl(x.b), x.scale)
        if hi == lo:
            maps.append((torch.eye(128, device="cuda").expand(32, 128, 128).contiguous(),
                         torch.zeros(32, 128, 128, device="cuda")))
            runs.append(None)
        elif r == 0:
            direct = CP._run_direct(None, *args, x.state[0], *gates)
            maps.append((torch.zeros(32, 128, 128, device="cuda"), direct[1]))
            runs.append(direct)
        else:
            seg = CP._KernelSegment(*args, *gates)
            maps.append(seg.pass_a())
            runs.append(seg)
    outs, end = [], None
    for r, run in enumerate(runs):
        s_in = CP.fold_states(x.state[0], maps[:r])
        if run is None:
            end = s_in
        elif r == 0:
            outs.append(run[0])
            end = run[1]
        else:
            o, end = run.finish(s_in, CP._default_affine())
            outs.append(o)
    return torch.cat(outs), end


@pytest.mark.parametrize("T,world,w", [(4096, 2, 1.0), (8192, 4, 1.3), (1000, 3, 1.0),
                                       (100, 3, 1.0), (20000, 2, 1.3)])
def test_cp_emulated_matches_whole_sequence(T, world, w):
    x = W.make_prefill_inputs([T], seed=200 + world, device="cuda")
    out, end = _emulate(x, world, w)
    torch.cuda.synchronize()
    c = {n: getattr(x, n).cpu() for n in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b",
                                          "cu_seqlens")}
    ro, rs = O.prefill_chunked(c["q"], c["k"], c["v"], c["state"], c["A_log"], c["a"],
                               c["dt_bias"], c["b"], c["cu_seqlens"], x.scale)
    assert_prefill_close(out.cpu(), end[None].cpu(), ro, rs)
    mo, ms = K.prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                       x.scale)
    assert_prefill_close(out.cpu(), end[None].cpu(), mo.cpu(), ms.cpu())
