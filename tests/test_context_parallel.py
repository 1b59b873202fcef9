"""Context-parallel prefill host logic on CPU: segment split, the affine map of
a segment, and the full protocol over gloo ranks with the fp32 oracle standing
in for the CUDA kernels."""

import pytest
import torch

import dist_workers as DW
from gdn_kernel_b200 import context_parallel as CP, sharding as S, workloads as W
from oracle import gdn_oracle as O


@pytest.mark.parametrize("T,world", [(0, 2), (1, 3), (333, 2), (640, 4), (8192, 8), (100, 8)])
def test_segments_are_chunk_aligned_and_cover(T, world):
    segs = CP.cp_segments(T, world)
    assert len(segs) == world
    assert segs[0][0] == 0 and segs[-1][1] == T
    for (lo, hi), (lo2, _) in zip(segs, segs[1:]):
        assert hi == lo2 and lo <= hi
    for lo, hi in segs[:-1]:
        assert (lo % 64 == 0 or lo == T) and (hi % 64 == 0 or hi == T)
    chunks = [(hi - lo + 63) // 64 for lo, hi in segs]
    assert max(chunks) - min(chunks) <= 1


@pytest.mark.parametrize("T,world,w", [(65536, 2, 1.3), (65536, 8, 1.3), (640, 4, 2.0),
                                       (100, 3, 1.3), (0, 2, 1.3), (8192, 1, 1.3)])
def test_weighted_segments(T, world, w):
    segs = CP.cp_segments(T, world, first_weight=w)
    assert len(segs) == world and segs[0][0] == 0 and segs[-1][1] == T
    for (lo, hi), (lo2, _) in zip(segs, segs[1:]):
        assert hi == lo2 and lo <= hi and (hi % 64 == 0 or hi == T)
    chunks = [(hi - lo + 63) // 64 for lo, hi in segs]
    assert max(chunks[1:] or [0]) - min(chunks[1:] or [0]) <= 1
    nch = (T + 63) // 64
    if world > 1:
        assert abs(chunks[0] - nch * w / (w + world - 1)) <= 1


def test_first_segment_weight_by_world():
    assert CP.first_segment_weight(1) == 1.0
    assert CP.first_segment_weight(2) == CP.FIRST_SEGMENT_WEIGHT
    assert CP.first_segment_weight(4) == 1.5 and CP.first_segment_weight(8) == 1.8
    segs = CP.cp_segments(65536, 4, CP.first_segment_weight(4))
    assert segs[0] == (0, 21824) and all(hi - lo in (14592, 14528) for lo, hi in segs[1:])


def test_outputs_are_affine_in_the_initial_state():
    """Pass A's two output sets give the outputs of a run from any initial
    state: O_0 + S_0 Q~ per head (oracle, fp32 runs, bf16 outputs)."""
    x = W.make_prefill_inputs([150], seed=8, h_qk=1, h_v=2)
    m, n, out0, qt = CP.segment_pass_a(x.q, x.k, x.v, x.A_log, x.a, x.dt_bias, x.b, x.scale,
                                       prefill_fn=DW.oracle_prefill_dps)
    for seed in (1, 2):
        s0 = torch.randn(2, 128, 128, generator=torch.Generator().manual_seed(seed)) * 0.05
        ref_o, ref_s = O.prefill_chunked(x.q, x.k, x.v, s0[None], x.A_log, x.a, x.dt_bias, x.b,
                                         x.cu_seqlens, x.scale)
        out = CP.correct_outputs(out0.clone(), qt, s0)
        torch.testing.assert_close(out.float(), ref_o.float(), atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(s0 @ m + n, ref_s[0], atol=2e-5, rtol=1e-4)


def test_segment_affine_map_is_exact():
    """A run from any initial state ends at S0 @ M + N (oracle, fp32)."""
    x = W.make_prefill_inputs([150], seed=8, h_qk=1, h_v=2)
    m, n = CP.segment_affine(x.q, x.k, x.v, x.A_log, x.a, x.dt_bias, x.b, x.scale,
                             prefill_fn=DW.oracle_prefill_dps)
    for seed in (1, 2):
        s0 = torch.randn(2, 128, 128, generator=torch.Generator().manual_seed(seed)) * 0.05
        _, ref = O.prefill_chunked(x.q, x.k, x.v, s0[None], x.A_log, x.a, x.dt_bias, x.b,
                                   x.cu_seqlens, x.scale)
        torch.testing.assert_close(s0 @ m + n, ref[0], atol=2e-5, rtol=1e-4)


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_cp_protocol_over_gloo_equals_whole_sequence(world):
    res = S.launch_workers(DW.cp_worker, world, timeout_s=300)
    assert all(r.ok for r in res), [r.error for r in res]
    out, end = res[0].value
    x = DW._cp_inputs()
    ro, rs = O.prefill_chunked(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                               x.cu_seqlens, x.scale)
    torch.testing.assert_close(out.float(), ro.float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(end, rs[0], atol=2e-5, rtol=1e-4)
