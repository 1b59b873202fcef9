"""Context-parallel prefill: one long sequence split across the GPUs of a node.

A single sequence's chunk chain is sequential, so the sequence-sharded driver
(``sharding``) cannot spread it.  This module splits its tokens into contiguous
64-token-aligned segments, one per rank, and removes the dependency between
segments with the affine structure of the recurrence.  Over a segment every
state row evolves by the same affine map, ``S_end = S_0 @ M + N`` (row = v,
k-last layout; the per-chunk map is ``e^{gamma_last} I - W^T K_decay``, ref
solution/cuda/kernel_prefill.cu:286-293), so each rank

1. prepares its segment once (chunk table and per-chunk records, which do not
   depend on V or on the state) and runs pass A, two recurrences over the
   prepared segment on two streams: the real V from a zero state, whose
   outputs are ``O_0`` and whose final state is the offset N, and V = 0 from
   the identity, whose final state is the transfer M and whose outputs are
   ``q~_t = M_t q_t`` (scaled), with M_t the transfer up to token t;
2. all-gathers (M, N) across the ranks: 2 x H_v x 64 KiB per rank, the only
   exchange, issued once per call;
3. folds the maps of the segments before it into its true initial state,
   ``S_g = S_{g-1} @ M_{g-1} + N_{g-1}`` (``gdn_b200_state_affine``), starting
   from the sequence's initial state;
4. finishes without another recurrence.  The outputs are affine in the initial
   state like the state is, ``o_t = S_g q~_t + O_0[t]``, so one batched GEMM
   per head adds ``q~ S_g^T`` to ``O_0`` in place, and the segment's end state
   is ``S_g @ M + N``.

Rank 0 knows its initial state, so it runs its segment as one ordinary prefill
(the one-sequence pieces path) and reports the map (M, N) = (0, S_end):
folding it into any state gives its true end state.  Every other rank runs its
segment's chain once, and all ranks' chains run at the same time: the
per-head sequential depth drops from T/64 chunks to about T/(64 G).  A rank
other than 0 spends more per token than rank 0 (the records are prepared
before its chain starts, two recurrences share its SMs, and the correction
reads its outputs again), so ``cp_segments`` can give rank 0 a larger share
(``first_segment_weight``).  The reference is single-GPU (its harness requests
one B200, ref scripts/run_modal.py:36); this is the split its recurrence
admits.

The compute is a parameter: ``prefill_fn`` (a full prefill with the reference
``kernel`` signature) switches to the generic form of passes A and B through
that function, which is how the host logic runs in CPU tests with the fp32
oracle standing in for the CUDA kernels.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch

CHUNK = 64


# Per-token cost of a rank other than 0 (prepare, then two concurrent
# recurrences, then the output correction) over that of rank 0's direct
# one-sequence prefill, measured on B200 at qk16_v32 for 65,536 tokens: 1.3 was
# the best of a sweep at 2 ranks; at 4 ranks (1.3 given) rank 0 ran 38.9 us per
# 1K tokens and the others 58.4, a ratio of 1.5; at 8 ranks (1.5 given) 50.8
# against about 91, a ratio of 1.8.  The fixed costs of the others (gather,
# fold, correction) weigh more on shorter segments.
FIRST_SEGMENT_WEIGHT = 1.3


def first_segment_weight(world: int) -> float:
    """The ``first_weight`` of ``cp_segments`` for ``world`` ranks."""
    if world <= 1:
        return 1.0
    if world == 2:
        return FIRST_SEGMENT_WEIGHT
    return 1.5 if world <= 4 else 1.8


def cp_segments(total_tokens: int, world: int, first_weight: float = 1.0
                ) -> List[Tuple[int, int]]:
    """Contiguous [lo, hi) token segments, one per rank, on 64-token chunk
    boundaries.  Rank 0 gets ``first_weight`` times the chunks of each other
    rank (rounded); the others' chunk counts differ by at most one.  A rank may
    get an empty segment when there are fewer chunks than ranks."""
    if world < 1 or total_tokens < 0 or first_weight <= 0:
        raise ValueError("world must be >= 1, total_tokens >= 0 and first_weight > 0")
    nchunks = (total_tokens + CHUNK - 1) // CHUNK
    if world == 1:
        counts = [nchunks]
    elif first_weight == 1.0:
        base, extra = divmod(nchunks, world)
        counts = [base + (1 if r < extra else 0) for r in range(world)]
    else:
        first = min(nchunks, int(round(nchunks * first_weight / (first_weight + world - 1))))
        base, extra = divmod(nchunks - first, world - 1)
        counts = [first] + [base + (1 if r < extra else 0) for r in range(world - 1)]
    out, c = [], 0
    for n in counts:
        lo, hi = min(c * CHUNK, total_tokens), min((c + n) * CHUNK, total_tokens)
        out.append((lo, hi))
        c += n
    return out


def _default_prefill():
    from .kernel import gdn_prefill
    return gdn_prefill


def _default_affine():
    from .kernel import state_affine
    return lambda s, m, n: state_affine(s, m, n)


def segment_pass_a(q, k, v, A_log, a, dt_bias, b, scale,
                   prefill_fn: Optional[Callable] = None):
    """Pass A through one packed prefill call (the segment twice: real V from a
    zero state, V = 0 from the identity).  Returns ``(M, N, O_0, Q~)``: the
    segment's affine map, each [H_v, 128, 128] fp32, and the two runs' outputs
    [T, H_v, 128] bf16, such that a run from any initial state S_0 ends at
    ``S_0 @ M + N`` and outputs ``O_0[t] + S_0 @ Q~[t]`` per head."""
    prefill_fn = prefill_fn or _default_prefill()
    T, _, D = q.shape
    h_v = v.shape[1]
    dev = q.device
    cat = lambda x: torch.cat([x, x], dim=0)
    v2 = torch.cat([v, torch.zeros_like(v)], dim=0)
    cu = torch.tensor([0, T, 2 * T], dtype=torch.int32, device=dev)
    state = torch.zeros(2, h_v, D, D, dtype=torch.float32, device=dev)
    state[1] = torch.eye(D, dtype=torch.float32, device=dev)
    out = torch.empty(2 * T, h_v, D, dtype=torch.bfloat16, device=dev)
    ns = torch.empty(2, h_v, D, D, dtype=torch.float32, device=dev)
    prefill_fn(cat(q), cat(k), v2, state, A_log, cat(a), dt_bias, cat(b), cu, scale, out, ns)
    return ns[1].contiguous(), ns[0].contiguous(), out[:T], out[T:]


def segment_affine(q, k, v, A_log, a, dt_bias, b, scale,
                   prefill_fn: Optional[Callable] = None):
    """(M, N), each [H_v, 128, 128] fp32, such that a run of this segment from
    any initial state S_0 ends at ``S_0 @ M + N``."""
    m, n, _, _ = segment_pass_a(q, k, v, A_log, a, dt_bias, b, scale, prefill_fn)
    return m, n


def correct_outputs(out0: torch.Tensor, qt: torch.Tensor, s_in: torch.Tensor) -> torch.Tensor:
    """``out0[t, h] += s_in[h] @ qt[t, h]`` in place, for all tokens and heads:
    the outputs of a run from the initial state ``s_in`` [H_v, 128, 128] out of
    pass A's two output sets [T, H_v, 128].  On CUDA this is one strided,
    batched bf16 GEMM (fp32 accumulation, one rounding) over the token-major
    views; elsewhere an fp32 product."""
    if out0.shape[0] == 0:
        return out0
    if out0.is_cuda:
        s_t = s_in.to(out0.dtype).transpose(1, 2)               # [H, K, V]
        out0.permute(1, 0, 2).baddbmm_(qt.permute(1, 0, 2), s_t)
    else:
        corr = torch.einsum("thk,hvk->thv", qt.float(), s_in.float())
        out0.copy_((out0.float() + corr).to(out0.dtype))
    return out0


def fold_states(state0: Optional[torch.Tensor], maps, affine_fn: Optional[Callable] = None):
    """Apply the affine maps ``[(M_0, N_0), (M_1, N_1), ...]`` in order to the
    initial state (None = zero); returns the state after the last one."""
    affine_fn = affine_fn or _default_affine()
    s = state0
    for m, n in maps:
        s = affine_fn(s, m, n)
    return s


class _KernelSegment:
    """Pass A with the CUDA kernels: one prepare, two concurrent recurrences
    over the prepared records, both with outputs."""

    def __init__(self, q, k, v, A_log, a, dt_bias, b, scale):
        from . import kernel as K
        self.K, self.k, self.v, self.scale = K, k, v, scale
        T, _, D = q.shape
        self.h_v, self.D = v.shape[1], D
        cu = torch.tensor([0, T], dtype=torch.int32, device=q.device)
        self.ws = torch.empty(K.prefill_workspace_bytes(1, T, self.h_v), dtype=torch.uint8,
                              device=q.device)
        K.gdn_prefill_prepare(q, k, A_log, a, dt_bias, b, cu, self.ws)

    def pass_a(self):
        K, dev, h_v, D = self.K, self.k.device, self.h_v, self.D
        T = self.k.shape[0]
        n = torch.empty(1, h_v, D, D, dtype=torch.float32, device=dev)
        m = torch.empty(1, h_v, D, D, dtype=torch.float32, device=dev)
        self.out0 = torch.empty(T, h_v, D, dtype=torch.bfloat16, device=dev)
        self.qt = torch.empty(T, h_v, D, dtype=torch.bfloat16, device=dev)
        eye = torch.eye(D, dtype=torch.float32, device=dev).expand(1, h_v, D, D).contiguous()
        main = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(main)
        K.gdn_prefill_recur(self.k, self.v, None, self.scale, self.out0, n, 1, h_v, self.ws)
        with torch.cuda.stream(side):
            K.gdn_prefill_recur(self.k, None, eye, self.scale, self.qt, m, 1, h_v, self.ws)
        main.wait_stream(side)
        self.m, self.n = m[0], n[0]
        return self.m, self.n

    def finish(self, state, affine_fn):
        out = correct_outputs(self.out0, self.qt, state)
        return out, affine_fn(state, self.m, self.n)


class _FunctionSegment:
    """Pass A through a full prefill function (reference signature)."""

    def __init__(self, prefill_fn, q, k, v, A_log, a, dt_bias, b, scale):
        self.fn = prefill_fn
        self.args = (q, k, v, A_log, a, dt_bias, b, scale)

    def pass_a(self):
        self.m, self.n, self.out0, self.qt = segment_pass_a(*self.args, prefill_fn=self.fn)
        return self.m, self.n

    def finish(self, state, affine_fn):
        out = correct_outputs(self.out0, self.qt, state)
        return out, affine_fn(state, self.m, self.n)


def cp_prefill(rank: int, world: int, q, k, v, state, A_log, a, dt_bias, b, scale, *,
               prefill_fn: Optional[Callable] = None, affine_fn: Optional[Callable] = None,
               group=None):
    """Context-parallel prefill of one sequence.

    Rank ``rank`` passes its segment's packed inputs (q, k [T_g, H_qk, 128],
    v [T_g, H_v, 128], a, b [T_g, H_v]; segments from ``cp_segments``) and the
    sequence's initial state ``state`` [H_v, 128, 128] fp32 (or None) on every
    rank.  Returns ``(output [T_g, H_v, 128] bf16, end_state [H_v, 128, 128])``;
    ``end_state`` on the last rank is the sequence's final state.  Collective:
    one all-gather of this rank's (M, N) over ``group``.
    """
    import torch.distributed as dist

    T, _, D = q.shape
    h_v = v.shape[1]
    dev = q.device
    seg, direct = None, None
    if T > 0 and rank == 0:
        # the sequence's own initial state: run the segment outright
        direct = _run_direct(prefill_fn, q, k, v, state, A_log, a, dt_bias, b, scale)
        m = torch.zeros(h_v, D, D, dtype=torch.float32, device=dev)
        n = direct[1]
    elif T > 0:
        seg = (_FunctionSegment(prefill_fn, q, k, v, A_log, a, dt_bias, b, scale)
               if prefill_fn is not None
               else _KernelSegment(q, k, v, A_log, a, dt_bias, b, scale))
        m, n = seg.pass_a()
    else:   # an empty segment maps every state to itself
        m = torch.eye(D, dtype=torch.float32, device=dev).expand(h_v, D, D).contiguous()
        n = torch.zeros(h_v, D, D, dtype=torch.float32, device=dev)
    mine = torch.stack([m, n])
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine, group=group)
    if direct is not None:
        return direct
    s_in = fold_states(state, [(p[0], p[1]) for p in parts[:rank]], affine_fn)
    if s_in is None:
        s_in = torch.zeros(h_v, D, D, dtype=torch.float32, device=dev)
    if seg is None:
        return torch.empty(0, h_v, D, dtype=torch.bfloat16, device=dev), s_in.clone()
    return seg.finish(s_in, affine_fn or _default_affine())


def _run_direct(prefill_fn, q, k, v, state, A_log, a, dt_bias, b, scale):
    """One segment as an ordinary one-sequence prefill from ``state`` (None =
    zero): ``(output, end_state)``."""
    if prefill_fn is None:
        from .kernel import gdn_prefill
        prefill_fn = gdn_prefill
    T, _, D = q.shape
    h_v = v.shape[1]
    out = torch.empty(T, h_v, D, dtype=torch.bfloat16, device=q.device)
    ns = torch.empty(1, h_v, D, D, dtype=torch.float32, device=q.device)
    cu = torch.tensor([0, T], dtype=torch.int32, device=q.device)
    st = None if state is None else state.unsqueeze(0).contiguous()
    prefill_fn(q, k, v, st, A_log, a, dt_bias, b, cu, scale, out, ns)
    return out, ns[0]
