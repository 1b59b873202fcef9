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
   prepared segment on two streams: the real V from a zero state (final state
   = the offset N) and V = 0 from the identity (final state = the transfer M);
2. all-gathers (M, N) across the ranks: 2 x H_v x 64 KiB per rank, the only
   exchange, issued once per call;
3. folds the maps of the segments before it into its true initial state,
   ``S_g = S_{g-1} @ M_{g-1} + N_{g-1}`` (``gdn_b200_state_affine``), starting
   from the sequence's initial state;
4. runs pass B, the recurrence of its segment from ``S_g`` over the same
   prepared records, giving its outputs and the state at its segment's end (on
   the last rank: the sequence's final state).

Two ranks need less.  Rank 0 knows its initial state, so it runs its segment
as one ordinary prefill (the one-sequence pieces path) and reports the map
(M, N) = (0, S_end): folding it into any state gives its true end state.  The
last rank's map is folded by no one, so it only prepares, then waits for the
gather.  Each middle rank prepares T/G tokens once and runs three recurrences
over them (two of them concurrently) instead of the whole chain, and the
per-head sequential depth drops from T/64 chunks to about 2T/(64 G).  The reference is
single-GPU (its harness requests one B200, ref scripts/run_modal.py:36); this
is the split its recurrence admits.

The compute is a parameter: ``prefill_fn`` (a full prefill with the reference
``kernel`` signature) switches to the generic form of passes A and B through
that function, which is how the host logic runs in CPU tests with the fp32
oracle standing in for the CUDA kernels.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch

CHUNK = 64


def cp_segments(total_tokens: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous [lo, hi) token segments, one per rank, on 64-token chunk
    boundaries, with chunk counts differing by at most one (a rank may get an
    empty segment when there are fewer chunks than ranks)."""
    if world < 1 or total_tokens < 0:
        raise ValueError("world must be >= 1 and total_tokens >= 0")
    nchunks = (total_tokens + CHUNK - 1) // CHUNK
    base, extra = divmod(nchunks, world)
    out, c = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
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


def segment_affine(q, k, v, A_log, a, dt_bias, b, scale,
                   prefill_fn: Optional[Callable] = None):
    """Pass A: (M, N), each [H_v, 128, 128] fp32, such that a run of this
    segment from any initial state S_0 ends at ``S_0 @ M + N``."""
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
    return ns[1].contiguous(), ns[0].contiguous()


def fold_states(state0: Optional[torch.Tensor], maps, affine_fn: Optional[Callable] = None):
    """Apply the affine maps ``[(M_0, N_0), (M_1, N_1), ...]`` in order to the
    initial state (None = zero); returns the state after the last one."""
    affine_fn = affine_fn or _default_affine()
    s = state0
    for m, n in maps:
        s = affine_fn(s, m, n)
    return s


class _KernelSegment:
    """Passes A and B with the CUDA kernels: one prepare, three recurrences."""

    def __init__(self, q, k, v, A_log, a, dt_bias, b, scale):
        from . import kernel as K
        self.K, self.k, self.v, self.scale = K, k, v, scale
        T, _, D = q.shape
        self.h_v, self.D = v.shape[1], D
        cu = torch.tensor([0, T], dtype=torch.int32, device=q.device)
        self.ws = torch.empty(K.prefill_workspace_bytes(1, T, self.h_v), dtype=torch.uint8,
                              device=q.device)
        K.gdn_prefill_prepare(q, k, A_log, a, dt_bias, b, cu, self.ws)

    def maps(self):
        K, dev, h_v, D = self.K, self.k.device, self.h_v, self.D
        n = torch.empty(1, h_v, D, D, dtype=torch.float32, device=dev)
        m = torch.empty(1, h_v, D, D, dtype=torch.float32, device=dev)
        eye = torch.eye(D, dtype=torch.float32, device=dev).expand(1, h_v, D, D).contiguous()
        main = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(main)
        K.gdn_prefill_recur(self.k, self.v, None, self.scale, None, n, 1, h_v, self.ws)
        with torch.cuda.stream(side):
            K.gdn_prefill_recur(self.k, None, eye, self.scale, None, m, 1, h_v, self.ws)
        main.wait_stream(side)
        return m[0], n[0]

    def run(self, state):
        K, dev = self.K, self.k.device
        out = torch.empty(self.k.shape[0], self.h_v, self.D, dtype=torch.bfloat16, device=dev)
        ns = torch.empty(1, self.h_v, self.D, self.D, dtype=torch.float32, device=dev)
        K.gdn_prefill_recur(self.k, self.v, state.unsqueeze(0).contiguous(), self.scale, out, ns,
                            1, self.h_v, self.ws)
        return out, ns[0]


class _FunctionSegment:
    """Passes A and B through a full prefill function (reference signature)."""

    def __init__(self, prefill_fn, q, k, v, A_log, a, dt_bias, b, scale):
        self.fn = prefill_fn
        self.args = (q, k, v, A_log, a, dt_bias, b, scale)

    def maps(self):
        return segment_affine(*self.args, prefill_fn=self.fn)

    def run(self, state):
        q, k, v, A_log, a, dt_bias, b, scale = self.args
        T, _, D = q.shape
        h_v = v.shape[1]
        out = torch.empty(T, h_v, D, dtype=torch.bfloat16, device=q.device)
        ns = torch.empty(1, h_v, D, D, dtype=torch.float32, device=q.device)
        cu = torch.tensor([0, T], dtype=torch.int32, device=q.device)
        self.fn(q, k, v, state.unsqueeze(0).contiguous(), A_log, a, dt_bias, b, cu, scale, out,
                ns)
        return out, ns[0]


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
        if rank < world - 1:
            m, n = seg.maps()
        else:   # no later rank folds the last rank's map
            m = torch.zeros(h_v, D, D, dtype=torch.float32, device=dev)
            n = torch.zeros(h_v, D, D, dtype=torch.float32, device=dev)
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
    return seg.run(s_in)


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
