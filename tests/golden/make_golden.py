"""Generate the golden fixtures that pin the CPU oracle.

The reference repository ships no tests or fixtures; its correctness
contract is the contest's definition reference (ref design.md:157-226 for
decode, the packed ``cu_seqlens`` prefill definition of the
``gdn_prefill_*_k_last`` contest definitions).  Those definition functions are
published in flashinfer 0.6.11.post2 as
``flashinfer.trace.templates.gdn._gdn_decode_reference`` and
``_gdn_prefill_reference``; this script runs them on seeded inputs and stores
inputs and outputs under ``tests/golden/``.

One deliberate deviation: for an empty sequence the definition template
leaves the returned state at zero, while the reference CUDA kernel copies the
initial state through (ref solution/cuda/kernel_prefill.cu:61-66).  This
build follows the reference kernel, so the fixture records the copy.

Large cases store outputs in full and the final state as per-row sums, per-row
sums of squares and two complete heads, so the fixtures stay small; their
inputs are regenerated from the seed and checked against stored checksums.

Run from the repository root:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from gdn_kernel_b200 import workloads as W  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def _np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def checksum(t: torch.Tensor) -> np.ndarray:
    f = t.double()
    return np.array([f.sum().item(), (f * f).sum().item()], dtype=np.float64)


def state_summary(s: torch.Tensor) -> dict:
    """Row sums and row sums of squares of a [N, H, V, K] state, plus two heads."""
    return {
        "state_rowsum": s.double().sum(-1).numpy(),
        "state_rowsq": (s.double() ** 2).sum(-1).numpy(),
        "state_head_first": s[0, 0].numpy().copy(),
        "state_head_last": s[-1, -1].numpy().copy(),
    }


def main():
    from flashinfer.trace.templates.gdn import (_gdn_decode_reference,
                                                _gdn_prefill_reference)

    # decode B=4, qk16_v32, 16 consecutive steps from seed 0.
    first, tokens = W.make_decode_run(4, 16, seed=0)
    state = first.state.clone()
    outs = []
    for (q, k, v, a, b) in tokens:
        o, state = _gdn_decode_reference(q, k, v, state, first.A_log, a, first.dt_bias, b,
                                         first.scale)
        outs.append(o)
    rec = {"outputs": _np(torch.stack(outs)),
           "in_state": checksum(first.state), "in_A_log": checksum(first.A_log),
           "in_dt_bias": checksum(first.dt_bias)}
    for s, (q, k, v, a, b) in enumerate(tokens):
        for name, t in (("q", q), ("k", k), ("v", v), ("a", a), ("b", b)):
            rec[f"in_{name}_{s}"] = checksum(t.float())
    rec.update(state_summary(state))
    np.savez_compressed(os.path.join(OUT, "decode_b4_qk16v32_16steps.npz"), **rec)

    # Small decode cases with every tensor stored: qk1_v2, with and without state.
    for with_state in (True, False):
        x = W.make_decode_inputs(2, seed=11, h_qk=1, h_v=2, with_state=with_state)
        o, ns = _gdn_decode_reference(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                                      0.0)  # scale 0 -> 1/sqrt(K)
        rec = {n: _np(getattr(x, n)) for n in ("q", "k", "v", "A_log", "a", "dt_bias", "b")}
        if with_state:
            rec["state"] = _np(x.state)
        rec["output"] = _np(o)
        rec["new_state"] = _np(ns)
        tag = "state" if with_state else "nostate"
        np.savez_compressed(os.path.join(OUT, f"decode_small_{tag}.npz"), **rec)

    # Small varlen prefill: ragged tails, an empty sequence, a 1-token sequence,
    # a 129-token sequence (two full chunks and a 1-token tail), int64 cu_seqlens; every tensor stored.
    for with_state in (True, False):
        lengths = [37, 0, 129, 1]
        x = W.make_prefill_inputs(lengths, seed=5, h_qk=1, h_v=2, with_state=with_state,
                                  cu_dtype=torch.int64)
        o, ns = _gdn_prefill_reference(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                                       x.cu_seqlens, x.scale)
        if with_state:
            for i, L in enumerate(lengths):
                if L == 0:
                    ns[i] = x.state[i]   # reference kernel semantics (kernel_prefill.cu:61-66)
        rec = {n: _np(getattr(x, n)) for n in ("q", "k", "v", "A_log", "a", "dt_bias", "b",
                                                "cu_seqlens")}
        if with_state:
            rec["state"] = _np(x.state)
        rec["output"] = _np(o)
        rec["new_state"] = _np(ns)
        tag = "state" if with_state else "nostate"
        np.savez_compressed(os.path.join(OUT, f"prefill_small_{tag}.npz"), **rec)

    # Full head layout, one ragged sequence of 150 tokens (64 + 64 + 22), seed 3.
    x = W.make_prefill_inputs([150], seed=3)
    o, ns = _gdn_prefill_reference(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b,
                                   x.cu_seqlens, x.scale)
    rec = {"output": _np(o)}
    for n in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b"):
        rec[f"in_{n}"] = checksum(getattr(x, n).float())
    rec.update(state_summary(ns))
    np.savez_compressed(os.path.join(OUT, "prefill_qk16v32_T150.npz"), **rec)
    print("fixtures written to", OUT)
    make_mtp()


def make_mtp():
    """Multi-token (MTP / speculative verify) decode against a state pool, from the
    next definition of the same family: ``_gdn_mtp_reference`` in
    ``flashinfer.trace.templates.gdn`` (flashinfer 0.6.11.post2).  B=3 sequences of
    T=3 tokens, qk1_v2, a pool of 5 fp32 slots of which slots 2, 0 and 3 are read
    (slots 1 and 4 stay untouched), and an intermediate-state buffer.  Inputs are
    regenerated from the seed and checked against stored checksums; outputs are
    stored in full, pool and intermediate states as row sums / sums of squares and
    one complete head."""
    from flashinfer.trace.templates.gdn import _gdn_mtp_reference

    x = W.make_pool_decode_inputs(3, 3, 5, seed=21, h_qk=1, h_v=2)
    idx = torch.tensor([2, 0, 3], dtype=torch.int32)
    inter = torch.zeros(5, 3, 2, 128, 128, dtype=torch.float32)
    o, final = _gdn_mtp_reference(x.q, x.k, x.v, x.pool, idx, x.A_log, x.a, x.dt_bias, x.b,
                                  0.0, intermediate_states_buffer=inter)
    rec = {"output": _np(o), "indices": idx.numpy()}
    for n in ("q", "k", "v", "pool", "A_log", "a", "dt_bias", "b"):
        rec[f"in_{n}"] = checksum(getattr(x, n).float())
    rec["pool_rowsum"] = final.double().sum(-1).numpy()
    rec["pool_rowsq"] = (final.double() ** 2).sum(-1).numpy()
    rec["pool_slot2_head1"] = final[2, 1].numpy().copy()
    rec["inter_rowsum"] = inter.double().sum(-1).numpy()
    rec["inter_slot0_t1_head0"] = inter[0, 1, 0].numpy().copy()
    np.savez_compressed(os.path.join(OUT, "mtp_b3_t3_qk1v2_pool5.npz"), **rec)
    print("MTP fixture written to", OUT)


if __name__ == "__main__":
    if sys.argv[1:] == ["--mtp"]:
        make_mtp()
    else:
        main()
