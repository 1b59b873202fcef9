"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (Qwen3-Next-style GDN head layout: 16 qk heads,
32 v heads, head dim 128).

The contest's own workload tensors (the ``mlsys26-contest`` dataset that the
reference's harness reads, ref: scripts/run_local.py:30-74) are not available
offline; these generators stand in for them:

* q, k ~ N(0, 1) in bf16, L2-normalised per head (normalised in fp32, then
  rounded to bf16);
* v, a, b ~ N(0, 1) in bf16;
* A_log = log(U(1, 16)), dt_bias ~ N(0, 0.1), both fp32 per v head;
* state ~ N(0, 0.02) fp32 (standard deviation 0.02), k-last ``[N, H_v, V, K]``;
* scale = 1/sqrt(128).

Tensors are generated with a ``torch.Generator`` on the requested device so
that large benchmark inputs can be drawn directly in HBM.
"""

from __future__ import annotations

import dataclasses
import math
from typing import Optional

import torch

HEAD_DIM = 128
NUM_QK_HEADS = 16
NUM_V_HEADS = 32


@dataclasses.dataclass
class DecodeInputs:
    q: torch.Tensor        # [B, 1, H_qk, K] bf16
    k: torch.Tensor        # [B, 1, H_qk, K] bf16
    v: torch.Tensor        # [B, 1, H_v, V] bf16
    state: Optional[torch.Tensor]  # [B, H_v, V, K] fp32 or None
    A_log: torch.Tensor    # [H_v] fp32
    a: torch.Tensor        # [B, 1, H_v] bf16
    dt_bias: torch.Tensor  # [H_v] fp32
    b: torch.Tensor        # [B, 1, H_v] bf16
    scale: float


@dataclasses.dataclass
class PrefillInputs:
    q: torch.Tensor        # [T, H_qk, K] bf16 (packed tokens)
    k: torch.Tensor        # [T, H_qk, K] bf16
    v: torch.Tensor        # [T, H_v, V] bf16
    state: Optional[torch.Tensor]  # [N, H_v, V, K] fp32 or None
    A_log: torch.Tensor    # [H_v] fp32
    a: torch.Tensor        # [T, H_v] bf16
    dt_bias: torch.Tensor  # [H_v] fp32
    b: torch.Tensor        # [T, H_v] bf16
    cu_seqlens: torch.Tensor  # [N + 1] int32 or int64
    scale: float


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _normal(shape, gen, device, std=1.0):
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std


def _unit_heads(x: torch.Tensor) -> torch.Tensor:
    """L2-normalise along the last (head_dim) axis in fp32, return bf16."""
    return (x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)).to(torch.bfloat16)


def _head_params(gen, device, h_v):
    A_log = torch.log(torch.rand((h_v,), generator=gen, device=device) * 15.0 + 1.0)
    dt_bias = _normal((h_v,), gen, device, std=0.1)
    return A_log.float(), dt_bias.float()


def make_decode_inputs(batch: int, seed: int = 0, device="cpu", h_qk: int = NUM_QK_HEADS,
                       h_v: int = NUM_V_HEADS, d: int = HEAD_DIM, with_state: bool = True,
                       state_std: float = 0.02) -> DecodeInputs:
    """Inputs of one decode step (T=1) of the decode configurations."""
    gen = _gen(seed, device)
    q = _unit_heads(_normal((batch, 1, h_qk, d), gen, device))
    k = _unit_heads(_normal((batch, 1, h_qk, d), gen, device))
    v = _normal((batch, 1, h_v, d), gen, device).to(torch.bfloat16)
    A_log, dt_bias = _head_params(gen, device, h_v)
    a = _normal((batch, 1, h_v), gen, device).to(torch.bfloat16)
    b = _normal((batch, 1, h_v), gen, device).to(torch.bfloat16)
    state = _normal((batch, h_v, d, d), gen, device, std=state_std) if with_state else None
    return DecodeInputs(q, k, v, state, A_log, a, dt_bias, b, 1.0 / math.sqrt(d))


def make_decode_step_tokens(batch: int, seed: int, device="cpu", h_qk: int = NUM_QK_HEADS,
                            h_v: int = NUM_V_HEADS, d: int = HEAD_DIM):
    """Per-step token inputs (q, k, v, a, b) for a multi-step decode run."""
    gen = _gen(seed, device)
    q = _unit_heads(_normal((batch, 1, h_qk, d), gen, device))
    k = _unit_heads(_normal((batch, 1, h_qk, d), gen, device))
    v = _normal((batch, 1, h_v, d), gen, device).to(torch.bfloat16)
    a = _normal((batch, 1, h_v), gen, device).to(torch.bfloat16)
    b = _normal((batch, 1, h_v), gen, device).to(torch.bfloat16)
    return q, k, v, a, b


def make_decode_run(batch: int, steps: int, seed: int = 0, device="cpu", h_qk: int = NUM_QK_HEADS,
                    h_v: int = NUM_V_HEADS, d: int = HEAD_DIM, with_state: bool = True):
    """A multi-step decode run drawn from one seed: the step-0 inputs (with the
    initial state and per-head parameters) plus the token inputs of every later
    step, as a list of ``(q, k, v, a, b)`` tuples of length ``steps``."""
    first = make_decode_inputs(batch, seed, device, h_qk, h_v, d, with_state)
    tokens = [(first.q, first.k, first.v, first.a, first.b)]
    for s in range(1, steps):
        tokens.append(make_decode_step_tokens(batch, seed * 7919 + s, device, h_qk, h_v, d))
    return first, tokens


@dataclasses.dataclass
class PoolDecodeInputs:
    q: torch.Tensor          # [B, T, H_qk, D] bf16
    k: torch.Tensor          # [B, T, H_qk, D] bf16
    v: torch.Tensor          # [B, T, H_v, D] bf16
    pool: torch.Tensor       # [P, H_v, D, D] fp32 or bf16
    indices: torch.Tensor    # [B] int32 / int64: each entry's pool slot
    A_log: torch.Tensor
    a: torch.Tensor          # [B, T, H_v] bf16
    dt_bias: torch.Tensor
    b: torch.Tensor          # [B, T, H_v] bf16
    scale: float


def make_pool_decode_inputs(batch: int, seq_len: int, pool_size: int, seed: int = 0,
                            device="cpu", h_qk: int = NUM_QK_HEADS, h_v: int = NUM_V_HEADS,
                            d: int = HEAD_DIM, state_dtype=torch.float32,
                            idx_dtype=torch.int32, state_std: float = 0.02) -> PoolDecodeInputs:
    """Inputs of a pooled decode / MTP step: ``seq_len`` tokens per sequence, a
    state pool of ``pool_size`` slots and a random slot permutation (entries
    read distinct slots; ``pool_size >= batch``)."""
    if pool_size < batch:
        raise ValueError("pool_size must be >= batch")
    gen = _gen(seed, device)
    q = _unit_heads(_normal((batch, seq_len, h_qk, d), gen, device))
    k = _unit_heads(_normal((batch, seq_len, h_qk, d), gen, device))
    v = _normal((batch, seq_len, h_v, d), gen, device).to(torch.bfloat16)
    A_log, dt_bias = _head_params(gen, device, h_v)
    a = _normal((batch, seq_len, h_v), gen, device).to(torch.bfloat16)
    b = _normal((batch, seq_len, h_v), gen, device).to(torch.bfloat16)
    pool = _normal((pool_size, h_v, d, d), gen, device, std=state_std).to(state_dtype)
    perm = torch.randperm(pool_size, generator=gen, device=device)[:batch]
    return PoolDecodeInputs(q, k, v, pool, perm.to(idx_dtype), A_log, a, dt_bias, b,
                            1.0 / math.sqrt(d))


def varlen_lengths(num_seqs: int, lo: int, hi: int, seed: int) -> list:
    """Sequence lengths drawn uniformly from [lo, hi] by seed."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (num_seqs,), generator=gen).tolist()


def make_prefill_inputs(lengths, seed: int = 0, device="cpu", h_qk: int = NUM_QK_HEADS,
                        h_v: int = NUM_V_HEADS, d: int = HEAD_DIM, with_state: bool = True,
                        cu_dtype=torch.int32, state_std: float = 0.02) -> PrefillInputs:
    """Packed variable-length prefill inputs indexed by ``cu_seqlens``."""
    gen = _gen(seed, device)
    total = int(sum(lengths))
    q = _unit_heads(_normal((total, h_qk, d), gen, device))
    k = _unit_heads(_normal((total, h_qk, d), gen, device))
    v = _normal((total, h_v, d), gen, device).to(torch.bfloat16)
    A_log, dt_bias = _head_params(gen, device, h_v)
    a = _normal((total, h_v), gen, device).to(torch.bfloat16)
    b = _normal((total, h_v), gen, device).to(torch.bfloat16)
    n = len(lengths)
    state = _normal((n, h_v, d, d), gen, device, std=state_std) if with_state else None
    cu = torch.zeros(n + 1, dtype=torch.int64)
    cu[1:] = torch.cumsum(torch.tensor(lengths, dtype=torch.int64), 0)
    return PrefillInputs(q, k, v, state, A_log, a, dt_bias, b, cu.to(cu_dtype).to(device),
                         1.0 / math.sqrt(d))
