"""CPU fp32 oracle for the Gated DeltaNet hot path (decode T=1, chunked prefill).

TEST INFRASTRUCTURE ONLY.  This module is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it.  The product path (``gdn_kernel_b200``) never calls it and fails
loudly when its CUDA library is missing.

It restates, in vectorised PyTorch fp32 on the host, the algorithm of the
reference repository (jaewooMaeng/GDN_kernel):

* gate / beta math: ref solution/cuda/kernel.cu:44-53 and
  solution/cuda/kernel_prefill.cu:101-115 (softplus(x) = x for x > 20);
* decode step: ref solution/cuda/kernel.cu:55-96, whose semantics are the
  definition reference in ref design.md:157-226;
* sequential prefill: ref prefill_design.md:487-546, extended to packed
  variable-length tokens with ``cu_seqlens`` as in the contest definition;
* chunked prefill (C=64, WY/UT form): ref solution/cuda/kernel_prefill.cu:95-294;
* empty sequences copy their initial state: ref kernel_prefill.cu:61-66;
* ``scale == 0`` means 1/sqrt(K): ref kernel.cu:115-118;
* a missing (None) state means a zero initial state: ref kernel.cu:135-139,
  kernel_prefill.cu:327-330.

Parity pin: ``tests/golden/make_golden.py`` generates fixtures with the
published contest definition functions (flashinfer 0.6.11.post2,
``flashinfer.trace.templates.gdn``: ``_gdn_decode_reference`` and
``_gdn_prefill_reference``), and ``tests/test_oracle_golden.py`` checks this
module against them.  ``oracle/build_ref.sh`` compiles the reference's own
CUDA kernels (qk4_v8 head layout, as hard-coded there) into ``oracle/_ref``;
the GPU test ``tests/test_reference_kernels.py`` pins this oracle against
them on a B200.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

CHUNK = 64


def default_scale(scale: Optional[float], head_dim: int) -> float:
    """ref kernel.cu:115-118: a zero (or missing) scale means 1/sqrt(K)."""
    if scale is None or scale == 0.0:
        return 1.0 / math.sqrt(head_dim)
    return float(scale)


def log_gate_beta(A_log, a, dt_bias, b) -> Tuple[torch.Tensor, torch.Tensor]:
    """Log-gate and beta (ref kernel_prefill.cu:105-110, kernel.cu:44-53).

    log g = -exp(A_log) * softplus(a + dt_bias), softplus(x) = x for x > 20;
    beta = sigmoid(b).  Shapes broadcast over the trailing v-head axis.
    """
    x = a.float() + dt_bias.float()
    sp = F.softplus(x, beta=1.0, threshold=20.0)
    log_g = -torch.exp(A_log.float()) * sp
    beta = torch.sigmoid(b.float())
    return log_g, beta


def decode_step(q, k, v, state, A_log, a, dt_bias, b, scale=None):
    """One T=1 decode step (ref kernel.cu:55-96; ref design.md:157-226).

    q, k: [B, 1, H_qk, K] bf16; v: [B, 1, H_v, V] bf16; state: [B, H_v, V, K]
    fp32 or None; A_log, dt_bias: [H_v]; a, b: [B, 1, H_v].
    Returns (output [B, 1, H_v, V] bf16, new_state [B, H_v, V, K] fp32).
    """
    B, _, h_qk, K = q.shape
    h_v = v.shape[2]
    scale = default_scale(scale, K)
    log_g, beta = log_gate_beta(A_log, a[:, 0], dt_bias, b[:, 0])      # [B, H_v]
    g = torch.exp(log_g)
    rep = h_v // h_qk
    qf = q[:, 0].float().repeat_interleave(rep, dim=1)                 # [B, H_v, K]
    kf = k[:, 0].float().repeat_interleave(rep, dim=1)
    vf = v[:, 0].float()                                               # [B, H_v, V]
    if state is None:
        S = torch.zeros(B, h_v, v.shape[3], K, dtype=torch.float32)
    else:
        S = state.float()
    S = g[..., None, None] * S                                         # g * S
    old_v = torch.matmul(S, kf[..., None])[..., 0]                     # S k
    delta = beta[..., None] * (vf - old_v)                             # beta (v - S k)
    S = S + delta[..., None] * kf[:, :, None, :]                       # S += delta k^T
    out = scale * torch.matmul(S, qf[..., None])[..., 0]               # scale S q
    return out[:, None].to(torch.bfloat16), S


def _seq_bounds(cu_seqlens):
    cu = [int(x) for x in cu_seqlens.tolist()]
    return [(cu[i], cu[i + 1]) for i in range(len(cu) - 1)]


def prefill_sequential(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None):
    """Token-by-token recurrence over packed sequences, batched over heads.

    Follows ref prefill_design.md:487-546 (the decode step applied per token)
    with packed ``[T, H, D]`` tokens and ``cu_seqlens``; empty sequences copy
    their initial state (ref kernel_prefill.cu:61-66).
    Returns (output [T, H_v, V] bf16, new_state [N, H_v, V, K] fp32).
    """
    T, h_qk, K = q.shape
    h_v, V = v.shape[1], v.shape[2]
    scale = default_scale(scale, K)
    rep = h_v // h_qk
    log_g, beta = log_gate_beta(A_log, a, dt_bias, b)                  # [T, H_v]
    g = torch.exp(log_g)
    qf = q.float().repeat_interleave(rep, dim=1)
    kf = k.float().repeat_interleave(rep, dim=1)
    vf = v.float()
    bounds = _seq_bounds(cu_seqlens)
    out = torch.zeros(T, h_v, V, dtype=torch.float32)
    new_state = torch.zeros(len(bounds), h_v, V, K, dtype=torch.float32)
    for n, (s0, s1) in enumerate(bounds):
        S = torch.zeros(h_v, V, K) if state is None else state[n].float().clone()
        for t in range(s0, s1):
            S = g[t][:, None, None] * S
            old_v = torch.matmul(S, kf[t][:, :, None])[..., 0]
            delta = beta[t][:, None] * (vf[t] - old_v)
            S = S + delta[:, :, None] * kf[t][:, None, :]
            out[t] = scale * torch.matmul(S, qf[t][:, :, None])[..., 0]
        new_state[n] = S
    return out.to(torch.bfloat16), new_state


def prefill_chunked(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None,
                    chunk: int = CHUNK, return_chunk_states: bool = False):
    """Chunked (WY/UT) fp32 prefill, vectorised over heads.

    Restates ref kernel_prefill.cu:95-294 per chunk of ``chunk`` tokens:
      gamma = inclusive cumsum of the log-gate          (:101-122)
      A_ij  = -beta_i <k_i,k_j> e^{gamma_i-gamma_j}, i>j (:134-146)
      T     = (I - A)^{-1} (unit lower triangular)      (:148-163)
      P_ij  = <q_i,k_j> e^{gamma_i-gamma_j}, j<=i       (:165-185)
      W     = T (beta e^gamma K),  U = T (beta V)       (:187-195, :248-271)
      v_new = U - W S^T                                 (:236-271)
      O     = scale ((e^gamma Q) S^T + P v_new)         (:211-234, :273-284)
      S     = e^{gamma_last} S + v_new^T (K e^{gamma_last-gamma})  (:197-202, :286-293)
    With ``return_chunk_states`` the state entering every chunk is returned
    too (list per sequence of [n_chunks, H_v, V, K]), for drift reports.
    """
    T, h_qk, K = q.shape
    h_v, V = v.shape[1], v.shape[2]
    scale = default_scale(scale, K)
    rep = h_v // h_qk
    log_g, beta = log_gate_beta(A_log, a, dt_bias, b)                  # [T, H_v]
    qf = q.float().repeat_interleave(rep, dim=1).transpose(0, 1)       # [H_v, T, K]
    kf = k.float().repeat_interleave(rep, dim=1).transpose(0, 1)
    vf = v.float().transpose(0, 1)                                     # [H_v, T, V]
    lg = log_g.transpose(0, 1)                                         # [H_v, T]
    bt = beta.transpose(0, 1)
    bounds = _seq_bounds(cu_seqlens)
    out = torch.zeros(h_v, T, V, dtype=torch.float32)
    new_state = torch.zeros(len(bounds), h_v, V, K, dtype=torch.float32)
    chunk_states = []
    tri_strict = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool), -1)
    tri_incl = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool), 0)
    eye = torch.eye(chunk)
    for n, (s0, s1) in enumerate(bounds):
        S = torch.zeros(h_v, V, K) if state is None else state[n].float().clone()
        per_chunk = []
        for c0 in range(s0, s1, chunk):
            c1 = min(c0 + chunk, s1)
            L = c1 - c0
            Kc, Qc, Vc = kf[:, c0:c1], qf[:, c0:c1], vf[:, c0:c1]      # [H, L, D]
            gam = torch.cumsum(lg[:, c0:c1], dim=1)                     # [H, L]
            bc = bt[:, c0:c1]
            diff = gam[:, :, None] - gam[:, None, :]                    # gamma_i - gamma_j
            ms, mi = tri_strict[:L, :L], tri_incl[:L, :L]
            dec_s = torch.exp(torch.where(ms, diff, torch.full_like(diff, -math.inf)))
            dec_i = torch.exp(torch.where(mi, diff, torch.full_like(diff, -math.inf)))
            A = -bc[:, :, None] * (Kc @ Kc.transpose(1, 2)) * dec_s
            Tm = torch.linalg.solve_triangular(eye[:L, :L] - A, eye[:L, :L].expand(h_v, L, L),
                                               upper=False, unitriangular=True)
            eg = torch.exp(gam)
            W = Tm @ (Kc * (bc * eg)[:, :, None])
            U = Tm @ (Vc * bc[:, :, None])
            if return_chunk_states:
                per_chunk.append(S.clone())
            St = S.transpose(1, 2)                                      # [H, K, V]
            v_new = U - W @ St
            P = (Qc @ Kc.transpose(1, 2)) * dec_i
            out[:, c0:c1] = scale * ((Qc * eg[:, :, None]) @ St + P @ v_new)
            k_dec = Kc * torch.exp(gam[:, -1:] - gam)[:, :, None]
            S = torch.exp(gam[:, -1])[:, None, None] * S + v_new.transpose(1, 2) @ k_dec
        new_state[n] = S
        if return_chunk_states:
            chunk_states.append(torch.stack(per_chunk) if per_chunk else torch.zeros(0, h_v, V, K))
    res = (out.transpose(0, 1).to(torch.bfloat16).contiguous(), new_state)
    if return_chunk_states:
        return res + (chunk_states,)
    return res



def decode_pool(q, k, v, pool, read_idx, A_log, a, dt_bias, b, scale=None, write_idx=None,
                inter=None):
    """Decode of T >= 1 tokens per sequence against a state pool.

    Restates the MTP / speculative-verify definition (site
    flashinfer/trace/templates/gdn.py:378-466, ``_gdn_mtp_reference``: per token
    the decode step of ref kernel.cu:55-96, the state carried across the T
    tokens in fp32, the state after token t stored at ``inter[read_idx[b], t]``)
    and the pool addressing of FlashInfer's pooled decode (site
    flashinfer/gdn_decode.py:117-200: entry b reads slot ``read_idx[b]`` and
    writes slot ``write_idx[b]``, default the read slot; a negative index marks
    padding, whose outputs are zero and whose state is neither read nor
    written, the fp32 behaviour described at gdn_decode.py:182-195).

    q, k: [B, T, H_qk, K] bf16; v: [B, T, H_v, V] bf16; a, b: [B, T, H_v];
    pool: [P, H_v, V, K] fp32 or bf16; read_idx / write_idx: [B] integer;
    inter: None or [P, T, H_v, V, K] of the pool's dtype (updated in place).
    Returns (output [B, T, H_v, V] bf16, new_pool): ``new_pool`` is a copy of
    ``pool`` with the written slots replaced; a bf16 pool is rounded once per
    stored state.
    """
    B, T, h_qk, K = q.shape
    h_v = v.shape[2]
    scale = default_scale(scale, K)
    rep = h_v // h_qk
    log_g, beta = log_gate_beta(A_log, a, dt_bias, b)                  # [B, T, H_v]
    g = torch.exp(log_g)
    qf = q.float().repeat_interleave(rep, dim=2)                       # [B, T, H_v, K]
    kf = k.float().repeat_interleave(rep, dim=2)
    vf = v.float()
    out = torch.zeros(B, T, h_v, v.shape[3], dtype=torch.float32)
    new_pool = pool.clone()
    P = pool.shape[0]
    for bi in range(B):
        r = int(read_idx[bi])
        w = int(write_idx[bi]) if write_idx is not None else r
        if r < 0 or w < 0 or r >= P or w >= P:
            continue
        S = pool[r].float()                                            # [H_v, V, K]
        for t in range(T):
            S = g[bi, t][:, None, None] * S
            old_v = torch.matmul(S, kf[bi, t][..., None])[..., 0]      # [H_v, V]
            delta = beta[bi, t][:, None] * (vf[bi, t] - old_v)
            S = S + delta[..., None] * kf[bi, t][:, None, :]
            out[bi, t] = scale * torch.matmul(S, qf[bi, t][..., None])[..., 0]
            if inter is not None:
                inter[r, t] = S.to(inter.dtype)
        new_pool[w] = S.to(pool.dtype)
    return out.to(torch.bfloat16), new_pool
