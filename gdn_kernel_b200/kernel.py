"""Host-side mirror of the reference's ``kernel`` entry points.

The reference exports one TVM-FFI function named ``kernel`` per path, in
destination-passing style (all inputs, then the pre-allocated outputs):

* decode  (ref solution/cuda/kernel.cu:101-113):
  ``kernel(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)``
* prefill (ref solution/cuda/kernel_prefill.cu:300-305):
  ``kernel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state)``

``gdn_decode`` / ``gdn_prefill`` here take exactly those arguments (torch CUDA
tensors), validate them like the TVM-FFI exports of this package do (raising
``ValueError``), and call the C ABI of ``libgdn_b200.so`` on the current torch
stream.  ``decode`` / ``prefill`` are allocating conveniences on top.

``gdn_decode_pool`` / ``gdn_mtp`` / ``mtp`` are the serving-side forms of the
decode step that the next definitions of the same family add: a state pool
addressed by per-sequence indices (fp32 or bf16 state), and T > 1 tokens per
sequence with optional per-token intermediate states.
``load_tvm_kernel`` returns the TVM-FFI ``kernel`` itself, which is what the
reference's harness binds.

Semantics as in the reference: ``scale == 0`` means 1/sqrt(128); ``state`` may
be ``None`` (zero initial state); ``new_state`` may be ``state`` itself
(in-place); in prefill an empty sequence copies its initial state.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

HEAD_DIM = 128


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _check(t: torch.Tensor, name: str, dtype, shape, device) -> None:
    _require(isinstance(t, torch.Tensor), f"{name}: expected a torch.Tensor")
    _require(t.dtype == dtype, f"{name}: expected {dtype}, got {t.dtype}")
    _require(t.device == device, f"{name}: must be on {device}, got {t.device}")
    _require(tuple(t.shape) == tuple(shape), f"{name}: expected shape {tuple(shape)}, got {tuple(t.shape)}")
    _require(t.numel() == 0 or t.is_contiguous(), f"{name}: must be contiguous")


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _launch(dev, fn, *args) -> None:
    """Call a C entry point with ``dev`` current (the library launches on, and
    sets up, the current device) and ``dev``'s current torch stream as the last
    argument; raise on an error code."""
    with torch.cuda.device(dev):
        _lib.check(fn(*args, _stream(dev)))


def _cuda_device(q: torch.Tensor):
    _require(isinstance(q, torch.Tensor) and q.is_cuda, "q must be a CUDA tensor")
    return q.device


def gdn_decode(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state) -> None:
    """One T=1 decode step; same arguments as the reference decode ``kernel``.

    q, k: [B, 1, H_qk, 128] bf16; v: [B, 1, H_v, 128] bf16; state: [B, H_v, 128, 128]
    fp32 or None; A_log, dt_bias: [H_v] fp32; a, b: [B, 1, H_v] bf16;
    output: [B, 1, H_v, 128] bf16; new_state: [B, H_v, 128, 128] fp32 (may be state).
    """
    dev = _cuda_device(q)
    _require(q.dim() == 4 and v.dim() == 4, "q and v must be [B, 1, H, D]")
    B, T, h_qk, D = q.shape
    h_v = v.shape[2]
    _require(T == 1, "decode takes T == 1")
    _check(q, "q", torch.bfloat16, (B, 1, h_qk, D), dev)
    _check(k, "k", torch.bfloat16, (B, 1, h_qk, D), dev)
    _check(v, "v", torch.bfloat16, (B, 1, h_v, D), dev)
    _check(A_log, "A_log", torch.float32, (h_v,), dev)
    _check(a, "a", torch.bfloat16, (B, 1, h_v), dev)
    _check(dt_bias, "dt_bias", torch.float32, (h_v,), dev)
    _check(b, "b", torch.bfloat16, (B, 1, h_v), dev)
    _check(output, "output", torch.bfloat16, (B, 1, h_v, D), dev)
    _check(new_state, "new_state", torch.float32, (B, h_v, D, D), dev)
    if state is not None:
        _check(state, "state", torch.float32, (B, h_v, D, D), dev)
    lib = _lib.load()
    _launch(dev, lib.gdn_b200_decode,
        _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b),
        float(scale or 0.0), _ptr(output), _ptr(new_state), B, h_qk, h_v, D)


def gdn_decode_pool(q, k, v, state_pool, state_indices, A_log, a, dt_bias, b, scale, output,
                    *, new_state_pool=None, output_state_indices=None,
                    intermediate_states=None) -> None:
    """Decode of T >= 1 tokens per sequence against a state pool (serving form).

    Semantics of FlashInfer's pooled decode (``gated_delta_rule_decode_pretranspose``
    with ``initial_state`` / ``initial_state_indices`` / ``output_state_indices``,
    site flashinfer/gdn_decode.py:117-200) and, for T > 1, of the MTP definition
    (site flashinfer/trace/templates/gdn.py:378-466), with q and k as given (no
    L2 normalisation inside; the reference decode has none either).

    q, k: [B, T, H_qk, 128] bf16; v: [B, T, H_v, 128] bf16; a, b: [B, T, H_v] bf16;
    state_pool: [P, H_v, 128, 128] fp32 or bf16; state_indices: [B] int32/int64
    (entry b reads slot state_indices[b]; negative = padding: zero output, no state
    read or written); output: [B, T, H_v, 128] bf16.
    new_state_pool: where final states go (default: state_pool itself, in place);
    output_state_indices: [B] write slots (default: the read slots);
    intermediate_states: [P, T, H_v, 128, 128] of the pool's dtype or None; the
    state after token t of entry b lands at [state_indices[b], t].
    """
    dev = _cuda_device(q)
    _require(q.dim() == 4 and v.dim() == 4, "q and v must be [B, T, H, D]")
    B, T, h_qk, D = q.shape
    h_v = v.shape[2]
    _require(T >= 1, "T must be >= 1")
    _require(isinstance(state_pool, torch.Tensor) and state_pool.dim() == 4,
             "state_pool must be [P, H_v, D, D]")
    sdt = state_pool.dtype
    _require(sdt in (torch.float32, torch.bfloat16), "state_pool must be fp32 or bf16")
    P = state_pool.shape[0]
    _check(q, "q", torch.bfloat16, (B, T, h_qk, D), dev)
    _check(k, "k", torch.bfloat16, (B, T, h_qk, D), dev)
    _check(v, "v", torch.bfloat16, (B, T, h_v, D), dev)
    _check(A_log, "A_log", torch.float32, (h_v,), dev)
    _check(a, "a", torch.bfloat16, (B, T, h_v), dev)
    _check(dt_bias, "dt_bias", torch.float32, (h_v,), dev)
    _check(b, "b", torch.bfloat16, (B, T, h_v), dev)
    _check(output, "output", torch.bfloat16, (B, T, h_v, D), dev)
    _check(state_pool, "state_pool", sdt, (P, h_v, D, D), dev)
    if new_state_pool is None:
        new_state_pool = state_pool
    _check(new_state_pool, "new_state_pool", sdt, (P, h_v, D, D), dev)
    _require(isinstance(state_indices, torch.Tensor)
             and state_indices.dtype in (torch.int32, torch.int64),
             "state_indices must be an int32 or int64 tensor")
    _check(state_indices, "state_indices", state_indices.dtype, (B,), dev)
    if output_state_indices is not None:
        _check(output_state_indices, "output_state_indices", state_indices.dtype, (B,), dev)
    if intermediate_states is not None:
        _check(intermediate_states, "intermediate_states", sdt, (P, T, h_v, D, D), dev)
    lib = _lib.load()
    _launch(dev, lib.gdn_b200_decode_pool,
        _ptr(q), _ptr(k), _ptr(v), _ptr(state_pool), _ptr(new_state_pool),
        1 if sdt == torch.bfloat16 else 0, _ptr(state_indices), _ptr(output_state_indices),
        1 if state_indices.dtype == torch.int64 else 0, _ptr(intermediate_states),
        _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b), float(scale or 0.0), _ptr(output),
        B, T, P, h_qk, h_v, D)


def gdn_mtp(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale,
            output, final_state, intermediate_states_buffer=None) -> None:
    """Multi-token (MTP / speculative verify) decode in destination-passing style,
    argument order of the MTP definition (site flashinfer/trace/templates/gdn.py:
    378-466) with its outputs (output, final_state) appended.

    ``final_state`` may be ``initial_state`` (in place, the serving case);
    otherwise only the indexed slots of ``final_state`` are written, so a caller
    wanting the definition's full returned pool copies ``initial_state`` into it
    first (``mtp`` below does).
    """
    gdn_decode_pool(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale,
                    output, new_state_pool=final_state,
                    intermediate_states=intermediate_states_buffer)


def mtp(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale=0.0,
        intermediate_states_buffer=None):
    """Allocating MTP decode with the definition's return values: ``(output,
    final_state)``, ``final_state`` a new pool equal to ``initial_state`` except
    at the indexed slots."""
    B, T, _, D = q.shape
    h_v = v.shape[2]
    output = torch.empty((B, T, h_v, D), dtype=torch.bfloat16, device=q.device)
    final_state = initial_state.clone()
    gdn_mtp(q, k, v, initial_state, initial_state_indices, A_log, a, dt_bias, b, scale, output,
            final_state, intermediate_states_buffer)
    return output, final_state


def state_affine(state, transfer, offset, out=None):
    """``out[h] = state[h] @ transfer[h] + offset[h]`` for [H, 128, 128] fp32 CUDA
    tensors (``state`` None means zero): the affine combine of context-parallel
    prefill.  Returns ``out`` (allocated when omitted)."""
    dev = _cuda_device(offset)
    H = offset.shape[0]
    _check(offset, "offset", torch.float32, (H, HEAD_DIM, HEAD_DIM), dev)
    if state is not None:
        _check(state, "state", torch.float32, (H, HEAD_DIM, HEAD_DIM), dev)
        _check(transfer, "transfer", torch.float32, (H, HEAD_DIM, HEAD_DIM), dev)
    if out is None:
        out = torch.empty_like(offset)
    _check(out, "out", torch.float32, (H, HEAD_DIM, HEAD_DIM), dev)
    _launch(dev, _lib.load().gdn_b200_state_affine, _ptr(state), _ptr(transfer), _ptr(offset),
                                                 _ptr(out), H)
    return out


PREFILL_PATHS = ("split", "ring", "fused")


def prefill_workspace_bytes(num_seqs: int, total_tokens: int, num_v_heads: int) -> int:
    """Device workspace of the two-stage prefill for this problem size."""
    return int(_lib.load().gdn_b200_prefill_workspace_size(num_seqs, total_tokens, num_v_heads))


def gdn_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
                new_state, *, path: str = "split", workspace=None) -> None:
    """Chunked prefill; same arguments as the reference prefill ``kernel``.

    q, k: [T, H_qk, 128] bf16 (packed tokens); v: [T, H_v, 128] bf16;
    state: [N, H_v, 128, 128] fp32 or None; a, b: [T, H_v] bf16;
    cu_seqlens: [N + 1] int32 or int64 on the same device;
    output: [T, H_v, 128] bf16; new_state: [N, H_v, 128, 128] fp32 (may be state).

    ``path="split"`` (default) runs the two-stage kernels (parallel per-chunk
    preparation, then the sequential state recurrence) with a device workspace
    (``workspace``: a uint8 CUDA tensor of at least ``prefill_workspace_bytes``
    bytes, allocated here when omitted); ``path="ring"`` runs the same kernels
    in the library's static record ring and allocates nothing (the C ABI's
    ``gdn_b200_prefill``, what the TVM-FFI ``kernel`` calls; bit-identical to
    "split"); ``path="fused"`` runs the single kernel that needs no workspace
    (agrees with the others to the prefill tolerance).
    """
    dev = _cuda_device(q)
    _require(q.dim() == 3 and v.dim() == 3, "q and v must be packed [T, H, D]")
    T, h_qk, D = q.shape
    h_v = v.shape[1]
    _require(isinstance(cu_seqlens, torch.Tensor) and cu_seqlens.dim() == 1
             and cu_seqlens.numel() >= 1, "cu_seqlens must be [N + 1]")
    _require(cu_seqlens.dtype in (torch.int32, torch.int64), "cu_seqlens must be int32 or int64")
    N = cu_seqlens.numel() - 1
    _check(cu_seqlens, "cu_seqlens", cu_seqlens.dtype, (N + 1,), dev)
    _check(q, "q", torch.bfloat16, (T, h_qk, D), dev)
    _check(k, "k", torch.bfloat16, (T, h_qk, D), dev)
    _check(v, "v", torch.bfloat16, (T, h_v, D), dev)
    _check(A_log, "A_log", torch.float32, (h_v,), dev)
    _check(a, "a", torch.bfloat16, (T, h_v), dev)
    _check(dt_bias, "dt_bias", torch.float32, (h_v,), dev)
    _check(b, "b", torch.bfloat16, (T, h_v), dev)
    _check(output, "output", torch.bfloat16, (T, h_v, D), dev)
    _check(new_state, "new_state", torch.float32, (N, h_v, D, D), dev)
    if state is not None:
        _check(state, "state", torch.float32, (N, h_v, D, D), dev)
    _require(path in PREFILL_PATHS, f"path must be one of {PREFILL_PATHS}")
    lib = _lib.load()
    args = (_ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b),
            _ptr(cu_seqlens), 1 if cu_seqlens.dtype == torch.int64 else 0, float(scale or 0.0),
            _ptr(output), _ptr(new_state), N, T, h_qk, h_v, D)
    if path == "fused":
        _launch(dev, lib.gdn_b200_prefill_fused, *args)
        return
    if path == "ring" or N == 0:
        _launch(dev, lib.gdn_b200_prefill, *args)
        return
    need = prefill_workspace_bytes(N, T, h_v)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    _require(isinstance(workspace, torch.Tensor) and workspace.device == dev
             and workspace.numel() * workspace.element_size() >= need,
             f"workspace must be a tensor on {dev} of at least {need} bytes")
    _launch(dev, lib.gdn_b200_prefill_ws, *args, _ptr(workspace),
                                       workspace.numel() * workspace.element_size())


def gdn_prefill_prepare(q, k, A_log, a, dt_bias, b, cu_seqlens, workspace) -> None:
    """First stage of the two-stage prefill: the chunk table and the per-(chunk,
    v-head) records into ``workspace`` (see ``prefill_workspace_bytes``); depends
    on q, k, a, b and the head parameters only."""
    dev = _cuda_device(q)
    T, h_qk, D = q.shape
    h_v = a.shape[1]
    N = cu_seqlens.numel() - 1
    _require(cu_seqlens.dtype in (torch.int32, torch.int64), "cu_seqlens must be int32 or int64")
    _check(cu_seqlens, "cu_seqlens", cu_seqlens.dtype, (N + 1,), dev)
    _check(q, "q", torch.bfloat16, (T, h_qk, D), dev)
    _check(k, "k", torch.bfloat16, (T, h_qk, D), dev)
    _check(A_log, "A_log", torch.float32, (h_v,), dev)
    _check(a, "a", torch.bfloat16, (T, h_v), dev)
    _check(dt_bias, "dt_bias", torch.float32, (h_v,), dev)
    _check(b, "b", torch.bfloat16, (T, h_v), dev)
    _launch(dev, _lib.load().gdn_b200_prefill_prepare,
        _ptr(q), _ptr(k), _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b), _ptr(cu_seqlens),
        1 if cu_seqlens.dtype == torch.int64 else 0, N, T, h_qk, h_v, D, _ptr(workspace),
        workspace.numel() * workspace.element_size())


def gdn_prefill_recur(k, v, state, scale, output, new_state, num_seqs, num_v_heads,
                      workspace) -> None:
    """Second stage: the state recurrence over a workspace a preceding
    ``gdn_prefill_prepare`` filled (read only, so several may run concurrently).
    ``v`` None means zero values, ``output`` None skips the outputs, ``state``
    None means zero initial states."""
    dev = _cuda_device(k)
    T, h_qk, D = k.shape
    _check(k, "k", torch.bfloat16, (T, h_qk, D), dev)
    if v is not None:
        _check(v, "v", torch.bfloat16, (T, num_v_heads, D), dev)
    if output is not None:
        _check(output, "output", torch.bfloat16, (T, num_v_heads, D), dev)
    _check(new_state, "new_state", torch.float32, (num_seqs, num_v_heads, D, D), dev)
    if state is not None:
        _check(state, "state", torch.float32, (num_seqs, num_v_heads, D, D), dev)
    _launch(dev, _lib.load().gdn_b200_prefill_recur,
        _ptr(k), _ptr(v), _ptr(state), float(scale or 0.0), _ptr(output), _ptr(new_state),
        num_seqs, T, h_qk, num_v_heads, D, _ptr(workspace),
        workspace.numel() * workspace.element_size())


def decode(q, k, v, state, A_log, a, dt_bias, b, scale: float = 0.0, *, in_place: bool = False):
    """Allocating decode: returns ``(output, new_state)``; with ``in_place`` the
    new state is written into ``state``."""
    B, _, _, D = q.shape
    h_v = v.shape[2]
    output = torch.empty((B, 1, h_v, D), dtype=torch.bfloat16, device=q.device)
    if in_place:
        _require(state is not None, "in_place needs a state tensor")
        new_state = state
    else:
        new_state = torch.empty((B, h_v, D, D), dtype=torch.float32, device=q.device)
    gdn_decode(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)
    return output, new_state


def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale: float = 0.0, *,
            in_place: bool = False, path: str = "split"):
    """Allocating prefill: returns ``(output, new_state)``."""
    T, _, D = q.shape
    h_v = v.shape[1]
    N = cu_seqlens.numel() - 1
    output = torch.empty((T, h_v, D), dtype=torch.bfloat16, device=q.device)
    if in_place:
        _require(state is not None, "in_place needs a state tensor")
        new_state = state
    else:
        new_state = torch.empty((N, h_v, D, D), dtype=torch.float32, device=q.device)
    gdn_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
                path=path)
    return output, new_state


def load_tvm_kernel(kind: str):
    """The TVM-FFI ``kernel`` function of this package for ``kind`` in
    {"decode", "prefill"}: the object the reference's harness binds."""
    import tvm_ffi

    path = {"decode": _lib.TVM_DECODE_PATH, "prefill": _lib.TVM_PREFILL_PATH}[kind]
    return tvm_ffi.load_module(path)["kernel"]
