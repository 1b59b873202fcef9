"""Shared helpers of the GPU parity tests: device copies, tolerances, reports."""

import torch

# Tolerances (the reference's harness defaults are not available offline; these
# are this build's stated bars).
DECODE_OUT_TOL = dict(atol=1e-2, rtol=1e-2)      # bf16 output
DECODE_STATE_TOL = dict(atol=1e-4, rtol=1e-4)    # fp32 state (reassociation only)
PREFILL_OUT_TOL = dict(atol=2e-2, rtol=2e-2)     # bf16 output, bf16 tensor-core operands
PREFILL_STATE_REL_FRO = 1e-2                     # ||S - S_ref||_F / ||S_ref||_F per (seq, head)


def to_dev(x, dev="cuda"):
    return None if x is None else x.to(dev)


def rel_fro(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Relative Frobenius error per leading [N, H] block of [N, H, V, K] states."""
    a, b = a.double(), b.double()
    num = (a - b).flatten(2).norm(dim=-1)
    den = b.flatten(2).norm(dim=-1).clamp_min(1e-30)
    return num / den


def assert_prefill_close(out, new_state, ref_out, ref_state, lengths=None):
    torch.testing.assert_close(out.float().cpu(), ref_out.float(), **PREFILL_OUT_TOL)
    err = rel_fro(new_state.cpu(), ref_state)
    if lengths is not None:
        # an empty sequence with a zero state has no scale: compare absolutely
        for i, L in enumerate(lengths):
            if ref_state[i].abs().max() == 0:
                err[i] = (new_state[i].cpu() - ref_state[i]).abs().max().double()
    assert err.max().item() <= PREFILL_STATE_REL_FRO, f"state rel-Frobenius {err.max().item():.3e}"
    return err
