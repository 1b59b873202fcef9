"""Pooled / multi-token decode (gdn_b200_decode_pool) against the CPU oracle and
the MTP definition fixture, through the C ABI."""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from helpers import DECODE_OUT_TOL, DECODE_STATE_TOL
from gdn_kernel_b200 import _lib, kernel as K, workloads as W
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

BF16_STATE_TOL = dict(atol=2e-3, rtol=1e-2)   # one bf16 rounding of each stored state


def _cpu(x):
    return x.cpu() if isinstance(x, torch.Tensor) else x


def _run(x, idx, *, write=None, inter=False, in_place=True):
    dev = "cuda"
    q, k, v, a, b = (t.to(dev) for t in (x.q, x.k, x.v, x.a, x.b))
    pool = x.pool.to(dev).clone()
    B, T, _, D = x.q.shape
    h_v = x.v.shape[2]
    out = torch.full((B, T, h_v, D), float("nan"), dtype=torch.bfloat16, device=dev)
    new_pool = pool if in_place else pool.clone()
    ibuf = (torch.zeros((pool.shape[0], T, h_v, D, D), dtype=pool.dtype, device=dev)
            if inter else None)
    K.gdn_decode_pool(q, k, v, pool, idx.to(dev), x.A_log.to(dev), a, x.dt_bias.to(dev), b,
                      x.scale, out, new_state_pool=new_pool,
                      output_state_indices=None if write is None else write.to(dev),
                      intermediate_states=ibuf)
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0
    return out.cpu(), new_pool.cpu(), None if ibuf is None else ibuf.cpu()


def _oracle(x, idx, write=None, inter=False):
    ibuf = None
    if inter:
        B, T, _, D = x.q.shape
        ibuf = torch.zeros((x.pool.shape[0], T, x.v.shape[2], D, D), dtype=x.pool.dtype)
    o, p = O.decode_pool(x.q, x.k, x.v, x.pool, idx, x.A_log, x.a, x.dt_bias, x.b, x.scale,
                         write_idx=write, inter=ibuf)
    return o, p, ibuf


def test_t1_identity_slots_equals_plain_decode():
    """T=1 with slots 0..B-1 is the plain decode step: same kernel arithmetic."""
    x = W.make_pool_decode_inputs(8, 1, 8, seed=3)
    idx = torch.arange(8, dtype=torch.int32)
    out, pool, _ = _run(x, idx)
    ro, rs = K.decode(x.q.cuda(), x.k.cuda(), x.v.cuda(), x.pool.cuda(), x.A_log.cuda(),
                      x.a.cuda(), x.dt_bias.cuda(), x.b.cuda(), x.scale)
    assert torch.equal(out, ro.cpu())
    assert torch.equal(pool, rs.cpu())


@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64])
def test_t1_permuted_slots_padding_and_write_slots(idx_dtype):
    x = W.make_pool_decode_inputs(5, 1, 12, seed=5, idx_dtype=idx_dtype)
    read = torch.tensor([7, -1, 0, 11, 3], dtype=idx_dtype)
    write = torch.tensor([1, 9, 2, 4, 6], dtype=idx_dtype)
    out, pool, _ = _run(x, read, write=write)
    ro, rp, _ = _oracle(x, read, write=write)
    torch.testing.assert_close(out.float(), ro.float(), **DECODE_OUT_TOL)
    assert out[1].float().abs().max().item() == 0.0          # padding entry
    torch.testing.assert_close(pool, rp, **DECODE_STATE_TOL)
    for s in (0, 3, 5, 7, 8, 9, 10, 11):                       # slots nobody writes
        assert torch.equal(pool[s], x.pool[s])


@pytest.mark.parametrize("T", [2, 4, 7, 20])   # 20: two staged token groups of 16
def test_mtp_fp32_with_intermediate_states(T):
    x = W.make_pool_decode_inputs(6, T, 9, seed=10 + T)
    out, pool, inter = _run(x, x.indices, inter=True)
    ro, rp, ri = _oracle(x, x.indices, inter=True)
    torch.testing.assert_close(out.float(), ro.float(), **DECODE_OUT_TOL)
    torch.testing.assert_close(pool, rp, **DECODE_STATE_TOL)
    torch.testing.assert_close(inter, ri, **DECODE_STATE_TOL)


@pytest.mark.parametrize("T", [1, 3, 17])
def test_bf16_state_pool(T):
    x = W.make_pool_decode_inputs(4, T, 6, seed=30 + T, state_dtype=torch.bfloat16)
    out, pool, inter = _run(x, x.indices, inter=True)
    ro, rp, ri = _oracle(x, x.indices, inter=True)
    assert pool.dtype == torch.bfloat16
    torch.testing.assert_close(out.float(), ro.float(), **DECODE_OUT_TOL)
    torch.testing.assert_close(pool.float(), rp.float(), **BF16_STATE_TOL)
    torch.testing.assert_close(inter.float(), ri.float(), **BF16_STATE_TOL)


@pytest.mark.parametrize("state_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T", [2, 16])   # both ends of the two-row-blocks-per-CTA path
def test_multi_token_padding_and_write_slots(T, state_dtype):
    """T > 1 with a padding entry (read index -1) and separate write slots: the
    padding entry's outputs are zero on every row of both row blocks a CTA
    owns (the output buffer starts as NaN), and no slot but the written ones
    changes."""
    x = W.make_pool_decode_inputs(4, T, 10, seed=70 + T, state_dtype=state_dtype)
    read = torch.tensor([6, -1, 0, 9], dtype=torch.int32)
    write = torch.tensor([1, 8, 2, 7], dtype=torch.int32)   # no slot both read and written
    out, pool, _ = _run(x, read, write=write)
    ro, rp, _ = _oracle(x, read, write=write)
    tol = DECODE_STATE_TOL if state_dtype == torch.float32 else BF16_STATE_TOL
    torch.testing.assert_close(out.float(), ro.float(), **DECODE_OUT_TOL)
    assert torch.equal(out[1].float(), torch.zeros_like(out[1].float()))
    torch.testing.assert_close(pool.float(), rp.float(), **tol)
    for s in (0, 3, 4, 5, 6, 8, 9):   # read-only, untouched or the padding entry's slot
        assert torch.equal(pool[s], x.pool[s])


def test_in_place_equals_out_of_place():
    x = W.make_pool_decode_inputs(4, 3, 4, seed=40)
    o1, p1, _ = _run(x, x.indices, in_place=True)
    o2, p2, _ = _run(x, x.indices, in_place=False)
    assert torch.equal(o1, o2) and torch.equal(p1, p2)


def test_mtp_definition_fixture():
    """The MTP definition function's fixture (qk1_v2, pool of 5, T=3) on the GPU."""
    g = dict(np.load(os.path.join(GOLDEN, "mtp_b3_t3_qk1v2_pool5.npz")))
    x = W.make_pool_decode_inputs(3, 3, 5, seed=21, h_qk=1, h_v=2)
    idx = torch.from_numpy(g["indices"].copy())
    q, k, v, a, b = (t.cuda() for t in (x.q, x.k, x.v, x.a, x.b))
    inter = torch.zeros(5, 3, 2, 128, 128, device="cuda")
    out, final = K.mtp(q, k, v, x.pool.cuda(), idx.cuda(), x.A_log.cuda(), a, x.dt_bias.cuda(),
                       b, 0.0, intermediate_states_buffer=inter)
    torch.cuda.synchronize()
    ref = torch.from_numpy(g["output"].view(np.int16).copy()).view(torch.bfloat16).float()
    torch.testing.assert_close(out.cpu().float(), ref, **DECODE_OUT_TOL)
    final = final.cpu().double()
    np.testing.assert_allclose(final.sum(-1).numpy(), g["pool_rowsum"], atol=1e-3)
    np.testing.assert_allclose(final[2, 1].numpy(), g["pool_slot2_head1"], **DECODE_STATE_TOL)
    inter = inter.cpu().double()
    np.testing.assert_allclose(inter.sum(-1).numpy(), g["inter_rowsum"], atol=1e-3)
    np.testing.assert_allclose(inter[0, 1, 0].numpy(), g["inter_slot0_t1_head0"],
                               **DECODE_STATE_TOL)


def test_out_of_range_index_is_padding_and_flagged():
    x = W.make_pool_decode_inputs(2, 2, 3, seed=50)
    dev = "cuda"
    pool = x.pool.to(dev).clone()
    out = torch.full((2, 2, 32, 128), float("nan"), dtype=torch.bfloat16, device=dev)
    idx = torch.tensor([1, 3], dtype=torch.int32, device=dev)      # 3 >= pool_size
    K.gdn_decode_pool(x.q.to(dev), x.k.to(dev), x.v.to(dev), pool, idx, x.A_log.to(dev),
                      x.a.to(dev), x.dt_bias.to(dev), x.b.to(dev), x.scale, out)
    status = _lib.device_status(torch.cuda.current_device())
    assert status == _lib.STATUS_BAD_INDEX
    assert out[1].float().abs().max().item() == 0.0
    assert torch.equal(pool[0].cpu(), x.pool[0]) and torch.equal(pool[2].cpu(), x.pool[2])
    ro, rp = O.decode_pool(x.q[:1], x.k[:1], x.v[:1], x.pool, torch.tensor([1]), x.A_log,
                           x.a[:1], x.dt_bias, x.b[:1], x.scale)
    torch.testing.assert_close(out[:1].cpu().float(), ro.float(), **DECODE_OUT_TOL)
    torch.testing.assert_close(pool[1].cpu(), rp[1], **DECODE_STATE_TOL)


def test_large_batch_mtp_slices():
    """B=64, T=4, qk16_v32, a pool of 96 slots and an intermediate-state buffer
    ([96, 4, 32, 128, 128] fp32, 805 MB); the oracle checks three entries."""
    x = W.make_pool_decode_inputs(64, 4, 96, seed=60, device="cuda")
    out = torch.empty(64, 4, 32, 128, dtype=torch.bfloat16, device="cuda")
    pool = x.pool.clone()
    inter = torch.zeros(96, 4, 32, 128, 128, device="cuda")
    K.gdn_decode_pool(x.q, x.k, x.v, pool, x.indices, x.A_log, x.a, x.dt_bias, x.b, x.scale,
                      out, intermediate_states=inter)
    torch.cuda.synchronize()
    for bi in (0, 31, 63):
        sl = slice(bi, bi + 1)
        s = int(x.indices[bi])
        ro, rp = O.decode_pool(x.q[sl].cpu(), x.k[sl].cpu(), x.v[sl].cpu(), x.pool.cpu(),
                               torch.tensor([s]), x.A_log.cpu(), x.a[sl].cpu(),
                               x.dt_bias.cpu(), x.b[sl].cpu(), x.scale)
        torch.testing.assert_close(out[sl].cpu().float(), ro.float(), **DECODE_OUT_TOL)
        torch.testing.assert_close(pool[s].cpu(), rp[s], **DECODE_STATE_TOL)
