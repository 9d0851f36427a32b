"""Pair masks ([N, N] / [B, N, N]) on the tensor-core paths, against the oracle.

The tensor-core kernels take a pair mask as packed bits (one row-major copy
for the row pass, one transposed copy for the column pass) with the key and
query masks folded in.  Tolerances as in test_gpu_parity.py.
"""

import pytest
import torch

from _helpers import max_rel
from test_gpu_parity import oracle_for, run

import kvblockmass_b200 as kb

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 2e-5, torch.bfloat16: 1e-3, torch.float16: 1e-3}


def _qk(B, Hq, Hkv, N, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, N, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    return q, k, g


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64), (torch.float32, 64)])
@pytest.mark.parametrize("causal", [True, False])
def test_random_pair_mask_tensor_core(cuda_device, dtype, D, causal):
    q, k, g = _qk(2, 8, 2, 1000, D, dtype, 31)
    pm = torch.rand(1000, 1000, generator=g) > 0.3
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    prep = kb.make_problem(qd, kd, attn_mask=pm.to(cuda_device), causal=causal, block_size=64)
    assert kb.kernel_path(prep) in (1, 2)
    got = run(qd, kd, attn_mask=pm.to(cuda_device), causal=causal, block_size=64)
    want = oracle_for(q, k, attn_mask=pm, causal=causal, block_size=64)
    assert max_rel(got.cpu().numpy(), want) < TOL[dtype]
    skip_off = run(qd, kd, attn_mask=pm.to(cuda_device), causal=causal, block_size=64, causal_skip=False)
    assert torch.equal(got, skip_off)


def test_batch_pair_mask_with_key_and_query_masks(cuda_device):
    q, k, g = _qk(3, 8, 2, 700, 128, torch.bfloat16, 32)
    pm = torch.rand(3, 700, 700, generator=g) > 0.2
    km = torch.rand(700, generator=g) > 0.1
    qm = torch.rand(3, 700, generator=g) > 0.1
    # the oracle takes one attn_mask: fold the key mask into the pair mask for it
    want = oracle_for(q, k, attn_mask=pm & km[None, None, :], query_mask=qm, causal=True, block_size=100)
    got = run(q.to(cuda_device), k.to(cuda_device), attn_mask=(pm & km[None, None, :]).to(cuda_device),
              query_mask=qm.to(cuda_device), causal=True, block_size=100)
    assert max_rel(got.cpu().numpy(), want) < 1e-3


def test_sliding_window_and_dead_rows(cuda_device):
    N, w = 1500, 200
    q, k, _ = _qk(1, 4, 1, N, 128, torch.bfloat16, 33)
    i = torch.arange(N)
    pm = (i[:, None] - i[None, :]).abs() < w        # a band around the diagonal
    pm[10:20, :] = False                             # rows that keep nothing
    got = run(q.to(cuda_device), k.to(cuda_device), attn_mask=pm.to(cuda_device), causal=True, block_size=64)
    want = oracle_for(q, k, attn_mask=pm, causal=True, block_size=64)
    assert max_rel(got.cpu().numpy(), want) < 1e-3
    alive = N - 10
    assert abs(float(got.double().sum()) - 4 * alive) <= 1e-5 * 4 * alive


def test_pair_mask_matches_query_mask_form(cuda_device):
    """Dead rows written as a pair mask equal the same rows dropped by query_mask."""
    q, k, g = _qk(2, 8, 2, 513, 64, torch.bfloat16, 34)
    qm = torch.rand(2, 513, generator=g) > 0.2
    pm = qm[:, :, None].expand(2, 513, 513).contiguous()
    a = run(q.to(cuda_device), k.to(cuda_device), query_mask=qm.to(cuda_device), causal=True, block_size=64)
    b = run(q.to(cuda_device), k.to(cuda_device), attn_mask=pm.to(cuda_device), causal=True, block_size=64)
    assert max_rel(a.cpu().numpy(), b.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64), (torch.float32, 64)])
@pytest.mark.parametrize("per_batch", [False, True])
def test_key_mask_drops_non_finite_keys(cuda_device, dtype, D, per_batch):
    """Keys dropped by a key mask add nothing, whatever their rows of k hold:
    the reference's masked_fill (reference.py:113-114) discards NaN and
    infinite scores too.  The tensor-core kernels fold a key mask into the
    accumulator as a -inf bias; a masked key holding NaN or inf makes the
    tile take the select instead.  Same bits as with those rows zeroed."""
    B, N = 2, 1000
    q, k, g = _qk(B, 8, 2, N, D, dtype, 35)
    km = torch.rand(B, 1, N, generator=g) > 0.3 if per_batch else torch.rand(N, generator=g) > 0.3
    dropped = (~km[:, 0] if per_batch else ~km[None].expand(B, N))
    bad = k.clone()
    zero = k.clone()
    for b in range(B):
        idx = torch.nonzero(dropped[b]).flatten()
        bad[b, :, idx[::3]] = float("nan")
        bad[b, :, idx[1::3]] = float("inf")
        bad[b, :, idx[2::3]] = -float("inf")
        zero[b, :, idx] = 0
    kmd = km.to(cuda_device)
    got = run(q.to(cuda_device), bad.to(cuda_device), attn_mask=kmd, causal=True, block_size=64)
    clean = run(q.to(cuda_device), zero.to(cuda_device), attn_mask=kmd, causal=True, block_size=64)
    assert torch.isfinite(got).all()
    assert torch.equal(got, clean)
    if not per_batch:
        want = oracle_for(q, zero, attn_mask=km, causal=True, block_size=64)
        assert max_rel(got.cpu().numpy(), want) < TOL[dtype]
    kb.check_device_errors(cuda_device)
