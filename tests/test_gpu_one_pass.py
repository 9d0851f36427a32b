"""The one-pass method against the oracle and against the two-pass method.

One pass: pass 1 keeps, per query row, the log2-sum of 2^(s * scale * log2 e)
over each 64-key segment it visits (a segment of block_size / 128 key tiles
when the block size is a multiple of 128), and once the row's lse2 is final
turns them into per-(head, query tile, bucket) partials,
sum_i 2^(segment sum - lse2_i).  It is the mass of the reference
(reference.py:113-124: per row, the softmax summed over the bucket's keys)
from the row statistics alone, so the scores are computed once.

Tolerances as in test_gpu_parity.py (max relative error per bucket): 1e-3 for
bf16/fp16 against the fp32-upcast oracle, 2e-5 for fp32.  The two methods are
fp32 arithmetic on the same scores and agree within 2e-5 for fp32 inputs and
1e-4 for bf16/fp16, where the one-pass kernel takes a quarter of its
exponentials from a degree-3 polynomial (7.5e-5 max relative error per
element) and the two-pass kernels from a degree-4 one.  causal_skip on/off
gives the same bits on either method.
"""

import numpy as np
import pytest
import torch

from _helpers import max_rel
from test_gpu_parity import oracle_for, run

import kvblockmass_b200 as kb

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 2e-5, torch.bfloat16: 1e-3, torch.float16: 1e-3}
AGREE = {torch.float32: 2e-5, torch.bfloat16: 1e-4, torch.float16: 1e-4}  # one pass vs two passes


def _qk(B, Hq, Hkv, N, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, N, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    return q, k, g


def _both(qd, kd, **kw):
    one = run(qd, kd, method="one_pass", **kw)
    two = run(qd, kd, method="two_pass", **kw)
    return one, two


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64), (torch.bfloat16, 256),
                                     (torch.float32, 64), (torch.float32, 128)])
@pytest.mark.parametrize("bs", [64, 128, 192, 256, 512])
@pytest.mark.parametrize("causal", [True, False])
def test_one_pass_matches_oracle_and_two_pass(cuda_device, dtype, D, bs, causal):
    N = 1500 if D <= 128 else 700  # neither a multiple of 128 nor of the block size
    q, k, _ = _qk(2, 8, 2, N, D, dtype, 61)
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    prep = kb.make_problem(qd, kd, causal=causal, block_size=bs)
    assert kb.method_of(prep) == "one_pass"
    one, two = _both(qd, kd, causal=causal, block_size=bs)
    want = oracle_for(q, k, causal=causal, block_size=bs)
    assert max_rel(one.cpu().numpy(), want) < TOL[dtype]
    assert max_rel(one.double().cpu().numpy(), two.double().cpu().numpy()) < AGREE[dtype]
    rows = 2 * 8 * N
    assert abs(float(one.double().sum()) - rows) < 1e-5 * rows  # sum rule
    skip_off = run(qd, kd, causal=causal, block_size=bs, causal_skip=False, method="one_pass")
    assert torch.equal(one, skip_off)
    assert torch.equal(one, run(qd, kd, causal=causal, block_size=bs))  # auto takes one pass, same bits


@pytest.mark.parametrize("mask", ["keys", "pairs", "batch_pairs", "query"])
def test_one_pass_masks(cuda_device, mask):
    B, N = 3, 900
    q, k, g = _qk(B, 8, 2, N, 128, torch.bfloat16, 62)
    kw = dict(causal=True, block_size=128)
    if mask == "keys":
        kw["attn_mask"] = torch.rand(N, generator=g) > 0.3
    elif mask == "pairs":
        kw["attn_mask"] = torch.rand(N, N, generator=g) > 0.4
        kw["attn_mask"][5:40] = False  # rows that keep nothing
    elif mask == "batch_pairs":
        kw["attn_mask"] = torch.rand(B, N, N, generator=g) > 0.4
    else:
        kw["query_mask"] = torch.rand(B, N, generator=g) > 0.2
    dev_kw = {n: (v.to(cuda_device) if isinstance(v, torch.Tensor) else v) for n, v in kw.items()}
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    one, two = _both(qd, kd, **dev_kw)
    want = oracle_for(q, k, **kw)
    assert max_rel(one.cpu().numpy(), want) < 1e-3
    assert max_rel(one.cpu().numpy(), two.cpu().numpy()) < AGREE[torch.bfloat16]
    assert torch.equal(one, run(qd, kd, causal_skip=False, method="one_pass", **dev_kw))


def test_one_pass_ragged_and_per_sequence(cuda_device):
    """Padded ragged lengths with a per-sequence output: one pass equals the
    two-pass method within 1e-4 and the oracle run on each sequence alone."""
    B, N = 4, 1100
    q, k, _ = _qk(B, 8, 2, N, 128, torch.bfloat16, 63)
    lens = torch.tensor([1100, 1, 517, 0], dtype=torch.int32)
    for b in range(B):  # padding past each length is never part of a pair, whatever it holds
        q[b, :, int(lens[b]):] = float("nan")
        k[b, :, int(lens[b]):] = float("nan")
    qd, kd, ld = q.to(cuda_device), k.to(cuda_device), lens.to(cuda_device)
    one, two = _both(qd, kd, causal=True, block_size=64, seq_lens=ld, per_sequence=True)
    assert one.shape == (B, (N + 63) // 64)
    assert max_rel(one.cpu().numpy(), two.cpu().numpy()) < AGREE[torch.bfloat16]
    for b in range(B):
        n = int(lens[b])
        want = np.zeros(one.shape[1])
        if n > 0:
            w = oracle_for(q[b:b + 1, :, :n], k[b:b + 1, :, :n], causal=True, block_size=64)
            want[:len(w)] = w
        assert max_rel(one[b].cpu().numpy(), want) < 1e-3
    # the packed layout of the same batch: same bits
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    qp = torch.cat([q[b, :, :int(lens[b])].transpose(0, 1) for b in range(B)])
    kp = torch.cat([k[b, :, :int(lens[b])].transpose(0, 1) for b in range(B)])
    packed = kb.block_mass_varlen(qp.to(cuda_device), kp.to(cuda_device), cu.to(cuda_device), max_seqlen=N,
                                  causal=True, block_size=64, per_sequence=True)
    torch.cuda.synchronize()
    assert torch.equal(packed, one)


def test_one_pass_unit_ranges_add_up(cuda_device):
    """Unit ranges of one problem add up to the whole (mass is a sum over units)."""
    q, k, _ = _qk(2, 8, 2, 2000, 128, torch.bfloat16, 64)
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    whole = run(qd, kd, causal=True, block_size=256)
    parts = sum(run(qd, kd, causal=True, block_size=256, units=(u, u + 1)).double() for u in range(4))
    assert max_rel(parts.cpu().numpy(), whole.double().cpu().numpy()) < 1e-6


def test_method_choice(cuda_device):
    q, k, _ = _qk(1, 4, 1, 256, 128, torch.bfloat16, 65)
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    assert kb.method_of(kb.make_problem(qd, kd, causal=True, block_size=64)) == "one_pass"
    # block sizes that are not a multiple of 64, and float64 (SIMT), take two passes
    assert kb.method_of(kb.make_problem(qd, kd, causal=True, block_size=48)) == "two_pass"
    assert kb.method_of(kb.make_problem(qd.double(), kd.double(), causal=True, block_size=64)) == "two_pass"
    assert kb.method_of(kb.make_problem(qd, kd, causal=True, block_size=64, method="two_pass")) == "two_pass"
    with pytest.raises(ValueError):
        kb.make_problem(qd, kd, causal=True, block_size=48, method="one_pass")
    with pytest.raises(ValueError):
        kb.make_problem(qd, kd, causal=True, block_size=64, method="fast")
    kb.check_device_errors(cuda_device)


def test_one_pass_llama3_8b_shape_against_two_pass(cuda_device):
    """Llama-3-8B attention shape at N=8192 (B1 Hq32 Hkv8 D128, bf16, per-head
    scale): the two methods agree within 1e-4 per bucket and the sum rule holds."""
    from kvblockmass_b200.workloads import WORKLOADS, make_inputs

    q, k, _, _ = make_inputs(WORKLOADS["llama3_8b_n32k"], N=8192)
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    one, two = _both(qd, kd, causal=True, block_size=64)
    assert max_rel(one.cpu().numpy(), two.cpu().numpy()) < AGREE[torch.bfloat16]
    assert abs(float(one.double().sum()) - 32 * 8192) < 1e-5 * 32 * 8192


@pytest.mark.parametrize("with_lse", [False, True])
def test_one_pass_with_paged_keys_key_mask_ragged_and_lse(cuda_device, with_lse):
    """The extensions together on the one-pass kernel: padded ragged lengths
    (NaN past each length), a per-batch key mask (the key bias step and its
    pre-pass), per-sequence output, the caller's LSE or not, and k read from a
    paged cache.  Against the two-pass method, the paged call (same bits as
    the dense one) and the oracle run on each sequence alone."""
    from test_gpu_lse import torch_lse
    from test_gpu_paged import paginate

    B, N, bs = 3, 1000, 128
    q, k, g = _qk(B, 8, 2, N, 128, torch.bfloat16, 66)
    lens_l = [1000, 640, 77]
    km = torch.rand(B, 1, N, generator=g) > 0.25
    for b, L in enumerate(lens_l):
        q[b, :, L:] = float("nan")
        k[b, :, L:] = float("nan")
    qd, kd, kmd = q.to(cuda_device), k.to(cuda_device), km.to(cuda_device)
    lens = torch.tensor(lens_l, dtype=torch.int32, device=cuda_device)
    lse = None
    if with_lse:
        lse = torch.full((B, 8, N), float("-inf"), device=cuda_device)
        for b, L in enumerate(lens_l):
            lse[b, :, :L] = torch_lse(qd[b:b + 1, :, :L], kd[b:b + 1, :, :L], True, attn_mask=kmd[b, 0, :L])[0].float()
    kw = dict(attn_mask=kmd, causal=True, block_size=bs, seq_lens=lens, per_sequence=True, lse=lse)
    one, two = _both(qd, kd, **kw)
    # with the caller's LSE both methods take the degree-4 polynomial
    assert max_rel(one.cpu().numpy(), two.cpu().numpy()) < (2e-5 if with_lse else AGREE[torch.bfloat16])
    for b, L in enumerate(lens_l):
        w = oracle_for(q[b:b + 1, :, :L], k[b:b + 1, :, :L], attn_mask=km[b, 0, :L], causal=True, block_size=bs)
        want = np.zeros(one.shape[1])
        want[:len(w)] = w
        assert max_rel(one[b].cpu().numpy(), want) < 1e-3
    cache, table = paginate(kd, 16)
    paged = kb.block_mass_paged(qd, cache, table.to(cuda_device), attn_mask=kmd, causal=True, block_size=bs,
                                seq_lens=lens, per_sequence=True, lse=lse)
    paged2 = kb.block_mass_paged(qd, cache, table.to(cuda_device), attn_mask=kmd, causal=True, block_size=bs,
                                 seq_lens=lens, per_sequence=True, lse=lse, method="two_pass")
    torch.cuda.synchronize()
    assert torch.equal(paged, one) and torch.equal(paged2, two)
    kb.check_device_errors(cuda_device)
