"""Ragged batches on the GPU, through the C ABI (``kvbm_block_mass_ex``).

Padded layout with ``seq_lens``, packed (varlen) layout with ``cu_seqlens``,
per-sequence output, and their combinations with a paged cache, the LSE
input and unit ranges.  Parity: the oracle runs the reference algorithm on
each sequence alone (``block_mass_ragged``); padding positions hold NaN so
that any read of them into a pair would show.  Padded and packed layouts of
the same batch give the same bits, and so does a batch whose lengths all
equal N against the uniform kernels.
"""

import pytest
import torch

from _helpers import max_rel
from oracle.block_mass_np import block_mass_ragged
from test_gpu_paged import paginate

import kvblockmass_b200 as kb

pytestmark = pytest.mark.gpu

TOL = {torch.float64: 1e-9, torch.float32: 2e-5, torch.bfloat16: 1e-3, torch.float16: 1e-3}


def ragged_inputs(B, Hq, Hkv, N, D, dtype, lens, seed, device):
    """Padded q/k [B, H, N, D] with NaN past each length, plus the packed copies."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, N, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    for b, L in enumerate(lens):
        q[b, :, L:] = float("nan")
        k[b, :, L:] = float("nan")
    qp = torch.cat([q[b, :, :L].transpose(0, 1) for b, L in enumerate(lens)])   # [T, Hq, D]
    kp = torch.cat([k[b, :, :L].transpose(0, 1) for b, L in enumerate(lens)])
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    lens_t = torch.tensor(lens, dtype=torch.int32)
    return (q.to(device), k.to(device), qp.to(device), kp.to(device), cu.to(device), lens_t.to(device),
            q, k)


def oracle(q_cpu, k_cpu, lens, **kw):
    qn, kn = q_cpu, k_cpu
    if qn.dtype in (torch.bfloat16, torch.float16):
        qn, kn = qn.float(), kn.float()
    am = kw.pop("attn_mask", None)
    qm = kw.pop("query_mask", None)
    return block_mass_ragged(qn.numpy(), kn.numpy(), lens, attn_mask=None if am is None else am.cpu().numpy(),
                             query_mask=None if qm is None else qm.cpu().numpy(), **kw)


LENS = [1000, 333, 128, 1, 0, 777]


@pytest.mark.parametrize("dtype,D,path", [
    (torch.bfloat16, 128, 1), (torch.float16, 64, 1), (torch.float32, 64, 2),
    (torch.float64, 64, 0), (torch.bfloat16, 80, 1), (torch.bfloat16, 84, 0), (torch.float32, 128, 2),
])
@pytest.mark.parametrize("causal", [True, False])
def test_ragged_padded_and_packed_vs_oracle(cuda_device, dtype, D, path, causal):
    q, k, qp, kp, cu, lens, q_cpu, k_cpu = ragged_inputs(6, 8, 2, 1000, D, dtype, LENS, 60, cuda_device)
    assert kb.kernel_path(kb.make_problem(q, k, seq_lens=lens)) == path
    got = kb.block_mass_b200(q, k, causal=causal, block_size=64, seq_lens=lens)
    want = oracle(q_cpu, k_cpu, LENS, causal=causal, block_size=64)
    assert max_rel(got.cpu().numpy(), want) < TOL[dtype]
    # the packed layout of the same batch: same bits
    packed = kb.block_mass_varlen(qp, kp, cu, max_seqlen=1000, causal=causal, block_size=64)
    assert torch.equal(packed, got)
    # causal_skip off: same bits
    assert torch.equal(kb.block_mass_b200(q, k, causal=causal, block_size=64, seq_lens=lens, causal_skip=False),
                       got)
    kb.check_device_errors()


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float32, 64), (torch.float64, 32)])
def test_full_lengths_match_uniform_kernels(cuda_device, dtype, D):
    g = torch.Generator().manual_seed(61)
    q = torch.randn(2, 8, 900, D, generator=g).to(dtype).to(cuda_device)
    k = torch.randn(2, 2, 900, D, generator=g).to(dtype).to(cuda_device)
    lens = torch.tensor([900, 900], dtype=torch.int32, device=cuda_device)
    a = kb.block_mass_b200(q, k, causal=True, block_size=64)
    b = kb.block_mass_b200(q, k, causal=True, block_size=64, seq_lens=lens)
    assert torch.equal(a, b)


def test_per_sequence_rows(cuda_device):
    q, k, qp, kp, cu, lens, q_cpu, k_cpu = ragged_inputs(6, 8, 2, 1000, 128, torch.bfloat16, LENS, 62,
                                                         cuda_device)
    per = kb.block_mass_b200(q, k, causal=True, block_size=100, seq_lens=lens, per_sequence=True)
    assert per.shape == (6, 10)
    want = oracle(q_cpu, k_cpu, LENS, causal=True, block_size=100, per_sequence=True)
    assert max_rel(per.cpu().numpy(), want) < 1e-3
    for b, L in enumerate(LENS):
        assert abs(float(per[b].double().sum()) - 8 * L) <= 1e-5 * max(1, 8 * L)
        assert torch.all(per[b, -(-L // 100):] == 0)
        if L:
            # one sequence alone, dense: the same mass up to the fp64 reduce's grouping
            alone = kb.block_mass_b200(q[b:b + 1, :, :L], k[b:b + 1, :, :L], causal=True, block_size=100)
            assert max_rel(per[b, :alone.numel()].double().cpu().numpy(), alone.double().cpu().numpy()) < 1e-6
    summed = kb.block_mass_b200(q, k, causal=True, block_size=100, seq_lens=lens)
    assert max_rel(per.double().sum(0).cpu().numpy(), summed.double().cpu().numpy()) < 1e-6
    packed = kb.block_mass_varlen(qp, kp, cu, causal=True, block_size=100, per_sequence=True)
    assert torch.equal(packed, per)
    # per-sequence output of a unit range: rows outside the range are zeros
    part = kb.block_mass_b200(q, k, causal=True, block_size=100, seq_lens=lens, per_sequence=True, units=(3, 7))
    assert torch.all(part[0] == 0) and torch.all(part[4:] == 0)


def test_ragged_with_masks(cuda_device):
    q, k, qp, kp, cu, lens, q_cpu, k_cpu = ragged_inputs(6, 8, 2, 1000, 128, torch.bfloat16, LENS, 63,
                                                         cuda_device)
    g = torch.Generator().manual_seed(64)
    km = torch.rand(6, 1, 1000, generator=g) > 0.2
    pm = torch.rand(6, 1000, 1000, generator=g) > 0.3
    qm = torch.rand(6, 1000, generator=g) > 0.1
    for kw in ({"attn_mask": km}, {"attn_mask": pm, "query_mask": qm}):
        dev_kw = {n: v.to(cuda_device) for n, v in kw.items()}
        got = kb.block_mass_b200(q, k, causal=True, block_size=64, seq_lens=lens, **dev_kw)
        want = oracle(q_cpu, k_cpu, LENS, causal=True, block_size=64, **kw)
        assert max_rel(got.cpu().numpy(), want) < 1e-3
        assert torch.equal(kb.block_mass_varlen(qp, kp, cu, max_seqlen=1000, causal=True, block_size=64, **dev_kw),
                           got)


def test_ragged_with_lse(cuda_device):
    lens_l = [700, 129, 300]
    q, k, qp, kp, cu, lens, q_cpu, k_cpu = ragged_inputs(3, 8, 2, 700, 128, torch.bfloat16, lens_l, 65,
                                                         cuda_device)
    lse = torch.full((3, 8, 700), float("nan"), device=cuda_device)
    for b, L in enumerate(lens_l):
        s = (q[b, :, :L].float() @ k[b, :, :L].float().repeat_interleave(4, 0).transpose(-1, -2)) / 128 ** 0.5
        causal = torch.ones(L, L, dtype=torch.bool, device=cuda_device).tril()
        lse[b, :, :L] = s.masked_fill(~causal, float("-inf")).logsumexp(-1)
    got = kb.block_mass_b200(q, k, causal=True, block_size=64, seq_lens=lens, lse=lse)
    want = oracle(q_cpu, k_cpu, lens_l, causal=True, block_size=64)
    assert max_rel(got.cpu().numpy(), want) < 2e-3
    lse_packed = torch.cat([lse[b, :, :L] for b, L in enumerate(lens_l)], dim=1)   # [Hq, T]
    packed = kb.block_mass_varlen(qp, kp, cu, max_seqlen=700, causal=True, block_size=64, lse=lse_packed)
    assert torch.equal(packed, got)


def test_ragged_unit_shards_sum_to_whole(cuda_device):
    q, k, qp, kp, cu, lens, q_cpu, k_cpu = ragged_inputs(6, 8, 2, 1000, 64, torch.float16, LENS, 66,
                                                         cuda_device)
    whole = kb.block_mass_varlen(qp, kp, cu, max_seqlen=1000, causal=True, block_size=64)
    parts = sum(kb.block_mass_varlen(qp, kp, cu, max_seqlen=1000, causal=True, block_size=64,
                                     units=(u, min(12, u + 5))).double() for u in range(0, 12, 5))
    assert max_rel(whole.double().cpu().numpy(), parts.cpu().numpy()) < 1e-6


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float32, 64)])
def test_paged_ragged_and_packed(cuda_device, dtype, D):
    """Paged k with per-sequence lengths: table entries past a length are -1 and
    never read; padded or packed q give the bits of the dense ragged call."""
    q, k, qp, kp, cu, lens, q_cpu, k_cpu = ragged_inputs(6, 8, 2, 1000, D, dtype, LENS, 67, cuda_device)
    cache, table = paginate(torch.nan_to_num(k, nan=0.0), 16)
    for b, L in enumerate(LENS):
        table[b, -(-L // 16):] = -1
    want = kb.block_mass_b200(q, k, causal=True, block_size=16, seq_lens=lens)
    got = kb.block_mass_paged(q, cache, table, causal=True, block_size=16, seq_lens=lens)
    assert torch.equal(got, want)
    got_p = kb.block_mass_paged(qp, cache, table, causal=True, block_size=16, cu_seqlens=cu, max_seqlen=1000)
    assert torch.equal(got_p, want)
    per = kb.block_mass_paged(q, cache, table, causal=True, block_size=16, seq_lens=lens, per_sequence=True,
                              units=(2, 5))
    want_per = kb.block_mass_b200(q, k, causal=True, block_size=16, seq_lens=lens, per_sequence=True,
                                  units=(2, 5))
    assert torch.equal(per, want_per)
    kb.check_device_errors()  # no table entry past a length was read


@pytest.mark.slow
def test_ragged_serving_batch_full_size(cuda_device):
    """A serving-like packed batch (Llama-3-8B heads, 6 sequences, 32k tokens in
    all): the sum rule per sequence and the bits of the padded layout."""
    lens_l = [16384, 8192, 4096, 2048, 1024, 1000]
    q, k, qp, kp, cu, lens, _, _ = ragged_inputs(6, 32, 8, 16384, 128, torch.bfloat16, lens_l, 68, cuda_device)
    per = kb.block_mass_varlen(qp, kp, cu, causal=True, block_size=64, per_sequence=True)
    for b, L in enumerate(lens_l):
        assert abs(float(per[b].double().sum()) - 32 * L) <= 1e-5 * 32 * L
    padded = kb.block_mass_b200(q, k, causal=True, block_size=64, seq_lens=lens, per_sequence=True)
    assert torch.equal(per, padded)


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float64, 64), (torch.bfloat16, 84)])
def test_cu_seqlens_past_total_are_clamped(cuda_device, dtype, D):
    """A cu_seqlens entry past total_tokens reads nothing past the packed tensors:
    the sequence is cut at total_tokens (same result as the clamped offsets)."""
    lens_l = [300, 200]
    q, k, qp, kp, cu, lens, _, _ = ragged_inputs(2, 8, 2, 300, D, dtype, lens_l, 69, cuda_device)
    bad = torch.tensor([0, 300, 700], dtype=torch.int32, device=cuda_device)   # total is 500
    want = kb.block_mass_varlen(qp, kp, cu, max_seqlen=300, causal=True, block_size=64)
    got = kb.block_mass_varlen(qp, kp, bad, max_seqlen=300, causal=True, block_size=64)
    assert torch.equal(got, want)
    lse = torch.zeros(8, qp.shape[0], device=cuda_device)
    kb.block_mass_varlen(qp, kp, bad, max_seqlen=300, causal=True, block_size=64, lse=lse)
    torch.cuda.synchronize()


def test_decreasing_cu_seqlens_are_reported(cuda_device):
    """The tensor-core pass 1 of a packed batch launches at most
    ceil(total_tokens / 128) + B query tiles per kv-head.  cu_seqlens that
    decrease (so that the clamped sequences overlap and hold more rows than
    total_tokens) exceed that: the call reads nothing out of range and reports
    it through the device error word."""
    g = torch.Generator().manual_seed(70)
    T = 500
    qp = torch.randn(T, 8, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    kp = torch.randn(T, 2, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    kb.check_device_errors(cuda_device)
    good = torch.tensor([0, 250, 500], dtype=torch.int32, device=cuda_device)
    kb.block_mass_varlen(qp, kp, good, max_seqlen=500, causal=True, block_size=64)
    kb.check_device_errors(cuda_device)  # monotone offsets: no report
    bad = torch.tensor([0, 500, 0, 500], dtype=torch.int32, device=cuda_device)  # 500 + 0 + 500 rows
    kb.block_mass_varlen(qp, kp, bad, max_seqlen=500, causal=True, block_size=64)
    with pytest.raises(RuntimeError):
        kb.check_device_errors(cuda_device)
    kb.check_device_errors(cuda_device)  # the read cleared it
    assert torch.isfinite(kb.block_mass_varlen(qp, kp, good, max_seqlen=500, causal=True, block_size=64)).all()


@pytest.mark.slow
@pytest.mark.parametrize("dtype,D,N,short", [(torch.bfloat16, 128, 262144, 100000), (torch.float64, 32, 40000, 20000)])
def test_wide_query_chunks_past_64_chunks(cuda_device, dtype, D, N, short):
    """Past 64 query chunks per unit the chunks widen, keeping the partials O(N)
    (tensor-core path above N=131072, SIMT above N=32768).  A short sequence in
    the same call, which gets the wide chunks, has the mass of that sequence
    computed alone with the normal chunks (up to the fp64 reduce's grouping)."""
    g = torch.Generator().manual_seed(91)
    q = torch.randn(2, 4, N, D, generator=g).to(dtype).to(cuda_device)
    k = torch.randn(2, 1, N, D, generator=g).to(dtype).to(cuda_device)
    lens = torch.tensor([N, short], dtype=torch.int32, device=cuda_device)
    per = kb.block_mass_b200(q, k, causal=True, block_size=256, seq_lens=lens, per_sequence=True)
    for b, L in enumerate((N, short)):
        assert abs(float(per[b].double().sum()) - 4 * L) <= 1e-5 * 4 * L
    alone = kb.block_mass_b200(q[1:, :, :short], k[1:, :, :short], causal=True, block_size=256)
    tol = 1e-12 if dtype == torch.float64 else 1e-6
    assert max_rel(per[1, :alone.numel()].double().cpu().numpy(), alone.double().cpu().numpy()) < tol
    assert torch.all(per[1, alone.numel():] == 0)
