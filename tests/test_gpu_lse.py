"""Block mass from a caller-provided row log-sum-exp (no row statistics pass).

An attention forward already knows each query row's LSE; handing it to
``block_mass_b200(..., lse=...)`` (C ABI ``kvbm_block_mass_lse``) must give
the same mass as the two-pass computation.  The LSE here is computed in
float64 with torch on the GPU (a plain restatement of softmax's denominator,
not the library's pass 1).
"""

import pytest
import torch

from _helpers import max_rel
from test_gpu_parity import oracle_for, run

import kvblockmass_b200 as kb

pytestmark = pytest.mark.gpu


def torch_lse(q, k, causal, scale=None, attn_mask=None, query_mask=None):
    """[B, H_q, N] natural-log LSE of the kept scores, float64, -inf for empty rows."""
    B, Hq, N, D = q.shape
    G = Hq // k.shape[1]
    scale = 1.0 / D ** 0.5 if scale is None else scale
    kf = k.double().repeat_interleave(G, dim=1)
    s = torch.matmul(q.double(), kf.transpose(-1, -2)) * scale
    keep = torch.ones(N, N, dtype=torch.bool, device=q.device)
    if causal:
        keep = torch.tril(keep)
    keep = keep.expand(B, 1, N, N)
    if attn_mask is not None:
        m = attn_mask.to(q.device)
        keep = keep & (m.view(1, 1, 1, N) if m.dim() == 1 else m.view(-1, 1, N, N) if m.dim() == 3 else m.view(1, 1, N, N))
    if query_mask is not None:
        keep = keep & query_mask.to(q.device).view(B, 1, N, 1)
    s = s.masked_fill(~keep, float("-inf"))
    return torch.logsumexp(s, dim=-1)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("causal", [True, False])
def test_lse_input_matches_two_pass(cuda_device, dtype, causal):
    g = torch.Generator().manual_seed(5)
    q = torch.randn(2, 8, 700, 128, generator=g).to(dtype).to(cuda_device)
    k = torch.randn(2, 2, 700, 128, generator=g).to(dtype).to(cuda_device)
    lse = torch_lse(q, k, causal).float()
    a = run(q, k, causal=causal, block_size=64)
    b = run(q, k, causal=causal, block_size=64, lse=lse)
    # (the one-pass call without an LSE takes a quarter of its bf16 exponentials
    # from a degree-3 polynomial: 1e-4; fp32 runs degree 4 throughout)
    assert max_rel(b.cpu().numpy(), a.cpu().numpy()) < (1e-4 if dtype == torch.bfloat16 else 2e-5)
    # the same LSE through the two-pass method (pass 2 alone): same mass
    c = run(q, k, causal=causal, block_size=64, lse=lse, method="two_pass")
    assert max_rel(b.cpu().numpy(), c.cpu().numpy()) < 2e-5
    want = oracle_for(q, k, causal=causal, block_size=64)
    assert max_rel(b.cpu().numpy(), want) < (1e-3 if dtype == torch.bfloat16 else 2e-5)


def test_lse_input_masks_and_dead_rows(cuda_device):
    g = torch.Generator().manual_seed(6)
    B, Hq, Hkv, N, D = 2, 4, 2, 500, 64
    q = torch.randn(B, Hq, N, D, generator=g).to(torch.bfloat16).to(cuda_device)
    k = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).to(cuda_device)
    km = (torch.rand(N, generator=g) > 0.2).to(cuda_device)
    qm = (torch.rand(B, N, generator=g) > 0.2).to(cuda_device)
    lse = torch_lse(q, k, True, attn_mask=km, query_mask=qm).float()
    assert bool(torch.isinf(lse).any())        # dropped rows carry -inf
    a = run(q, k, attn_mask=km, query_mask=qm, causal=True, block_size=50)
    b = run(q, k, attn_mask=km, query_mask=qm, causal=True, block_size=50, lse=lse)
    assert max_rel(b.cpu().numpy(), a.cpu().numpy()) < 2e-5
    # the same without query_mask: the -inf LSE alone must zero the dropped rows
    c = run(q, k, attn_mask=km, causal=True, block_size=50, lse=lse)
    assert max_rel(c.cpu().numpy(), a.cpu().numpy()) < 2e-5


def test_lse_input_pair_mask_simt_and_strided(cuda_device):
    g = torch.Generator().manual_seed(7)
    B, Hq, Hkv, N, D = 1, 4, 1, 300, 32
    q = torch.randn(B, Hq, N, D, generator=g, dtype=torch.float64).float().to(cuda_device)
    k = torch.randn(B, Hkv, N, D, generator=g, dtype=torch.float64).float().to(cuda_device)
    pm = (torch.rand(N, N, generator=g) > 0.5)
    pm[0, :] = False                                   # a row that keeps nothing
    pm = pm.to(cuda_device)
    lse = torch_lse(q, k, True, attn_mask=pm).float()
    lse_view = lse.transpose(1, 2).contiguous().transpose(1, 2)   # [B, H, N] view, N-major storage
    a = run(q, k, attn_mask=pm, causal=True, block_size=32)
    b = run(q, k, attn_mask=pm, causal=True, block_size=32, lse=lse_view)
    assert max_rel(b.cpu().numpy(), a.cpu().numpy()) < 2e-5


def test_lse_input_shape_checked(cuda_device):
    q = torch.randn(1, 2, 64, 64, device=cuda_device)
    k = torch.randn(1, 1, 64, 64, device=cuda_device)
    with pytest.raises(ValueError):
        kb.block_mass_b200(q, k, lse=torch.zeros(1, 2, 63, device=cuda_device))
