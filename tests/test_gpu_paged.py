"""Paged-KV input on the GPU, through the C ABI (``kvbm_block_mass_paged``).

The paged call gathers the named key rows into the workspace and runs the
dense kernels on them, so its result must have the SAME BITS as the dense
call on the keys the block table names (checked for every kernel path, unit
ranges, masks and the LSE input), and match the oracle on
``dense_keys_from_pages`` within the dense tolerances.  Unused pages and the
unused tail of the last page hold NaN: any read of them would show.
"""

import pytest
import torch

from _helpers import max_rel
from oracle.block_mass_np import dense_keys_from_pages
from test_gpu_parity import oracle_for

import kvblockmass_b200 as kb
from kvblockmass_b200 import _lib

pytestmark = pytest.mark.gpu


def paginate(k, page_size, extra_pages=3, seed=0):
    """Scatter dense k [B, H_kv, N, D] into a shuffled paged cache; NaN elsewhere."""
    B, Hkv, N, D = k.shape
    npg = -(-N // page_size)
    total = B * npg + extra_pages
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(total, generator=g)
    table = perm[:B * npg].reshape(B, npg).to(torch.int32)
    kp = torch.full((B, Hkv, npg * page_size, D), float("nan"), dtype=k.dtype, device=k.device)
    kp[:, :, :N] = k
    pages = kp.reshape(B, Hkv, npg, page_size, D).permute(0, 2, 3, 1, 4).reshape(B * npg, page_size, Hkv, D)
    cache = torch.full((total, page_size, Hkv, D), float("nan"), dtype=k.dtype, device=k.device)
    cache[table.flatten().long().to(k.device)] = pages
    return cache, table.to(k.device)


def _qk(B, Hq, Hkv, N, D, dtype, seed, device):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, N, D, generator=g).to(dtype).to(device)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype).to(device)
    return q, k


@pytest.mark.parametrize("dtype,D,path", [
    (torch.bfloat16, 128, 1), (torch.float16, 64, 1), (torch.float32, 64, 2),
    (torch.float64, 64, 0), (torch.bfloat16, 80, 1), (torch.bfloat16, 84, 0), (torch.float32, 128, 2),
    (torch.float32, 160, 0),
])
@pytest.mark.parametrize("page_size", [16, 128, 7])
def test_paged_bits_equal_dense(cuda_device, dtype, D, path, page_size):
    q, k = _qk(2, 8, 2, 777, D, dtype, 40 + page_size, cuda_device)
    cache, table = paginate(k, page_size, seed=page_size)
    prep = kb.make_problem(q, k, causal=True, block_size=64)
    assert kb.kernel_path(prep) == path
    want = kb.block_mass_b200(q, k, causal=True, block_size=64)
    got = kb.block_mass_paged(q, cache, table, causal=True, block_size=64)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    kb.check_device_errors()


def test_paged_matches_oracle(cuda_device):
    q, k = _qk(2, 8, 2, 1000, 128, torch.bfloat16, 41, cuda_device)
    cache, table = paginate(k, 16)
    got = kb.block_mass_paged(q, cache, table, causal=True, block_size=16)
    kd = dense_keys_from_pages(cache.float().cpu().numpy(), table.cpu().numpy(), 1000)
    want = oracle_for(q.cpu(), torch.from_numpy(kd), causal=True, block_size=16)
    assert max_rel(got.cpu().numpy(), want) < 1e-3
    assert abs(float(got.double().sum()) - 2 * 8 * 1000) < 1e-5 * 2 * 8 * 1000


@pytest.mark.parametrize("units", [(0, 1), (1, 3), (2, 6), (5, 6), (3, 6), (0, 6)])
def test_paged_unit_ranges(cuda_device, units):
    """A unit range gathers only its batch x kv-head box; the bits match the dense call."""
    q, k = _qk(3, 8, 2, 500, 128, torch.bfloat16, 42, cuda_device)
    cache, table = paginate(k, 32)
    want = kb.block_mass_b200(q, k, causal=True, block_size=64, units=units)
    got = kb.block_mass_paged(q, cache, table, causal=True, block_size=64, units=units)
    assert torch.equal(got, want)


def test_paged_unit_ranges_sum_to_whole(cuda_device):
    q, k = _qk(2, 8, 4, 600, 64, torch.float16, 43, cuda_device)
    cache, table = paginate(k, 64)
    whole = kb.block_mass_paged(q, cache, table, causal=True, block_size=64)
    parts = sum(kb.block_mass_paged(q, cache, table, causal=True, block_size=64, units=(u, u + 1)).double()
                for u in range(8))
    assert max_rel(whole.double().cpu().numpy(), parts.cpu().numpy()) < 1e-6


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float32, 64)])
def test_paged_with_masks(cuda_device, dtype, D):
    q, k = _qk(2, 8, 2, 600, D, dtype, 44, cuda_device)
    g = torch.Generator().manual_seed(45)
    pm = (torch.rand(2, 600, 600, generator=g) > 0.2).to(cuda_device)
    km = (torch.rand(2, 1, 600, generator=g) > 0.1).to(cuda_device)
    qm = (torch.rand(2, 600, generator=g) > 0.1).to(cuda_device)
    cache, table = paginate(k, 16)
    for kw in ({"attn_mask": pm}, {"attn_mask": km, "query_mask": qm}, {"attn_mask": pm, "query_mask": qm}):
        want = kb.block_mass_b200(q, k, causal=True, block_size=100, **kw)
        got = kb.block_mass_paged(q, cache, table, causal=True, block_size=100, **kw)
        assert torch.equal(got, want)
        got_u = kb.block_mass_paged(q, cache, table, causal=True, block_size=100, units=(3, 4), **kw)
        assert torch.equal(got_u, kb.block_mass_b200(q, k, causal=True, block_size=100, units=(3, 4), **kw))


def test_paged_with_lse(cuda_device):
    q, k = _qk(2, 8, 2, 900, 128, torch.bfloat16, 46, cuda_device)
    cache, table = paginate(k, 16)
    s = (q.float() @ k.float().repeat_interleave(4, dim=1).transpose(-1, -2)) / 128 ** 0.5
    causal = torch.ones(900, 900, dtype=torch.bool, device=cuda_device).tril()
    lse = s.masked_fill(~causal, float("-inf")).logsumexp(-1)
    want = kb.block_mass_b200(q, k, causal=True, block_size=64, lse=lse)
    got = kb.block_mass_paged(q, cache, table, causal=True, block_size=64, lse=lse)
    assert torch.equal(got, want)
    got_u = kb.block_mass_paged(q, cache, table, causal=True, block_size=64, lse=lse, units=(1, 3))
    assert torch.equal(got_u, kb.block_mass_b200(q, k, causal=True, block_size=64, lse=lse, units=(1, 3)))


def test_paged_strided_cache_and_int64_table(cuda_device):
    """A cache view with a non-unit head-dim stride takes the element-wise gather."""
    q, k = _qk(1, 4, 2, 300, 64, torch.float32, 47, cuda_device)
    cache, table = paginate(k, 16)
    wide = torch.full(cache.shape[:3] + (128,), float("nan"), device=cuda_device)
    wide[..., ::2] = cache
    view = wide[..., ::2]
    assert view.stride(3) == 2
    want = kb.block_mass_b200(q, k, causal=False, block_size=32)
    got = kb.block_mass_paged(q, view, table.long(), causal=False, block_size=32)
    assert torch.equal(got, want)


def test_bad_page_id_is_reported_not_read(cuda_device):
    """An out-of-range page id is skipped (its keys read as zeros) and reported."""
    q, k = _qk(2, 8, 2, 256, 128, torch.bfloat16, 48, cuda_device)
    cache, table = paginate(k, 16)
    kb.check_device_errors()
    bad = table.clone()
    bad[1, 3] = cache.shape[0] + 1000
    bad[0, 0] = -5
    got = kb.block_mass_paged(q, cache, bad, causal=True, block_size=64)
    kz = k.clone()
    kz[1, :, 48:64] = 0
    kz[0, :, 0:16] = 0
    want = kb.block_mass_b200(q, kz, causal=True, block_size=64)
    assert torch.equal(got, want)
    with pytest.raises(RuntimeError, match=f"kvbm error {_lib.KVBM_ERR_PAGE}"):
        kb.check_device_errors()
    kb.check_device_errors()  # the word was cleared


def test_paged_workspace_errors(cuda_device):
    q, k = _qk(1, 8, 2, 256, 128, torch.bfloat16, 49, cuda_device)
    cache, table = paginate(k, 16)
    pp = kb.make_paged_problem(q, cache, table, causal=True, block_size=64)
    need = kb.paged_workspace_bytes(pp)
    assert need >= 2 * 256 * 128 * 2
    small = torch.empty(need - 256, dtype=torch.uint8, device=cuda_device)
    out = torch.empty(4, device=cuda_device)
    lib = _lib.load()
    import ctypes
    code = lib.kvbm_block_mass_paged(ctypes.byref(pp.prep.prob), ctypes.byref(pp.kv), None, None, out.data_ptr(),
                                     small.data_ptr(), small.numel(), torch.cuda.current_stream().cuda_stream)
    assert code == _lib.KVBM_ERR_WORKSPACE
    ws = torch.empty(need, dtype=torch.uint8, device=cuda_device)
    got = kb.run_paged(pp, out=out, workspace=ws)
    assert torch.equal(got, kb.block_mass_b200(q, k, causal=True, block_size=64))


@pytest.mark.slow
def test_paged_llama3_8b_full_size(cuda_device):
    """Llama-3-8B attention shape, N=32768, 16-key pages: same bits as dense."""
    q, k = _qk(1, 32, 8, 32768, 128, torch.bfloat16, 50, cuda_device)
    cache, table = paginate(k, 16)
    want = kb.block_mass_b200(q, k, causal=True, block_size=16)
    got = kb.block_mass_paged(q, cache, table, causal=True, block_size=16)
    assert torch.equal(got, want)
    assert abs(float(got.double().sum()) - 32 * 32768) < 1e-5 * 32 * 32768
