"""Paged-KV input, host side (no GPU): C validation, workspace sizing, the
Python wrapper's argument checks and the oracle's definition of the layout."""

import ctypes

import numpy as np
import pytest
import torch

from kvblockmass_b200 import _lib
from kvblockmass_b200.ops import make_paged_problem, paged_workspace_bytes
from oracle.block_mass_np import block_mass_stream, dense_keys_from_pages
from test_abi import _problem


def _kv(num_pages=8, page_size=16, Hkv=2, D=64, max_pages=8, table_stride=None):
    kv = _lib.PagedKV()
    kv.k_cache = 4096
    for i, s in enumerate((page_size * Hkv * D, Hkv * D, D, 1)):
        kv.cache_stride[i] = s
    kv.num_pages, kv.page_size = num_pages, page_size
    kv.block_table = 8192
    kv.block_table_stride = max_pages if table_stride is None else table_stride
    kv.max_pages = max_pages
    return kv


def test_validate_paged_codes():
    lib = _lib.load()
    p = _problem(shape=(2, 8, 2, 128, 64))
    assert lib.kvbm_validate_paged(ctypes.byref(p), ctypes.byref(_kv())) == _lib.KVBM_OK
    assert lib.kvbm_validate_paged(ctypes.byref(p), ctypes.byref(_kv(max_pages=7))) == _lib.KVBM_ERR_SHAPE
    assert lib.kvbm_validate_paged(ctypes.byref(p), ctypes.byref(_kv(page_size=0))) == _lib.KVBM_ERR_SHAPE
    assert lib.kvbm_validate_paged(ctypes.byref(p), ctypes.byref(_kv(num_pages=0))) == _lib.KVBM_ERR_SHAPE
    kv = _kv()
    kv.block_table = None
    assert lib.kvbm_validate_paged(ctypes.byref(p), ctypes.byref(kv)) == _lib.KVBM_ERR_NULL
    kv = _kv()
    kv.k_cache = None
    assert lib.kvbm_validate_paged(ctypes.byref(p), ctypes.byref(kv)) == _lib.KVBM_ERR_NULL
    kv = _kv()
    kv.cache_stride[2] = -1
    assert lib.kvbm_validate_paged(ctypes.byref(p), ctypes.byref(kv)) == _lib.KVBM_ERR_SHAPE
    # the dense checks still apply (p.k is ignored: a NULL k is fine)
    p.k = None
    assert lib.kvbm_validate_paged(ctypes.byref(p), ctypes.byref(_kv())) == _lib.KVBM_OK
    bad = _problem(shape=(1, 6, 4, 8, 4))
    assert lib.kvbm_validate_paged(ctypes.byref(bad), ctypes.byref(_kv(Hkv=4, D=4))) == _lib.KVBM_ERR_GQA
    assert lib.kvbm_validate_paged(None, ctypes.byref(_kv())) == _lib.KVBM_ERR_NULL
    assert _lib.status_string(_lib.KVBM_ERR_PAGE).startswith("a block-table entry")


@pytest.mark.parametrize("dtype,esize", [(_lib.KVBM_BF16, 2), (_lib.KVBM_F32, 4), (_lib.KVBM_F64, 8)])
def test_paged_workspace_covers_gathered_units(dtype, esize):
    """Workspace = dense workspace (largest path) + the gathered keys of the
    smallest batch x kv-head box holding the unit range."""
    lib = _lib.load()
    B, Hq, Hkv, N, D = 3, 8, 4, 200, 64
    kv = _kv(Hkv=Hkv, D=D, max_pages=13)

    def sub_dense(units):
        # the dense sub-problem: batches [b0, b1] (or kv-heads [g0, g1] of one batch)
        b0, b1 = units[0] // Hkv, (units[1] - 1) // Hkv
        g0, ng = (units[0] % Hkv, (units[1] - 1) % Hkv - units[0] % Hkv + 1) if b0 == b1 else (0, Hkv)
        G = Hq // Hkv
        sub = _problem(shape=(b1 - b0 + 1, ng * G, ng, N, D), dtype=dtype,
                       units=(units[0] - b0 * Hkv - g0, units[1] - b0 * Hkv - g0))
        return lib.kvbm_workspace_bytes(ctypes.byref(sub)), (b1 - b0 + 1) * ng

    row = N * D * esize
    for units, heads in [((0, 12), 12), ((5, 7), 2), ((4, 8), 4), ((3, 6), 8), ((11, 12), 1)]:
        p = _problem(shape=(B, Hq, Hkv, N, D), dtype=dtype, units=units)
        paged = lib.kvbm_paged_workspace_bytes(ctypes.byref(p), ctypes.byref(kv))
        dense, boxed = sub_dense(units)
        assert boxed == heads
        assert paged % 256 == 0
        # a range that crosses a batch boundary gathers whole batches
        assert paged - dense == -(-heads * row // 256) * 256, (units, paged, dense)
    p = _problem(shape=(B, Hq, Hkv, N, D), dtype=dtype)
    assert lib.kvbm_paged_workspace_bytes(ctypes.byref(p), ctypes.byref(_kv(max_pages=1))) == 0


def test_paged_compute_without_device_fails_cleanly():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    p = _problem(shape=(2, 8, 2, 128, 64))
    code = lib.kvbm_block_mass_paged(ctypes.byref(p), ctypes.byref(_kv()), None, None, ctypes.c_void_p(256),
                                     ctypes.c_void_p(256), 1 << 30, None)
    assert code in (_lib.KVBM_ERR_CUDA, _lib.KVBM_ERR_DEVICE)


def test_python_paged_argument_checks():
    q = torch.randn(2, 8, 100, 64)
    cache = torch.randn(20, 16, 2, 64)
    table = torch.arange(14).reshape(2, 7)
    pp = make_paged_problem(q, cache, table, causal=True, block_size=16)
    assert pp.kv.page_size == 16 and pp.kv.num_pages == 20 and pp.kv.max_pages == 7
    assert pp.keep[1].dtype == torch.int32
    assert paged_workspace_bytes(pp) > 0
    with pytest.raises(ValueError, match="covers"):
        make_paged_problem(q, cache, table[:, :6])
    with pytest.raises(ValueError, match="dtype"):
        make_paged_problem(q, cache.double(), table)
    with pytest.raises(ValueError, match="head dim"):
        make_paged_problem(q, cache[..., :32], table)
    with pytest.raises(ValueError, match="block_table"):
        make_paged_problem(q, cache, table[:1])
    with pytest.raises(ValueError, match="integer"):
        make_paged_problem(q, cache, table.float())
    with pytest.raises(ValueError, match="GQA"):
        make_paged_problem(torch.randn(2, 6, 100, 64), torch.randn(20, 16, 4, 64), table)


def test_oracle_paged_definition():
    """The paged input equals the dense keys it names; unused pages never matter."""
    rng = np.random.default_rng(5)
    B, Hq, Hkv, N, D, P = 2, 4, 2, 70, 16, 8
    q = rng.standard_normal((B, Hq, N, D)).astype(np.float32)
    k = rng.standard_normal((B, Hkv, N, D)).astype(np.float32)
    npg = -(-N // P)
    perm = rng.permutation(B * npg + 5)
    cache = rng.standard_normal((B * npg + 5, P, Hkv, D)).astype(np.float32)
    table = perm[:B * npg].reshape(B, npg)
    for b in range(B):
        for c in range(N):
            cache[table[b, c // P], c % P] = k[b, :, c]
    dense = dense_keys_from_pages(cache, table, N)
    assert np.array_equal(dense, k)
    want = block_mass_stream(q, k, causal=True, block_size=P)
    got = block_mass_stream(q, dense, causal=True, block_size=P)
    assert np.array_equal(want, got)
