"""Ragged / packed batches and per-sequence output, host side (no GPU): the
oracle's definition, C validation of kvbm_options, Python argument checks."""

import ctypes

import numpy as np
import pytest
import torch

from kvblockmass_b200 import _lib
from kvblockmass_b200.ops import make_problem, make_varlen_problem, workspace_bytes
from oracle.block_mass_np import block_mass_ragged, block_mass_stream
from test_abi import _problem


@pytest.mark.parametrize("causal", [True, False])
def test_oracle_ragged_equals_length_masks(causal):
    """Each sequence alone == the batch with key/query masks cut at its length."""
    rng = np.random.default_rng(1)
    B, Hq, Hkv, N, D = 4, 4, 2, 90, 16
    q = rng.standard_normal((B, Hq, N, D)).astype(np.float32)
    k = rng.standard_normal((B, Hkv, N, D)).astype(np.float32)
    lens = [90, 41, 1, 0]
    pos = np.arange(N)
    live = np.stack([pos < L for L in lens])
    for extra in (None, rng.random((B, N, N)) > 0.3, rng.random((B, 1, N)) > 0.2):
        pm = live[:, None, :] if extra is None else (extra & live[:, None, :])
        want = block_mass_stream(q, k, attn_mask=pm, query_mask=live, causal=causal, block_size=16)
        got = block_mass_ragged(q, k, lens, attn_mask=extra, causal=causal, block_size=16)
        assert np.allclose(got, want, rtol=1e-5, atol=1e-6)
    per = block_mass_ragged(q, k, lens, causal=causal, block_size=16, per_sequence=True)
    assert per.shape == (B, 6)
    for b, L in enumerate(lens):
        assert abs(per[b].sum() - (Hq * L if causal or L else 0)) < 1e-3 * max(1, Hq * L)
        assert np.all(per[b, -(-L // 16):] == 0)


def _opts(**kw):
    o = _lib.Options()
    for name, v in kw.items():
        setattr(o, name, v)
    return o


def test_validate_ex_codes():
    lib = _lib.load()
    p = _problem(shape=(2, 8, 2, 128, 64))
    ok = lambda o: lib.kvbm_validate_ex(ctypes.byref(p), None if o is None else ctypes.byref(o))  # noqa: E731
    assert ok(None) == _lib.KVBM_OK
    assert ok(_opts(seq_lens=4096)) == _lib.KVBM_OK
    assert ok(_opts(cu_seqlens=4096, total_tokens=300)) == _lib.KVBM_OK
    assert ok(_opts(seq_lens=4096, cu_seqlens=8192, total_tokens=300)) == _lib.KVBM_ERR_SHAPE
    assert ok(_opts(cu_seqlens=4096)) == _lib.KVBM_ERR_SHAPE          # total_tokens missing
    assert ok(_opts(per_sequence=1)) == _lib.KVBM_OK
    o = _opts(lse=4096)
    o.lse_stride[1] = -1
    assert ok(o) == _lib.KVBM_ERR_SHAPE
    assert lib.kvbm_validate_ex(None, None) == _lib.KVBM_ERR_NULL


def test_workspace_ex_sizes_packed_split_by_tokens():
    """3xTF32 copies every q/k row: a packed fp32 batch sizes them by total_tokens."""
    lib = _lib.load()
    p = _problem(shape=(4, 8, 2, 1024, 64), dtype=_lib.KVBM_F32)
    dense = lib.kvbm_workspace_bytes_ex(ctypes.byref(p), None)
    assert dense == lib.kvbm_workspace_bytes(ctypes.byref(p))
    small = lib.kvbm_workspace_bytes_ex(ctypes.byref(p), ctypes.byref(_opts(cu_seqlens=4096, total_tokens=1500)))
    big = lib.kvbm_workspace_bytes_ex(ctypes.byref(p), ctypes.byref(_opts(cu_seqlens=4096, total_tokens=4096)))
    assert 0 < small < big
    assert lib.kvbm_workspace_bytes_ex(ctypes.byref(p), ctypes.byref(_opts(seq_lens=1, cu_seqlens=2))) == 0


def test_python_ragged_argument_checks():
    q, k = torch.randn(3, 8, 100, 64), torch.randn(3, 2, 100, 64)
    prep = make_problem(q, k, seq_lens=torch.tensor([100, 7, 0]), per_sequence=True)
    assert prep.out_shape == (3, 2) and prep.opts.per_sequence == 1
    assert workspace_bytes(prep) > 0
    with pytest.raises(ValueError, match="seq_lens"):
        make_problem(q, k, seq_lens=torch.tensor([1, 2]))
    with pytest.raises(ValueError, match="integers"):
        make_problem(q, k, seq_lens=torch.tensor([1.0, 2.0, 3.0]))
    qp, kp = torch.randn(250, 8, 64), torch.randn(250, 2, 64)
    cu = torch.tensor([0, 100, 107, 250], dtype=torch.int32)
    vp = make_varlen_problem(qp, kp, cu, causal=True)
    assert vp.prob.N == 143 and vp.prob.B == 3 and vp.packed and vp.total == 250
    assert vp.prob.q_stride[0] == 0 and vp.prob.q_stride[2] == 8 * 64
    with pytest.raises(ValueError, match="3-D"):
        make_varlen_problem(q, k, cu)
    with pytest.raises(ValueError, match="B \\+ 1"):
        make_varlen_problem(qp, kp, cu[:1])
    with pytest.raises(ValueError, match="GQA"):
        make_varlen_problem(torch.randn(250, 6, 64), torch.randn(250, 4, 64), cu)
