"""Device-side eviction design, host side (no GPU): C argument checks and the
Python wrapper's errors, which follow the reference's (evict.py:79-83, 132-139)."""

import ctypes

import pytest
import torch

from kvblockmass_b200 import _lib
from kvblockmass_b200.design import _args, design_from_mass


def _d(**kw):
    # a valid set first; the fields under test are then overwritten in the C struct
    a, _ = _args(torch.rand(16, dtype=torch.float64), 1000, 64, 10, 4, 32, 0, 1e-6, False)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_design_workspace_and_checks():
    lib = _lib.load()
    ws = lib.kvbm_design_workspace_bytes(ctypes.byref(_d()))
    assert ws > 0 and ws % 256 == 0
    assert lib.kvbm_design_workspace_bytes(ctypes.byref(_d(eps=0.0))) == 0
    assert lib.kvbm_design_workspace_bytes(ctypes.byref(_d(tail_budget=-1))) == 0
    assert lib.kvbm_design_workspace_bytes(ctypes.byref(_d(mass_dtype=_lib.KVBM_BF16))) == 0
    assert lib.kvbm_design_workspace_bytes(ctypes.byref(_d(num_blocks=15))) == 0   # 15 * 64 < 1000
    assert lib.kvbm_design_workspace_bytes(ctypes.byref(_d(rows=2, mass_row_stride=8))) == 0
    assert lib.kvbm_design_workspace_bytes(None) == 0
    # sizes near the int32 limit are rejected, not overflowed
    big = 2**31 - 1
    assert lib.kvbm_design_workspace_bytes(ctypes.byref(_d(seq_len=big, block_size=2, num_blocks=big))) == 0
    assert lib.kvbm_design_workspace_bytes(ctypes.byref(_d(seq_len=(1 << 28) + 1, num_blocks=(1 << 22) + 1))) == 0
    assert lib.kvbm_design_workspace_bytes(ctypes.byref(_d(seq_len=1 << 28, num_blocks=1 << 22))) > 0
    out = _lib.DesignOut()
    code = lib.kvbm_design(ctypes.byref(_d()), ctypes.byref(out), None, 0, None)
    assert code == _lib.KVBM_ERR_NULL          # counts is required


def test_python_errors_follow_the_reference():
    m = torch.rand(4, dtype=torch.float64)
    with pytest.raises(ValueError, match="eps must be > 0"):
        _args(m, 100, 32, 1, 4, 32, 0, 0.0, False)
    with pytest.raises(ValueError, match="tail_budget must be >= 0"):
        _args(m, 100, 32, -1, 4, 32, 0, 1e-6, False)
    with pytest.raises(ValueError, match="cannot cover seq_len=200"):
        _args(m, 200, 32, 1, 4, 32, 0, 1e-6, False)
    with pytest.raises(ValueError, match="1-D"):
        _args(torch.rand(2, 2, 2), 4, 1, 1, 0, 0, 0, 1e-6, False)
    with pytest.raises(ValueError, match="CUDA"):
        design_from_mass(m, 100, 32, 5)
