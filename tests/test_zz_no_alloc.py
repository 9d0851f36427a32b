"""kvbm_block_mass_static: block mass without any device allocation.

Callers such as a serving engine that has reserved all free device memory for
its KV-cache pool (so cudaMalloc fails, and a cudaMalloc/cudaFree in its step
loop would synchronise the device) cannot hand the library a workspace.  For
them the library keeps a fixed scratch array in device memory.  These tests
call that entry point through the C ABI and check it against the regular
workspace-taking entry point.  Two calls run back to back on different
problems, so the second call finds the first one's data in the shared array.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from kvblockmass_b200 import _lib
from kvblockmass_b200.ops import make_problem

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 2e-5, torch.bfloat16: 1e-3}


def _inputs(B, Hq, Hkv, N, D, dtype, seed, dev):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, N, D, generator=g).to(dtype).to(dev)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype).to(dev)
    return q, k


def _regular(prep, dev):
    """The existing entry point, with a caller-allocated workspace."""
    lib = _lib.load()
    ws = torch.empty(max(lib.kvbm_workspace_bytes(ctypes.byref(prep.prob)), 256), dtype=torch.uint8,
                     device=dev)
    out = torch.empty(prep.nb, dtype=prep.out_dtype, device=dev)
    rc = lib.kvbm_block_mass(ctypes.byref(prep.prob), out.data_ptr(), ws.data_ptr(), ws.numel(),
                             torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 0, _lib.status_string(rc)
    return out


def test_static_matches_workspace_entry_point(cuda_device):
    dev = cuda_device
    lib = _lib.load()
    assert lib.kvbm_static_scratch_bytes() == 64 << 20
    cases = [
        # tensor-core path: bf16, D=128, causal, ragged N
        (dict(B=1, Hq=8, Hkv=2, N=3000, D=128, dtype=torch.bfloat16, seed=11), dict(causal=True, block_size=64)),
        # SIMT path: fp32, D=64, key mask, non-causal
        (dict(B=2, Hq=4, Hkv=2, N=777, D=64, dtype=torch.float32, seed=12), dict(causal=False, block_size=48)),
    ]
    preps, outs = [], []
    stream = torch.cuda.current_stream(dev).cuda_stream
    for shape, kw in cases:
        q, k = _inputs(dev=dev, **shape)
        if shape["dtype"] == torch.float32:
            kw = dict(kw, attn_mask=(torch.rand(shape["N"], generator=torch.Generator().manual_seed(3)) > 0.2).to(dev))
        prep = make_problem(q, k, **kw)
        out = torch.full((prep.nb,), float("nan"), dtype=prep.out_dtype, device=dev)
        # two static calls in a row: the second finds the first's data in the array
        rc = lib.kvbm_block_mass_static(ctypes.byref(prep.prob), out.data_ptr(), stream)
        assert rc == 0, _lib.status_string(rc)
        preps.append((prep, shape["dtype"]))
        outs.append(out)
    torch.cuda.synchronize()
    assert lib.kvbm_check_device_errors(stream) == 0
    for (prep, dtype), got in zip(preps, outs):
        want = _regular(prep, dev)
        torch.cuda.synchronize()
        g, w = got.double().cpu().numpy(), want.double().cpu().numpy()
        assert np.isfinite(g).all()
        rel = float(np.max(np.abs(g - w) / np.maximum(np.abs(w), 1e-6)))
        assert rel < TOL[dtype], rel


def test_static_rejects_oversized_problem(cuda_device):
    """A problem whose scratch exceeds the fixed array is refused before any launch."""
    lib = _lib.load()
    q, k = _inputs(1, 8, 1, 256, 128, torch.bfloat16, 5, cuda_device)
    prep = make_problem(q, k, causal=True, block_size=256)
    # Describe the Llama-3-70B N=131072 shape over the same (valid, aligned)
    # pointers: the size check fails on the host, so nothing is read.
    p = prep.prob
    p.B, p.Hq, p.Hkv, p.N, p.D = 1, 64, 8, 131072, 128
    p.unit_begin, p.unit_end = 0, 8
    assert lib.kvbm_workspace_bytes(ctypes.byref(p)) > lib.kvbm_static_scratch_bytes()
    out = torch.empty(512, dtype=torch.float32, device=cuda_device)
    rc = lib.kvbm_block_mass_static(ctypes.byref(p), out.data_ptr(),
                                    torch.cuda.current_stream(cuda_device).cuda_stream)
    assert rc == _lib.KVBM_ERR_SCRATCH
    assert "scratch" in _lib.status_string(rc)
