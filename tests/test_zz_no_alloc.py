"""kvbm_block_mass_static: block mass without any device allocation.

Callers such as a serving engine that has reserved all free device memory for
its KV-cache pool (so cudaMalloc fails, and a cudaMalloc/cudaFree in its step
loop would synchronise the device) cannot hand the library a workspace.  For
them the library keeps a fixed scratch array in device memory.  These tests
call that entry point through the C ABI and check it against the regular
workspace-taking entry point and against the CPU oracle.  The calls run back
to back on problems of different shapes and kernel paths, so each call finds
the previous one's data in the shared array: the lse2 rows, the partials, the
tf32 copies of fp32 inputs and the packed pair-mask bits.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from _helpers import max_rel
from oracle import block_mass_np as orc

from kvblockmass_b200 import _lib
from kvblockmass_b200.ops import kernel_path, make_problem

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 2e-5, torch.bfloat16: 1e-3}


def _inputs(B, Hq, Hkv, N, D, dtype, seed, dev):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, N, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    return q, k, q.to(dev), k.to(dev)


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


def _static(prep, dev):
    lib = _lib.load()
    out = torch.full((prep.nb,), float("nan"), dtype=prep.out_dtype, device=dev)
    rc = lib.kvbm_block_mass_static(ctypes.byref(prep.prob), out.data_ptr(),
                                    torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 0, _lib.status_string(rc)
    return out


def _oracle(q, k, mask, kw):
    return orc.block_mass_stream(q.float().numpy(), k.float().numpy(),
                                 attn_mask=None if mask is None else mask.numpy(), **kw)


# (shape, call keywords, mask kind, kernel path it must take)
CASES = [
    # tcgen05 path: bf16, D=128, causal, ragged N
    (dict(B=1, Hq=8, Hkv=2, N=3000, D=128, dtype=torch.bfloat16, seed=11),
     dict(causal=True, block_size=64), None, 1),
    # SIMT path: fp32 with D=160 (the 3xTF32 path takes D <= 128), key mask, non-causal
    (dict(B=2, Hq=4, Hkv=2, N=777, D=160, dtype=torch.float32, seed=12),
     dict(causal=False, block_size=48), "keys", 0),
    # 3xTF32 path: fp32 with D=64, its tf32 copies of q/k in the scratch array
    (dict(B=1, Hq=4, Hkv=1, N=1000, D=64, dtype=torch.float32, seed=13),
     dict(causal=True, block_size=64), None, 2),
    # tcgen05 with a per-batch pair mask: its packed bits in the scratch array,
    # after calls of other shapes left their data there
    (dict(B=2, Hq=4, Hkv=2, N=500, D=64, dtype=torch.bfloat16, seed=14),
     dict(causal=True, block_size=32), "batch_pairs", 1),
]


def test_static_matches_workspace_entry_point_and_oracle(cuda_device):
    dev = cuda_device
    lib = _lib.load()
    assert lib.kvbm_static_scratch_bytes() == 64 << 20
    runs = []
    for shape, kw, mkind, path in CASES:
        q, k, qd, kd = _inputs(dev=dev, **shape)
        N, B = shape["N"], shape["B"]
        g = torch.Generator().manual_seed(3)
        mask = None
        if mkind == "keys":
            mask = torch.rand(N, generator=g) > 0.2
        elif mkind == "batch_pairs":
            mask = torch.rand(B, N, N, generator=g) > 0.3
        prep = make_problem(qd, kd, attn_mask=None if mask is None else mask.to(dev), **kw)
        assert kernel_path(prep) == path, (shape, path)
        runs.append((prep, shape["dtype"], q, k, mask, kw))
    # two rounds of static calls in a row on one stream: every call finds the
    # previous call's data in the shared array
    firsts = [_static(prep, dev) for prep, *_ in runs]
    seconds = [_static(prep, dev) for prep, *_ in runs]
    torch.cuda.synchronize()
    assert lib.kvbm_check_device_errors(torch.cuda.current_stream(dev).cuda_stream) == 0
    for (prep, dtype, q, k, mask, kw), a, b in zip(runs, firsts, seconds):
        want = _regular(prep, dev)
        torch.cuda.synchronize()
        ga, gb = a.double().cpu().numpy(), b.double().cpu().numpy()
        assert np.isfinite(ga).all() and np.isfinite(gb).all()
        assert max_rel(ga, want.double().cpu().numpy()) < TOL[dtype]
        assert max_rel(gb, want.double().cpu().numpy()) < TOL[dtype]
        assert max_rel(ga, _oracle(q, k, mask, kw)) < TOL[dtype]


def test_static_unit_ranges_split_a_problem_too_large_for_the_array(cuda_device):
    """An fp32 problem whose workspace is larger than the array is refused whole,
    and runs as unit ranges: a range inside one batch entry needs scratch for
    its own units' rows only.  The ranges add up to the whole."""
    dev = cuda_device
    lib = _lib.load()
    q, k, qd, kd = _inputs(1, 32, 8, 8192, 64, torch.float32, 21, dev)
    prep = make_problem(qd, kd, causal=True, block_size=64)
    assert kernel_path(prep) == 2
    assert lib.kvbm_workspace_bytes(ctypes.byref(prep.prob)) > lib.kvbm_static_scratch_bytes()
    out = torch.empty(prep.nb, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert lib.kvbm_block_mass_static(ctypes.byref(prep.prob), out.data_ptr(), stream) == _lib.KVBM_ERR_SCRATCH
    total = torch.zeros(prep.nb, dtype=torch.float64, device=dev)
    parts = []
    for u in range(8):
        prep.prob.unit_begin, prep.prob.unit_end = u, u + 1
        m = _static(prep, dev)
        parts.append(m)
        total += m.double()
    prep.prob.unit_begin, prep.prob.unit_end = 0, 8
    whole = _regular(prep, dev)
    torch.cuda.synchronize()
    assert max_rel(total.cpu().numpy(), whole.double().cpu().numpy()) < 1e-6
    # unit 5 alone against the oracle (q-heads 20..23 with kv-head 5)
    want = orc.block_mass_stream(q[:, 20:24].numpy(), k[:, 5:6].numpy(), causal=True, block_size=64, threads=8)
    assert max_rel(parts[5].cpu().numpy(), want) < 2e-5


def test_static_rejects_oversized_problem(cuda_device):
    """A problem whose scratch exceeds the fixed array is refused before any launch."""
    lib = _lib.load()
    _, _, q, k = _inputs(1, 8, 1, 256, 128, torch.bfloat16, 5, cuda_device)
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
