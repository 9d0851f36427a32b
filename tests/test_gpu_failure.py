"""Failure detection of the tensor-core pipelines, tested without a GPU fault.

Every mbarrier wait in the tcgen05 kernels is bounded: when it runs out it
sets a device error word and the kernel returns.  ``kvbm_selftest_wait_timeout``
drives that code path on purpose with a barrier nothing arrives at and a 1 ms
limit; the host then reads KVBM_ERR_TIMEOUT, the word is cleared, and the
context keeps computing correct results.
"""

import ctypes

import pytest
import torch

import kvblockmass_b200 as kb
from kvblockmass_b200 import _lib

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_survives(cuda_device):
    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    kb.check_device_errors()                       # start clean
    waited = ctypes.c_int(-1)
    assert lib.kvbm_selftest_wait_timeout(stream, 1_000_000, ctypes.byref(waited)) == _lib.KVBM_OK
    assert waited.value == 0                       # nothing arrived: the wait gave up
    assert lib.kvbm_check_device_errors(stream) == _lib.KVBM_ERR_TIMEOUT
    assert lib.kvbm_check_device_errors(stream) == _lib.KVBM_OK   # cleared by the read
    # the context is healthy: a tensor-core call after the timeout is correct
    g = torch.Generator().manual_seed(80)
    q = torch.randn(1, 8, 700, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    k = torch.randn(1, 2, 700, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    m = kb.block_mass_b200(q, k, causal=True, block_size=64)
    assert abs(float(m.double().sum()) - 8 * 700) < 1e-5 * 8 * 700
    kb.check_device_errors()


def test_timeout_is_reported_through_python(cuda_device):
    lib = _lib.load()
    waited = ctypes.c_int(-1)
    lib.kvbm_selftest_wait_timeout(torch.cuda.current_stream(cuda_device).cuda_stream, 20_000,
                                   ctypes.byref(waited))
    with pytest.raises(RuntimeError, match=f"kvbm error {_lib.KVBM_ERR_TIMEOUT}"):
        kb.check_device_errors()
