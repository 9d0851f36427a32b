"""C-ABI library checks that need no GPU: load, exports, host-side validation."""

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from kvblockmass_b200 import _lib
from kvblockmass_b200.ops import make_problem

ROOT = Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = []
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"\b(kvbm_\w+)\s*\(", text)
    return sorted(set(names))


def test_library_loads():
    lib = _lib.load()
    assert lib.kvbm_abi_version() == _lib.ABI_VERSION == 4


def test_every_declared_symbol_is_exported():
    decl = declared_functions()
    assert "kvbm_block_mass" in decl
    lib = _lib.load()
    for name in decl:
        assert hasattr(lib, name), f"{name} declared in include/*.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (kvbm_\w+)", out))
    assert set(decl) <= exported
    assert set(_lib.EXPORTED) <= exported


def _problem(**kw):
    p = _lib.Problem()
    p.q = 16
    p.k = 16
    B, Hq, Hkv, N, D = kw.get("shape", (1, 8, 2, 128, 64))
    p.B, p.Hq, p.Hkv, p.N, p.D = B, Hq, Hkv, N, D
    for i, s in enumerate((Hq * N * D, N * D, D, 1)):
        p.q_stride[i] = s
    for i, s in enumerate((Hkv * N * D, N * D, D, 1)):
        p.k_stride[i] = s
    p.dtype = kw.get("dtype", _lib.KVBM_F32)
    p.scale = 0.125
    p.block_size = kw.get("block_size", 64)
    p.causal = 1
    p.causal_skip = 1
    p.unit_begin, p.unit_end = kw.get("units", (0, B * Hkv))
    return p


@pytest.mark.parametrize("kw,code", [
    ({}, _lib.KVBM_OK),
    ({"shape": (1, 6, 4, 8, 4)}, _lib.KVBM_ERR_GQA),
    ({"shape": (1, 8, 2, 0, 64)}, _lib.KVBM_ERR_SHAPE),
    ({"dtype": 7}, _lib.KVBM_ERR_DTYPE),
    ({"shape": (1, 8, 2, 128, 300)}, _lib.KVBM_ERR_HEAD_DIM),
    ({"shape": (1, 8, 2, 128, 200), "dtype": _lib.KVBM_F64}, _lib.KVBM_ERR_HEAD_DIM),
    ({"block_size": 0}, _lib.KVBM_ERR_BLOCK_SIZE),
    ({"units": (0, 3)}, _lib.KVBM_ERR_UNITS),
    ({"units": (1, 1)}, _lib.KVBM_ERR_UNITS),
    ({"shape": (1, 8, 2, 1 << 28, 64)}, _lib.KVBM_OK),
    ({"shape": (1, 8, 2, (1 << 28) + 1, 64)}, _lib.KVBM_ERR_SHAPE),
    ({"shape": (1, 8, 2, 2**31 - 1, 64)}, _lib.KVBM_ERR_SHAPE),
    ({"shape": (4096, 16, 2, 128, 64)}, _lib.KVBM_ERR_SHAPE),
])
def test_validate_codes(kw, code):
    lib = _lib.load()
    assert lib.kvbm_validate(ctypes.byref(_problem(**kw))) == code
    assert _lib.status_string(code)


def test_num_blocks_and_workspace():
    lib = _lib.load()
    assert lib.kvbm_num_blocks(100, 64) == 2       # KVBM-05: ragged last block
    assert lib.kvbm_num_blocks(2048, 64) == 32
    assert lib.kvbm_num_blocks(16, 64) == 1
    p = _problem()
    ws = lib.kvbm_workspace_bytes(ctypes.byref(p))
    # lse2 [U*G*N] + per-key partials [U*nchunk*N], fp32
    assert ws >= (2 * 4 * 128 + 2 * 1 * 128) * 4
    assert ws % 256 == 0
    assert lib.kvbm_workspace_bytes(ctypes.byref(_problem(shape=(1, 6, 4, 8, 4)))) == 0
    assert lib.kvbm_launches_per_call(ctypes.byref(p)) == 3
    # bf16 with a key mask: + the pre-pass over the dropped keys' rows on tensor-core path 1
    # (without a GPU and its driver the path here is the SIMT one)
    pk = _problem(dtype=_lib.KVBM_BF16)
    km = (ctypes.c_uint8 * 128)()
    pk.key_mask = ctypes.cast(km, ctypes.c_void_p).value
    tc = lib.kvbm_kernel_path(ctypes.byref(pk)) == 1
    assert lib.kvbm_launches_per_call(ctypes.byref(pk)) == 3 + (1 if tc else 0)


def test_block_mass_without_device_fails_cleanly():
    """No GPU here: the compute entry point reports an error, it never falls back."""
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    p = _problem()
    code = lib.kvbm_block_mass(ctypes.byref(p), ctypes.c_void_p(256), ctypes.c_void_p(256), 1 << 20, None)
    assert code in (_lib.KVBM_ERR_CUDA, _lib.KVBM_ERR_DEVICE)


def test_python_wrapper_errors_match_reference():
    """ValueError with the reference's message for GQA (reference.py:29-30, KVBM-06)."""
    q = torch.randn(1, 6, 8, 4)
    k = torch.randn(1, 4, 8, 4)
    with pytest.raises(ValueError, match=r"GQA requires H_q % H_kv == 0, got H_q=6, H_kv=4"):
        make_problem(q, k, block_size=4)
    with pytest.raises(ValueError):
        make_problem(torch.randn(1, 2, 8, 4), torch.randn(1, 1, 9, 4))
    with pytest.raises(ValueError):
        make_problem(torch.randn(1, 2, 8, 4), torch.randn(1, 1, 8, 4), attn_mask=torch.ones(7, dtype=torch.bool))


def test_cpu_tensors_are_rejected():
    from kvblockmass_b200 import block_mass, block_mass_b200

    q = torch.randn(1, 2, 8, 4)
    k = torch.randn(1, 1, 8, 4)
    with pytest.raises(ValueError, match="CUDA"):
        block_mass_b200(q, k)
    with pytest.raises(ValueError):
        block_mass(q, k)


def test_signatures_are_drop_in():
    """Every argument of the reference's entry points is accepted."""
    import inspect

    from kvblockmass_b200 import block_mass_b200, block_mass_triton

    ref_reference = ["q", "k", "attn_mask", "causal", "block_size", "scale", "query_chunk", "device",
                     "causal_skip"]                       # reference.py:35-45
    ref_triton = ["q", "k", "attn_mask", "causal", "block_size", "scale", "BLOCK_M", "BLOCK_N",
                  "causal_skip"]                          # triton_kernel.py:148-158
    params = inspect.signature(block_mass_b200).parameters
    for name in ref_reference + ref_triton:
        assert name in params, name
    assert list(inspect.signature(block_mass_triton).parameters) == ref_triton


def test_selftest_argument_checks():
    lib = _lib.load()
    w = ctypes.c_int(0)
    assert lib.kvbm_selftest_wait_timeout(None, 10, ctypes.byref(w)) == _lib.KVBM_ERR_SHAPE   # < 1 us
    assert lib.kvbm_selftest_wait_timeout(None, 3_000_000_000, ctypes.byref(w)) == _lib.KVBM_ERR_SHAPE
    assert lib.kvbm_selftest_wait_timeout(None, 1_000_000, None) == _lib.KVBM_ERR_NULL
    if not torch.cuda.is_available():
        code = lib.kvbm_selftest_wait_timeout(None, 1_000_000, ctypes.byref(w))
        assert code in (_lib.KVBM_ERR_CUDA, _lib.KVBM_ERR_DEVICE)


def test_validate_survives_random_problems():
    """kvbm_validate / kvbm_workspace_bytes / kvbm_num_blocks on 3000 random
    problems (negative, zero, huge and mismatched sizes and strides): every call
    returns a known status, and an accepted problem has a workspace size."""
    lib = _lib.load()
    rng = np.random.default_rng(5)
    known = {_lib.KVBM_OK, _lib.KVBM_ERR_GQA, _lib.KVBM_ERR_SHAPE, _lib.KVBM_ERR_DTYPE,
             _lib.KVBM_ERR_HEAD_DIM, _lib.KVBM_ERR_BLOCK_SIZE, _lib.KVBM_ERR_UNITS, _lib.KVBM_ERR_NULL}
    picks = [-(2**31), -5, -1, 0, 1, 2, 3, 7, 8, 64, 100, 128, 257, 4096, 65536, 1 << 28, 2**31 - 1]
    for _ in range(3000):
        B, Hq, Hkv, N, D, bs = (int(rng.choice(picks)) for _ in range(6))
        p = _problem(shape=(B, Hq, Hkv, N, D), dtype=int(rng.integers(-1, 5)), block_size=bs,
                     units=(int(rng.choice(picks)), int(rng.choice(picks))))
        if rng.random() < 0.2:
            p.q_stride[int(rng.integers(0, 4))] = -int(rng.integers(1, 1 << 40))
        if rng.random() < 0.1:
            p.scale = float("nan")
        st = lib.kvbm_validate(ctypes.byref(p))
        assert st in known
        ws = lib.kvbm_workspace_bytes(ctypes.byref(p))
        if st == _lib.KVBM_OK:
            assert ws > 0
        else:
            assert ws == 0
        lib.kvbm_num_blocks(N, bs)


def test_validate_ex_survives_random_options():
    """kvbm_validate_ex / kvbm_workspace_bytes_ex with random extension options
    (LSE strides, paged caches, padded or packed lengths).  The option pointers
    are device addresses the host must never read, so they are fake here: a
    host-side read would crash this test."""
    lib = _lib.load()
    rng = np.random.default_rng(6)
    known = {_lib.KVBM_OK, _lib.KVBM_ERR_GQA, _lib.KVBM_ERR_SHAPE, _lib.KVBM_ERR_DTYPE,
             _lib.KVBM_ERR_HEAD_DIM, _lib.KVBM_ERR_BLOCK_SIZE, _lib.KVBM_ERR_UNITS, _lib.KVBM_ERR_NULL}
    fake = 0x10000
    picks = [-(2**31), -3, -1, 0, 1, 2, 16, 64, 129, 4096, 1 << 28, 2**31 - 1]
    for _ in range(2000):
        N = int(rng.choice([1, 64, 1000, 4096, 1 << 20]))
        p = _problem(shape=(int(rng.choice([1, 2, 3])), 8, 2, N, 64), dtype=int(rng.integers(0, 4)))
        o = _lib.Options()
        if rng.random() < 0.4:
            o.lse = fake
            for i in range(3):
                o.lse_stride[i] = int(rng.choice(picks))
        kv = None
        if rng.random() < 0.4:
            kv = _lib.PagedKV()
            kv.k_cache = fake if rng.random() < 0.9 else None
            for i in range(4):
                kv.cache_stride[i] = int(rng.choice(picks))
            kv.num_pages = int(rng.choice(picks))
            kv.page_size = int(rng.choice(picks))
            kv.block_table = fake if rng.random() < 0.9 else None
            kv.block_table_stride = int(rng.choice(picks))
            kv.max_pages = int(rng.choice(picks))
            o.paged = ctypes.pointer(kv)
        r = rng.random()
        if r < 0.3:
            o.seq_lens = fake
        elif r < 0.6:
            o.cu_seqlens = fake
            o.total_tokens = int(rng.choice(picks + [2**40]))
        elif r < 0.7:
            o.seq_lens = fake
            o.cu_seqlens = fake
        o.per_sequence = int(rng.integers(0, 2))
        st = lib.kvbm_validate_ex(ctypes.byref(p), ctypes.byref(o))
        assert st in known
        ws = lib.kvbm_workspace_bytes_ex(ctypes.byref(p), ctypes.byref(o))
        assert (ws > 0) == (st == _lib.KVBM_OK)


def _opts(**kw):
    o = _lib.Options()
    for name, v in kw.items():
        setattr(o, name, v)
    return o


@pytest.mark.parametrize("kw,code", [
    (dict(stages=_lib.KVBM_STAGE_PASS1), _lib.KVBM_OK),
    (dict(stages=16), _lib.KVBM_ERR_SHAPE),
    (dict(stages=-1), _lib.KVBM_ERR_SHAPE),
    (dict(stages=_lib.KVBM_STAGE_PASS2, run_unit_begin=1, run_unit_end=2), _lib.KVBM_OK),
    (dict(run_unit_begin=1, run_unit_end=3), _lib.KVBM_ERR_UNITS),       # the problem has 2 units
    (dict(run_unit_begin=-1, run_unit_end=1), _lib.KVBM_ERR_UNITS),
    (dict(run_unit_begin=0, run_unit_end=1, run_head_begin=1, run_head_end=3), _lib.KVBM_OK),
    (dict(run_head_begin=1, run_head_end=3), _lib.KVBM_ERR_SHAPE),       # narrower than G=4 over 2 units
    (dict(run_head_begin=0, run_head_end=4), _lib.KVBM_OK),              # every head: any run range
    (dict(run_unit_begin=0, run_unit_end=1, run_head_begin=2, run_head_end=5), _lib.KVBM_ERR_SHAPE),
])
def test_staged_option_checks(kw, code):
    """Staged calls (kvbm_options.stages / run ranges) are checked on the host."""
    lib = _lib.load()
    p = _problem()  # B=1, H_q=8, H_kv=2: 2 units of G=4 heads
    assert lib.kvbm_validate_ex(ctypes.byref(p), ctypes.byref(_opts(**kw))) == code


@pytest.mark.parametrize("pkw,okw,code", [
    (dict(dtype=_lib.KVBM_BF16), dict(method=_lib.KVBM_METHOD_ONE_PASS), _lib.KVBM_OK),
    (dict(dtype=_lib.KVBM_F32), dict(method=_lib.KVBM_METHOD_ONE_PASS), _lib.KVBM_OK),
    (dict(dtype=_lib.KVBM_BF16, block_size=256), dict(method=_lib.KVBM_METHOD_ONE_PASS), _lib.KVBM_OK),
    (dict(dtype=_lib.KVBM_BF16, block_size=192), dict(method=_lib.KVBM_METHOD_ONE_PASS), _lib.KVBM_OK),
    # one pass needs block_size % 64 == 0 and tensor-core dtypes
    (dict(dtype=_lib.KVBM_BF16, block_size=48), dict(method=_lib.KVBM_METHOD_ONE_PASS), _lib.KVBM_ERR_SHAPE),
    (dict(dtype=_lib.KVBM_F64), dict(method=_lib.KVBM_METHOD_ONE_PASS), _lib.KVBM_ERR_SHAPE),
    (dict(dtype=_lib.KVBM_BF16), dict(method=_lib.KVBM_METHOD_ONE_PASS, lse=0x10000), _lib.KVBM_OK),
    (dict(dtype=_lib.KVBM_BF16, block_size=48), dict(method=_lib.KVBM_METHOD_AUTO), _lib.KVBM_OK),
    (dict(dtype=_lib.KVBM_BF16), dict(method=_lib.KVBM_METHOD_TWO_PASS), _lib.KVBM_OK),
    (dict(dtype=_lib.KVBM_BF16), dict(method=3), _lib.KVBM_ERR_SHAPE),
    (dict(dtype=_lib.KVBM_BF16), dict(method=-1), _lib.KVBM_ERR_SHAPE),
])
def test_method_option_checks(pkw, okw, code):
    """kvbm_options.method is checked on the host: the one-pass method needs a
    tensor-core dtype and a block size that is a multiple of 64 (with an LSE
    input its pass 1 takes the caller's row statistics)."""
    lib = _lib.load()
    o = _lib.Options()
    for name, v in okw.items():
        setattr(o, name, v)
    p = _problem(**pkw)
    assert lib.kvbm_validate_ex(ctypes.byref(p), ctypes.byref(o)) == code


def test_auto_method_falls_back_to_two_passes_for_long_sequences():
    """The one-pass partials grow as (N/128) * (N/block_size) per head: at
    N = 2^20 with 64-key blocks they would be 17 GiB, so the automatic choice
    takes two passes (the workspace equals the two-pass one), while a forced
    one-pass call still sizes its own."""
    lib = _lib.load()
    p = _problem(shape=(1, 32, 8, 1 << 20, 128), dtype=_lib.KVBM_BF16, block_size=64)
    auto = lib.kvbm_workspace_bytes_ex(ctypes.byref(p), ctypes.byref(_opts()))
    two = lib.kvbm_workspace_bytes_ex(ctypes.byref(p), ctypes.byref(_opts(method=_lib.KVBM_METHOD_TWO_PASS)))
    one = lib.kvbm_workspace_bytes_ex(ctypes.byref(p), ctypes.byref(_opts(method=_lib.KVBM_METHOD_ONE_PASS)))
    assert auto == two and one > 4 * two
    assert one >= 32 * 8192 * 16384 * 4  # the per-tile partials alone


def test_one_pass_workspace_holds_slots_and_tile_partials():
    """With the device unknown the workspace covers the one-pass layout: its
    per-tile partials [U*G, ceil(N/128), nb] fp32 and 2 x 160 slots of
    [ceil(N/128) / F * 2, 128] fp32 segment sums, where F = block_size / 128
    (or 1)."""
    lib = _lib.load()
    for bs in (64, 256):
        N, Hq, Hkv = 32768, 32, 8
        p = _problem(shape=(1, Hq, Hkv, N, 128), dtype=_lib.KVBM_BF16, block_size=bs)
        one = lib.kvbm_workspace_bytes_ex(ctypes.byref(p), ctypes.byref(_opts(method=_lib.KVBM_METHOD_ONE_PASS)))
        two = lib.kvbm_workspace_bytes_ex(ctypes.byref(p), ctypes.byref(_opts(method=_lib.KVBM_METHOD_TWO_PASS)))
        auto = lib.kvbm_workspace_bytes_ex(ctypes.byref(p), ctypes.byref(_opts()))
        nt, nb = N // 128, N // bs
        F = max(1, bs // 128)
        part1 = Hq * nt * nb * 4
        slots = 2 * 160 * (nt // F * 2) * 128 * 4
        assert one >= part1 + slots + Hq * N * 4
        assert auto == one and two <= one
        if bs == 64:  # larger than every SIMT layout (which an unknown device could also take)
            assert one < part1 + slots + Hq * N * 4 + (8 << 20)
            assert two < one


@pytest.mark.parametrize("rows,code", [
    ((0, 128), _lib.KVBM_OK),
    ((128, 256), _lib.KVBM_OK),
    ((256, 300), _lib.KVBM_OK),       # the end may be N
    ((128, 300), _lib.KVBM_OK),
    ((64, 128), _lib.KVBM_ERR_SHAPE),  # begin not a multiple of 128
    ((0, 200), _lib.KVBM_ERR_SHAPE),   # end neither a multiple of 128 nor N
    ((256, 384), _lib.KVBM_ERR_SHAPE),  # past N
    ((-128, 128), _lib.KVBM_ERR_SHAPE),
    ((128, 128), _lib.KVBM_OK),       # empty: every row
])
def test_staged_row_range_checks(rows, code):
    """A pass-1 query-row range (kvbm_options.run_row_begin/end) is checked on the host."""
    lib = _lib.load()
    p = _problem(shape=(1, 8, 2, 300, 64), dtype=_lib.KVBM_BF16)
    o = _opts(stages=_lib.KVBM_STAGE_PASS1, run_row_begin=rows[0], run_row_end=rows[1])
    assert lib.kvbm_validate_ex(ctypes.byref(p), ctypes.byref(o)) == code


def test_staged_row_range_excludes_the_lse_input():
    lib = _lib.load()
    p = _problem(shape=(1, 8, 2, 300, 64), dtype=_lib.KVBM_BF16)
    lse = torch.zeros(1, 8, 300)
    o = _opts(stages=_lib.KVBM_STAGE_PASS1, run_row_begin=0, run_row_end=128, lse=lse.data_ptr())
    for i, s in enumerate(lse.stride()):
        o.lse_stride[i] = s
    assert lib.kvbm_validate_ex(ctypes.byref(p), ctypes.byref(o)) == _lib.KVBM_ERR_SHAPE
    o.run_row_begin = o.run_row_end = 0
    assert lib.kvbm_validate_ex(ctypes.byref(p), ctypes.byref(o)) == _lib.KVBM_OK


def test_copy_2d_argument_checks():
    """kvbm_copy_2d_async checks its arguments on the host; zero sizes queue nothing."""
    lib = _lib.load()
    buf = ctypes.create_string_buffer(64)
    ptr = ctypes.addressof(buf)
    assert lib.kvbm_copy_2d_async(None, 8, ptr, 8, 8, 2, None) == _lib.KVBM_ERR_NULL
    assert lib.kvbm_copy_2d_async(ptr, 8, None, 8, 8, 2, None) == _lib.KVBM_ERR_NULL
    assert lib.kvbm_copy_2d_async(ptr, 8, ptr, 8, -1, 2, None) == _lib.KVBM_ERR_SHAPE
    assert lib.kvbm_copy_2d_async(ptr, 8, ptr, 8, 8, -2, None) == _lib.KVBM_ERR_SHAPE
    assert lib.kvbm_copy_2d_async(ptr, 4, ptr, 8, 8, 2, None) == _lib.KVBM_ERR_SHAPE  # pitch below width
    assert lib.kvbm_copy_2d_async(ptr, 8, ptr, 8, 0, 2, None) == _lib.KVBM_OK
    assert lib.kvbm_copy_2d_async(ptr, 8, ptr, 8, 8, 0, None) == _lib.KVBM_OK


def test_staged_calls_take_no_ragged_or_paged_inputs():
    lib = _lib.load()
    p = _problem()
    lens = torch.full((1,), 100, dtype=torch.int32)
    o = _opts(stages=_lib.KVBM_STAGE_PASS1, seq_lens=lens.data_ptr())
    assert lib.kvbm_validate_ex(ctypes.byref(p), ctypes.byref(o)) == _lib.KVBM_ERR_SHAPE
    o = _opts(seq_lens=lens.data_ptr())
    assert lib.kvbm_validate_ex(ctypes.byref(p), ctypes.byref(o)) == _lib.KVBM_OK


def test_unit_range_workspace_covers_only_its_rows():
    """The workspace of a unit range inside one batch entry holds only those
    units' rows: an fp32 problem's tf32 copies (path 2) shrink with the range,
    so a one-unit slice of a problem too large for the no-allocation entry
    point's 64 MiB fits it (with the two-pass method, which that entry point
    falls back to when the one-pass slots do not fit)."""
    lib = _lib.load()
    two_pass = _opts(method=_lib.KVBM_METHOD_TWO_PASS)

    def ws(p):
        return lib.kvbm_workspace_bytes_ex(ctypes.byref(p), ctypes.byref(two_pass))

    shape = (1, 32, 8, 8192, 64)  # fp32 D=64 runs the 3xTF32 path
    full = ws(_problem(shape=shape))
    one = ws(_problem(shape=shape, units=(3, 4)))
    limit = lib.kvbm_static_scratch_bytes()
    assert full > limit >= one
    # lse2 + partials + tf32 hi/lo of the unit's 4 q-heads and its kv-head (a bound, all paths)
    N, D, G = 8192, 64, 4
    assert one <= (G * N + 64 * N) * 4 + 2 * 4 * D * N * (G + 1) + 4096
    # a range that crosses a batch entry keeps whole batch entries
    two_b = _problem(shape=(2, 32, 8, 8192, 64), units=(7, 9))
    assert ws(two_b) > one
