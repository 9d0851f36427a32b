"""ctypes binding of ``libkvbm.so`` (C ABI declared in ``include/kvbm.h``).

The library is built in-tree by ``kv-block-mass_b200/build.py``.  There is no
fallback: if the library is missing or fails to load, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libkvbm.so"

KVBM_F32, KVBM_BF16, KVBM_F16, KVBM_F64 = 0, 1, 2, 3

KVBM_OK = 0
KVBM_ERR_GQA = 1
KVBM_ERR_SHAPE = 2
KVBM_ERR_DTYPE = 3
KVBM_ERR_HEAD_DIM = 4
KVBM_ERR_BLOCK_SIZE = 5
KVBM_ERR_UNITS = 6
KVBM_ERR_NULL = 7
KVBM_ERR_WORKSPACE = 8
KVBM_ERR_CUDA = 9
KVBM_ERR_DEVICE = 10
KVBM_ERR_TIMEOUT = 11
KVBM_ERR_SCRATCH = 12
KVBM_ERR_PAGE = 13

# Stages of a staged kvbm_block_mass_ex call (kvbm_options.stages).
KVBM_STAGE_MASKS = 1
KVBM_STAGE_PASS1 = 2
KVBM_STAGE_PASS2 = 4
KVBM_STAGE_REDUCE = 8
KVBM_METHOD_AUTO = 0
KVBM_METHOD_TWO_PASS = 1
KVBM_METHOD_ONE_PASS = 2

ABI_VERSION = 4

# Symbols include/kvbm.h declares; tests check the library exports each one.
EXPORTED = [
    "kvbm_abi_version",
    "kvbm_status_string",
    "kvbm_validate",
    "kvbm_num_blocks",
    "kvbm_workspace_bytes",
    "kvbm_kernel_path",
    "kvbm_launches_per_call",
    "kvbm_block_mass",
    "kvbm_block_mass_events",
    "kvbm_block_mass_lse",
    "kvbm_measure_ex2_rate",
    "kvbm_exp2_fma_fraction",
    "kvbm_check_device_errors",
    "kvbm_selftest_wait_timeout",
    "kvbm_block_mass_static",
    "kvbm_static_scratch_bytes",
    "kvbm_validate_paged",
    "kvbm_paged_workspace_bytes",
    "kvbm_block_mass_paged",
    "kvbm_validate_ex",
    "kvbm_workspace_bytes_ex",
    "kvbm_block_mass_ex",
    "kvbm_design_workspace_bytes",
    "kvbm_design",
    "kvbm_copy_2d_async",
    "kvbm_method",
]


class Problem(ctypes.Structure):
    """Mirror of ``struct kvbm_problem``."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("q_stride", ctypes.c_int64 * 4),
        ("k", ctypes.c_void_p),
        ("k_stride", ctypes.c_int64 * 4),
        ("dtype", ctypes.c_int32),
        ("B", ctypes.c_int32),
        ("Hq", ctypes.c_int32),
        ("Hkv", ctypes.c_int32),
        ("N", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("key_mask", ctypes.c_void_p),
        ("key_mask_bstride", ctypes.c_int64),
        ("query_mask", ctypes.c_void_p),
        ("query_mask_bstride", ctypes.c_int64),
        ("pair_mask", ctypes.c_void_p),
        ("pair_mask_bstride", ctypes.c_int64),
        ("pair_mask_rstride", ctypes.c_int64),
        ("scale", ctypes.c_double),
        ("block_size", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("causal_skip", ctypes.c_int32),
        ("unit_begin", ctypes.c_int32),
        ("unit_end", ctypes.c_int32),
    ]


class PagedKV(ctypes.Structure):
    """Mirror of ``struct kvbm_paged_kv``."""

    _fields_ = [
        ("k_cache", ctypes.c_void_p),
        ("cache_stride", ctypes.c_int64 * 4),
        ("num_pages", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("block_table", ctypes.c_void_p),
        ("block_table_stride", ctypes.c_int64),
        ("max_pages", ctypes.c_int32),
    ]


class Options(ctypes.Structure):
    """Mirror of ``struct kvbm_options``."""

    _fields_ = [
        ("lse", ctypes.c_void_p),
        ("lse_stride", ctypes.c_int64 * 3),
        ("paged", ctypes.POINTER(PagedKV)),
        ("seq_lens", ctypes.c_void_p),
        ("cu_seqlens", ctypes.c_void_p),
        ("total_tokens", ctypes.c_int64),
        ("per_sequence", ctypes.c_int32),
        ("events", ctypes.POINTER(ctypes.c_void_p)),
        ("stages", ctypes.c_int32),
        ("run_unit_begin", ctypes.c_int32),
        ("run_unit_end", ctypes.c_int32),
        ("run_head_begin", ctypes.c_int32),
        ("run_head_end", ctypes.c_int32),
        ("run_row_begin", ctypes.c_int32),
        ("run_row_end", ctypes.c_int32),
        ("method", ctypes.c_int32),
    ]


class DesignArgs(ctypes.Structure):
    """Mirror of ``struct kvbm_design_args``."""

    _fields_ = [
        ("mass", ctypes.c_void_p),
        ("mass_dtype", ctypes.c_int32),
        ("rows", ctypes.c_int32),
        ("mass_row_stride", ctypes.c_int64),
        ("num_blocks", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("n_sinks", ctypes.c_int32),
        ("recency", ctypes.c_int32),
        ("top_slice", ctypes.c_int32),
        ("tail_budget", ctypes.c_int64),
        ("eps", ctypes.c_double),
        ("uniform_tail", ctypes.c_int32),
        ("uniforms", ctypes.POINTER(ctypes.c_double)),
        ("uniforms_row_stride", ctypes.c_int64),
        ("seed", ctypes.c_uint64),
    ]


class DesignOut(ctypes.Structure):
    """Mirror of ``struct kvbm_design_out``."""

    _fields_ = [
        ("pi", ctypes.POINTER(ctypes.c_double)),
        ("keep", ctypes.POINTER(ctypes.c_uint8)),
        ("certainty", ctypes.POINTER(ctypes.c_uint8)),
        ("scores", ctypes.POINTER(ctypes.c_double)),
        ("log_offsets", ctypes.POINTER(ctypes.c_double)),
        ("counts", ctypes.POINTER(ctypes.c_int64)),
    ]


_lib = None


def load() -> ctypes.CDLL:
    """Load ``libkvbm.so`` once and declare its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python kv-block-mass_b200/build.py` "
            "(there is no CPU fallback for the block-mass kernels)")
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    P = ctypes.POINTER(Problem)
    lib.kvbm_abi_version.restype = ctypes.c_int
    lib.kvbm_abi_version.argtypes = []
    lib.kvbm_status_string.restype = ctypes.c_char_p
    lib.kvbm_status_string.argtypes = [ctypes.c_int]
    lib.kvbm_validate.restype = ctypes.c_int
    lib.kvbm_validate.argtypes = [P]
    lib.kvbm_num_blocks.restype = ctypes.c_int64
    lib.kvbm_num_blocks.argtypes = [ctypes.c_int32, ctypes.c_int32]
    lib.kvbm_workspace_bytes.restype = ctypes.c_size_t
    lib.kvbm_workspace_bytes.argtypes = [P]
    lib.kvbm_kernel_path.restype = ctypes.c_int
    lib.kvbm_kernel_path.argtypes = [P]
    lib.kvbm_launches_per_call.restype = ctypes.c_int
    lib.kvbm_launches_per_call.argtypes = [P]
    lib.kvbm_block_mass.restype = ctypes.c_int
    lib.kvbm_block_mass.argtypes = [P, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                    ctypes.c_void_p]
    lib.kvbm_block_mass_events.restype = ctypes.c_int
    lib.kvbm_block_mass_events.argtypes = [P, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                           ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
    lib.kvbm_block_mass_lse.restype = ctypes.c_int
    lib.kvbm_block_mass_lse.argtypes = [P, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.kvbm_measure_ex2_rate.restype = ctypes.c_int
    lib.kvbm_measure_ex2_rate.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_double)]
    lib.kvbm_exp2_fma_fraction.restype = ctypes.c_double
    lib.kvbm_exp2_fma_fraction.argtypes = []
    # No-allocation variant: scratch from a fixed device array inside the library.
    lib.kvbm_block_mass_static.restype = ctypes.c_int
    lib.kvbm_block_mass_static.argtypes = [P, ctypes.c_void_p, ctypes.c_void_p]
    lib.kvbm_static_scratch_bytes.restype = ctypes.c_size_t
    lib.kvbm_static_scratch_bytes.argtypes = []
    # Paged key cache (gathered into the workspace, then the dense kernels).
    K = ctypes.POINTER(PagedKV)
    lib.kvbm_validate_paged.restype = ctypes.c_int
    lib.kvbm_validate_paged.argtypes = [P, K]
    lib.kvbm_paged_workspace_bytes.restype = ctypes.c_size_t
    lib.kvbm_paged_workspace_bytes.argtypes = [P, K]
    lib.kvbm_block_mass_paged.restype = ctypes.c_int
    lib.kvbm_block_mass_paged.argtypes = [P, K, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    # Every option combined (paged / ragged / packed / LSE input / per-sequence output).
    O = ctypes.POINTER(Options)
    lib.kvbm_validate_ex.restype = ctypes.c_int
    lib.kvbm_validate_ex.argtypes = [P, O]
    lib.kvbm_workspace_bytes_ex.restype = ctypes.c_size_t
    lib.kvbm_workspace_bytes_ex.argtypes = [P, O]
    lib.kvbm_block_mass_ex.restype = ctypes.c_int
    lib.kvbm_block_mass_ex.argtypes = [P, O, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    # Device-side consumers (eviction design).
    lib.kvbm_design_workspace_bytes.restype = ctypes.c_size_t
    lib.kvbm_design_workspace_bytes.argtypes = [ctypes.POINTER(DesignArgs)]
    lib.kvbm_design.restype = ctypes.c_int
    lib.kvbm_design.argtypes = [ctypes.POINTER(DesignArgs), ctypes.POINTER(DesignOut), ctypes.c_void_p,
                                ctypes.c_size_t, ctypes.c_void_p]
    lib.kvbm_selftest_wait_timeout.restype = ctypes.c_int
    lib.kvbm_selftest_wait_timeout.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.POINTER(ctypes.c_int)]
    lib.kvbm_copy_2d_async.restype = ctypes.c_int
    lib.kvbm_copy_2d_async.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_void_p]
    lib.kvbm_method.restype = ctypes.c_int
    lib.kvbm_method.argtypes = [P, O]
    lib.kvbm_check_device_errors.restype = ctypes.c_int
    lib.kvbm_check_device_errors.argtypes = [ctypes.c_void_p]
    if lib.kvbm_abi_version() != ABI_VERSION:
        raise RuntimeError(f"libkvbm ABI {lib.kvbm_abi_version()} != {ABI_VERSION}: rebuild it with "
                           "`python kv-block-mass_b200/build.py`")
    _lib = lib
    return lib


def status_string(code: int) -> str:
    return load().kvbm_status_string(int(code)).decode()
