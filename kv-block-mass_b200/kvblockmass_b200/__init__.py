"""kvblockmass_b200: block-granular attention mass on B200 (sm_100a).

    mass[j] = sum over (b, h_q, query i, key c in block j) of softmax_c(q_i . k_c * scale)

A drop-in for the GPU path of kv-block-mass (``block_mass`` /
``block_mass_triton``), computed by hand-written CUDA kernels behind the C ABI
of ``include/kvbm.h`` (``libkvbm.so``, loaded with ctypes).

Beyond the reference's entry points:

* ``block_mass_b200(..., lse=, seq_lens=, per_sequence=)``: row LSE input,
  ragged batches, one mass row per sequence;
* ``block_mass_varlen``: packed (varlen) batches with ``cu_seqlens``;
* ``block_mass_paged``: keys from a paged KV cache and block table;
* ``design_from_mass``: the reference's eviction design (evict.py) on the GPU;
* ``kvblockmass_b200.distributed``: (batch, kv-head) shards over ranks.
"""

__version__ = "0.1.0"

from .ops import (  # noqa: F401
    block_mass,
    block_mass_b200,
    block_mass_paged,
    block_mass_triton,
    block_mass_varlen,
    check_device_errors,
    kernel_path,
    method_of,
    launches_per_call,
    make_paged_problem,
    make_problem,
    make_varlen_problem,
    paged_workspace_bytes,
    run_paged,
    run_prepared,
    workspace_bytes,
)
from .design import DeviceDesign, design_from_mass  # noqa: F401
from .workloads import WORKLOADS, Workload, make_inputs, pairs  # noqa: F401

__all__ = [
    "block_mass_b200",
    "block_mass_triton",
    "block_mass",
    "block_mass_paged",
    "block_mass_varlen",
    "make_varlen_problem",
    "run_prepared",
    "make_paged_problem",
    "paged_workspace_bytes",
    "run_paged",
    "check_device_errors",
    "design_from_mass",
    "DeviceDesign",
    "kernel_path",
    "method_of",
    "make_problem",
    "workspace_bytes",
    "launches_per_call",
    "WORKLOADS",
    "Workload",
    "make_inputs",
    "pairs",
    "__version__",
]
