"""Shared helpers: regenerate golden inputs from their recipes and compare."""

from __future__ import annotations

import math

import numpy as np
import torch


def qk_test(B, H_q, H_kv, N, D, seed, dtype=torch.float64):
    """Input protocol of the reference's tests (``tests/test_reference.py:10-14``)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H_q, N, D, generator=g, dtype=dtype)
    k = torch.randn(B, H_kv, N, D, generator=g, dtype=dtype)
    return q, k


def mask_recipe(kind, N, seed=None):
    """Masks of the reference's tests (same recipes as tests/golden/gen_golden.py)."""
    if kind is None:
        return None
    if kind == "keys_first_half":
        m = torch.ones(N, dtype=torch.bool)
        m[N // 2:] = False
        return m
    if kind == "row0_dead":
        m = torch.ones(N, N, dtype=torch.bool)
        m[0, :] = False
        return m
    if kind == "rows_from_64_dead":
        m = torch.ones(N, N, dtype=torch.bool)
        m[64:, :] = False
        return m
    if kind == "rand_pairs":
        return torch.rand(N, N, generator=torch.Generator().manual_seed(seed)) > 0.5
    if kind == "rand_keys":
        return torch.rand(N, generator=torch.Generator().manual_seed(seed)) > 0.3
    raise ValueError(kind)


def checksum_ok(t: torch.Tensor, ref: dict) -> bool:
    t64 = t.to(torch.float64).reshape(-1)
    return (math.isclose(float(t64.sum()), ref["sum"], rel_tol=1e-12, abs_tol=1e-9)
            and math.isclose(float(t64.abs().sum()), ref["abs_sum"], rel_tol=1e-12)
            and [float(x) for x in t64[:4]] == ref["first"]
            and [float(x) for x in t64[-4:]] == ref["last"])


def case_inputs(case: dict):
    q, k = qk_test(case["B"], case["Hq"], case["Hkv"], case["N"], case["D"], case["seed"])
    assert checksum_ok(q, case["q_checksum"]) and checksum_ok(k, case["k_checksum"]), \
        f"{case['name']}: regenerated inputs differ from the golden recipe"
    return q, k, mask_recipe(case["mask"], case["N"], case["mask_seed"])


def max_rel(a, b, floor: float = 1e-6) -> float:
    """Max per-bucket relative error |a-b| / max(|b|, floor)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float((np.abs(a - b) / np.maximum(np.abs(b), floor)).max()) if a.size else 0.0
