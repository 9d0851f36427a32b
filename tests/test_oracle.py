"""Pin the CPU oracle to the reference's own outputs (CPU only).

The golden vectors under ``tests/golden/`` were produced by running
kv-block-mass's ``block_mass_reference`` and its dense test oracle
(``tests/naive.py``) — see ``tests/golden/gen_golden.py``.  These tests show
that the numpy restatement in ``oracle/block_mass_np.py`` reproduces them, so
the GPU parity tests may use the oracle where no golden vector exists.
"""

import numpy as np
import pytest
import torch

from conftest import load_golden
from _helpers import case_inputs, checksum_ok, max_rel
from oracle import block_mass_np as orc


def test_golden_fixtures_present():
    for name in ("small_cases", "cpu_ref_n2048", "gqa_n8192_fp32"):
        assert load_golden(name) is not None, name


@pytest.mark.parametrize("idx", range(22))
def test_oracle_matches_reference_fp64(small_cases, idx):
    """fp64 oracle vs the reference's fp64 output on its own test shapes."""
    c = small_cases[idx]
    q, k, mask = case_inputs(c)
    got = orc.block_mass_stream(q.numpy(), k.numpy(), attn_mask=None if mask is None else mask.numpy(),
                                causal=c["causal"], block_size=c["block_size"])
    assert got.dtype == np.float64
    assert len(got) == len(c["mass_ref_fp64"])
    np.testing.assert_allclose(got, c["mass_ref_fp64"], rtol=1e-12, atol=1e-12)
    assert c["mass_ref_fp64_noskip_identical"]
    if c["mass_naive_fp64"] is not None:
        np.testing.assert_allclose(got, c["mass_naive_fp64"], rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("idx", range(22))
def test_oracle_matches_reference_fp32(small_cases, idx):
    c = small_cases[idx]
    q, k, mask = case_inputs(c)
    got = orc.block_mass_stream(q.float().numpy(), k.float().numpy(),
                                attn_mask=None if mask is None else mask.numpy(),
                                causal=c["causal"], block_size=c["block_size"])
    assert got.dtype == np.float32
    assert max_rel(got, c["mass_ref_fp32"]) < 2e-6


@pytest.mark.parametrize("idx", range(22))
def test_segment_lse_identity_matches_reference(small_cases, idx):
    """The one-pass method's identity, mass[j] = sum_i 2^(L_ij - lse2_i) with
    L_ij the row's log2-sum-exp2 over bucket j's keys, accumulated per 64-key
    piece against a running max as the kernel does, reproduces the
    reference's fp64 output on every one of its test shapes (masks, dead rows,
    GQA, ragged N, every block size they use)."""
    c = small_cases[idx]
    if c["N"] > 300:
        pytest.skip("per-row Python loop: small cases only")
    q, k, mask = case_inputs(c)
    got = orc.block_mass_segment_lse(q.numpy(), k.numpy(), attn_mask=None if mask is None else mask.numpy(),
                                     causal=c["causal"], block_size=c["block_size"])
    np.testing.assert_allclose(got, c["mass_ref_fp64"], rtol=1e-11, atol=1e-11)


@pytest.mark.parametrize("idx", range(22))
def test_dense_restatement_matches(small_cases, idx):
    c = small_cases[idx]
    q, k, mask = case_inputs(c)
    if mask is not None and mask.dim() == 1:
        pytest.skip("the reference's dense oracle takes [N, N] masks only")
    got = orc.dense_block_mass(q.numpy(), k.numpy(), attn_mask=None if mask is None else mask.numpy(),
                               causal=c["causal"], block_size=c["block_size"])
    np.testing.assert_allclose(got, c["mass_ref_fp64"], rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("name", ["cpu_ref_n2048", "gqa_n8192_fp32"])
def test_oracle_matches_reference_workloads(name):
    """The fp32 benchmark shapes, checked against the reference's fp32 and fp64 runs."""
    from kvblockmass_b200.workloads import WORKLOADS, make_inputs

    g = load_golden(name)
    w = WORKLOADS[name]
    q, k, km, qm = make_inputs(w)
    assert checksum_ok(q, g["q_checksum"]) and checksum_ok(k, g["k_checksum"])
    got = orc.block_mass_stream(q.numpy(), k.numpy(), causal=w.causal, block_size=w.block_size,
                                threads=8)
    assert max_rel(got, g["mass_ref_fp32"]) < 2e-6
    assert max_rel(got, g["mass_ref_fp64"]) < 2e-5
    assert g["mass_ref_fp32_noskip_identical"]
    # sum rule: every row keeps its diagonal key, so sum = B * H_q * N
    assert abs(float(np.sum(g["mass_ref_fp64"])) - w.B * w.Hq * w.N) < 1e-6 * w.B * w.Hq * w.N


def test_oracle_causal_skip_bit_identical():
    """Skipping keys above the causal diagonal changes work, never values (reference.py:96-100)."""
    q, k = torch.randn(1, 4, 600, 16, dtype=torch.float64, generator=torch.Generator().manual_seed(71)), None
    k = torch.randn(1, 2, 600, 16, dtype=torch.float64, generator=torch.Generator().manual_seed(72))
    a = orc.block_mass_stream(q.numpy(), k.numpy(), causal=True, block_size=64)
    b = orc.block_mass_stream(q.numpy(), k.numpy(), causal=True, block_size=64, causal_skip=False)
    np.testing.assert_allclose(a, b, rtol=1e-12, atol=0)


def test_oracle_engagement_extents():
    """Key extents per chunk match the reference's engagement test (test_reference.py:189-215)."""
    assert orc.causal_skip_extents(1024, 256, True, True) == [256, 512, 768, 1024]
    assert orc.causal_skip_extents(1024, 256, True, False) == [1024] * 4


def test_oracle_gqa_error():
    q = np.zeros((1, 6, 8, 4))
    k = np.zeros((1, 4, 8, 4))
    with pytest.raises(ValueError, match="GQA requires H_q % H_kv == 0"):
        orc.block_mass_stream(q, k, block_size=4)


def test_oracle_extensions_by_linearity():
    """Per-batch masks and the query-row mask equal per-batch reference runs."""
    g = torch.Generator().manual_seed(5)
    B, Hq, Hkv, N, D = 3, 4, 2, 150, 16
    q = torch.randn(B, Hq, N, D, generator=g, dtype=torch.float64).numpy()
    k = torch.randn(B, Hkv, N, D, generator=g, dtype=torch.float64).numpy()
    km = (torch.rand(B, 1, N, generator=g) > 0.2).numpy()
    qm = (torch.rand(B, N, generator=g) > 0.1).numpy()
    got = orc.block_mass_stream(q, k, attn_mask=km, query_mask=qm, causal=True, block_size=32)
    want = np.zeros_like(got)
    for b in range(B):
        pair = km[b, 0][None, :] & qm[b][:, None]
        want += orc.dense_block_mass(q[b:b + 1], k[b:b + 1], attn_mask=pair, causal=True, block_size=32)
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-10)
    # sum rule with dead rows: rows whose keep set is empty contribute exactly 0
    alive = 0
    for b in range(B):
        for i in range(N):
            alive += bool(qm[b, i] and km[b, 0, : i + 1].any())
    assert abs(got.sum() - Hq * alive) < 1e-8 * Hq * alive


# ---------------------------------------------------------------- mutation gate
def _mutant(q, k, causal, block_size, bug):
    """The oracle's chunk loop with one planted bug (the reference's four,
    tests/mutation_gate.py:7-18).  Bugs live only here, in the CPU checker."""
    B, Hq, N, D = q.shape
    G = Hq // k.shape[1]
    kf = np.repeat(k, G, axis=1)
    scale = 1.0 / D ** 0.5
    nb = orc.num_blocks(N, block_size)
    col_block = np.arange(N) // block_size
    if bug == "BUCKET_OFF_BY_ONE":
        col_block = (col_block + 1) % nb
    mass = np.zeros(nb)
    for start in range(0, N, 256):
        stop = min(start + 256, N)
        use_causal = causal and bug != "CAUSAL_DROPPED"
        n_lim = (start if bug == "EARLY_EXIT_TOO_TIGHT" else stop) if use_causal else N
        if n_lim == 0:
            continue
        rows = np.arange(start, stop)
        keep = rows[:, None] >= np.arange(n_lim)[None, :] if use_causal else np.ones((stop - start, n_lim), bool)
        s = q[:, :, start:stop] @ np.swapaxes(kf[:, :, :n_lim], -1, -2) * scale
        s = np.where(keep, s, -np.inf)
        with np.errstate(invalid="ignore"):
            if bug == "NO_DENOM":
                w = np.exp(s)
            else:
                m = s.max(-1, keepdims=True)
                e = np.exp(s - m)
                w = e / e.sum(-1, keepdims=True)
        w = np.nan_to_num(w, nan=0.0)
        mass += np.bincount(col_block[:n_lim], weights=w.sum((0, 1)).sum(0), minlength=nb)
    return mass


@pytest.mark.parametrize("bug", ["none", "CAUSAL_DROPPED", "NO_DENOM", "BUCKET_OFF_BY_ONE",
                                 "EARLY_EXIT_TOO_TIGHT"])
def test_mutation_gate(small_cases, bug):
    """The golden comparison used by the parity tests catches each planted bug."""
    c = next(x for x in small_cases if x["name"] == "skip_n600_gqa")
    q, k, _ = case_inputs(c)
    got = _mutant(q.numpy(), k.numpy(), True, c["block_size"], bug)
    ok = np.allclose(got, c["mass_ref_fp64"], rtol=1e-5, atol=1e-8)
    assert ok == (bug == "none"), f"{bug}: caught={not ok}"
