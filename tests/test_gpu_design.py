"""Device-side eviction design (``kvbm_design``) against the reference's own
designs (``tests/golden/evict_cases.json``) and the oracle (``oracle/evict_np.py``).

With the reference's uniforms the device design equals the reference's
exactly wherever the top slice does not split a run of tied scores (there
the reference's pick is ``torch.topk``'s); against the oracle, which takes
the lower index among ties like the kernel, it is exact everywhere.  pi is
compared to 1e-13 relative (the tail total's summation order differs).
"""

import numpy as np
import pytest
import torch

from oracle import evict_np as ev
from test_oracle_evict import case_arrays, compare_design, load_cases

import kvblockmass_b200 as kb

pytestmark = pytest.mark.gpu


def run_case(c, dev, mass=None, u=None):
    if mass is None:
        mass, u, *_ = case_arrays(c)
    return kb.design_from_mass(torch.from_numpy(mass).to(dev), c["seq_len"], c["block_size"], c["tail_budget"],
                               n_sinks=c["n_sinks"], recency=c["recency"], top_slice=c["top_slice"], eps=c["eps"],
                               uniform_tail=c["uniform_tail"], uniforms=torch.from_numpy(u).to(dev),
                               with_scores=True, with_log_offsets=True)


def oracle_case(c, mass, u):
    sc = ev.expand_block_scores(mass, c["seq_len"], c["block_size"])
    return ev.design_from_scores(sc, c["tail_budget"], n_sinks=c["n_sinks"], recency=c["recency"],
                                 top_slice=c["top_slice"], eps=c["eps"], uniforms=u,
                                 uniform_tail=c["uniform_tail"])


@pytest.mark.parametrize("c", load_cases(), ids=lambda c: c["name"])
def test_design_matches_reference(cuda_device, c):
    mass, u, ref_pi, ref_keep, ref_cert = case_arrays(c)
    d = run_case(c, cuda_device)
    keep, pi, cert = d.keep.cpu().numpy(), d.pi.cpu().numpy(), d.certainty.cpu().numpy()
    compare_design(c, keep, pi, cert, mass, ref_pi, ref_keep, ref_cert)
    # against the oracle (same tie rule): exact
    k2, p2, c2 = oracle_case(c, mass, u)
    assert np.array_equal(cert, c2) and np.array_equal(keep, k2)
    assert np.allclose(pi, p2, rtol=1e-13, atol=0)
    counts = d.counts[0].cpu().tolist()
    assert counts[0] == int(k2.sum()) and counts[1] == int(c2.sum()) and counts[2] == int((~c2).sum())
    assert counts[3] == ev.block_retention(k2, c["seq_len"], c["block_size"]) and counts[4] == 0
    assert np.array_equal(d.scores.cpu().numpy(), ev.expand_block_scores(mass, c["seq_len"], c["block_size"]))
    assert np.allclose(d.log_offsets.cpu().numpy(), ev.hajek_log_offsets(p2), rtol=1e-12, atol=1e-15)


def test_generator_mode_reproduces_reference(cuda_device):
    """generator= draws the reference's uniforms: same design for a tie-free case."""
    c = next(c for c in load_cases() if c["name"] == "top_on_block_edge")
    mass, _, ref_pi, ref_keep, ref_cert = case_arrays(c)
    d = kb.design_from_mass(torch.from_numpy(mass).to(cuda_device), c["seq_len"], c["block_size"],
                            c["tail_budget"], n_sinks=c["n_sinks"], recency=c["recency"], top_slice=c["top_slice"],
                            eps=c["eps"], generator=torch.Generator().manual_seed(c["seed"]))
    assert np.array_equal(d.keep.cpu().numpy(), ref_keep)
    assert np.array_equal(d.certainty.cpu().numpy(), ref_cert)
    assert np.allclose(d.pi.cpu().numpy(), ref_pi, rtol=1e-13, atol=0)
    assert int(d.n_kept()) == c["n_kept"] and int(d.blocks_kept()) == c["blocks_kept"]


@pytest.mark.parametrize("N,bs,top", [(131072, 64, 5000), (20000, 1, 777), (32768, 16, 0), (4097, 4096, 3000)])
def test_large_designs_vs_oracle(cuda_device, N, bs, top):
    rng = np.random.default_rng(N + bs)
    nb = -(-N // bs)
    mass = rng.integers(0, 50, nb).astype(np.float64) * 0.25        # many ties
    u = rng.random(N)
    c = {"seq_len": N, "block_size": bs, "tail_budget": N // 10, "n_sinks": 4, "recency": 128,
         "top_slice": top, "eps": 1e-6, "uniform_tail": False}
    d = run_case(c, cuda_device, mass=mass, u=u)
    k2, p2, c2 = oracle_case(c, mass, u)
    assert np.array_equal(d.certainty.cpu().numpy(), c2)
    assert np.array_equal(d.keep.cpu().numpy(), k2)
    assert np.allclose(d.pi.cpu().numpy(), p2, rtol=1e-12, atol=0)


def test_rows_and_block_mass_input(cuda_device):
    """Per-sequence mass rows from the block-mass kernels, designed in one call."""
    g = torch.Generator().manual_seed(70)
    q = torch.randn(4, 8, 2000, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    k = torch.randn(4, 2, 2000, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    lens = torch.tensor([2000, 1500, 999, 64], dtype=torch.int32, device=cuda_device)
    per = kb.block_mass_b200(q, k, causal=True, block_size=16, seq_lens=lens, per_sequence=True)  # [4, 125] fp32
    u = torch.rand(4, 2000, dtype=torch.float64, generator=g)
    d = kb.design_from_mass(per, 2000, 16, 200, n_sinks=4, recency=32, top_slice=100, uniforms=u)
    per_h = per.cpu().numpy().astype(np.float64)
    for r in range(4):
        sc = ev.expand_block_scores(per_h[r], 2000, 16)
        k2, p2, c2 = ev.design_from_scores(sc, 200, n_sinks=4, recency=32, top_slice=100, uniforms=u[r].numpy())
        assert np.array_equal(d.keep[r].cpu().numpy(), k2)
        assert np.allclose(d.pi[r].cpu().numpy(), p2, rtol=1e-12, atol=0)
        assert int(d.counts[r, 0]) == int(k2.sum())


def test_philox_budget_and_reproducibility(cuda_device):
    """The reference's budget test (tests/test_evict.py:43-57) on 300 rows in one call."""
    n, m, rows = 256, 20, 300
    g = torch.Generator().manual_seed(71)
    mass = torch.rand(rows, n, dtype=torch.float64, generator=g).to(cuda_device)
    d = kb.design_from_mass(mass, n, 1, m, n_sinks=2, recency=4, seed=1234)
    tail_kept = (d.counts[:, 0] - d.counts[:, 1]).double()
    sd = (m / rows) ** 0.5
    assert abs(float(tail_kept.mean()) - m) <= 4 * sd
    again = kb.design_from_mass(mass, n, 1, m, n_sinks=2, recency=4, seed=1234)
    other = kb.design_from_mass(mass, n, 1, m, n_sinks=2, recency=4, seed=99)
    assert torch.equal(again.keep, d.keep)
    assert not torch.equal(other.keep, d.keep)
    assert torch.equal(again.pi, d.pi)


def test_negative_mass_is_flagged(cuda_device):
    mass = torch.tensor([1.0, -2.0, 3.0], dtype=torch.float64, device=cuda_device)
    d = kb.design_from_mass(mass, 3, 1, 1, n_sinks=0, recency=0, seed=0)
    with pytest.raises(ValueError, match="non-negative"):
        d.check()
    kb.design_from_mass(mass.abs(), 3, 1, 1, n_sinks=0, recency=0, seed=0).check()
