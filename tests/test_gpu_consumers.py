"""The reference's own mass consumers run unchanged on this library's mass.

kv-block-mass turns the mass vector into an eviction plan with
``plan_reclaim`` (``src/kvblockmass/reclaim.py:58-124``), which calls
``expand_block_scores`` and ``design_from_scores`` (``src/kvblockmass/evict.py:64-174``)
and the byte audit (``budget.py:136-155``).  The drop-in claim is that those
functions take ``block_mass_b200(...).cpu()`` as they take the reference's
``block_mass_reference(...)``.  These tests import the unmodified reference
package (installed with ``pip install --target baseline/_ref``), feed it the
GPU mass of two workloads and the reference's own mass for the same inputs
(the golden fixtures), and compare the plans:

* the certainty sets are equal (the top slice takes whole blocks whose
  ranking the tolerance does not change: checked first);
* every tail inclusion probability agrees to 2x the mass tolerance;
* with the same seed the two designs draw the same uniforms, so kept tokens
  differ only where a uniform falls between the two probabilities (a few);
* the card's shape fields are equal, and its counts differ by those flips.
"""

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import load_golden
from _helpers import checksum_ok

import kvblockmass_b200 as kb
from kvblockmass_b200.workloads import WORKLOADS, make_inputs

pytestmark = pytest.mark.gpu

REF_SITE = Path(__file__).resolve().parent.parent / "baseline" / "_ref"


def _reference():
    if not (REF_SITE / "kvblockmass").is_dir():
        pytest.skip("the reference package is not installed in baseline/_ref")
    if str(REF_SITE) not in sys.path:
        sys.path.insert(0, str(REF_SITE))
    from kvblockmass import budget, evict, reclaim

    return budget, evict, reclaim


@pytest.mark.parametrize("name,tol", [("cpu_ref_n2048", 2e-5), ("llama3_8b_n32k", 1e-3)])
def test_reference_plan_reclaim_on_b200_mass(cuda_device, name, tol):
    budget, evict, reclaim = _reference()
    g = load_golden(name)
    w = WORKLOADS[name]
    q, k, _, _ = make_inputs(w)
    assert checksum_ok(q, g["q_checksum"]) and checksum_ok(k, g["k_checksum"])
    mine = kb.block_mass_b200(q.to(cuda_device), k.to(cuda_device), causal=w.causal,
                              block_size=w.block_size).cpu()
    theirs = torch.tensor(g["mass_ref_fp32"], dtype=torch.float32)
    assert mine.dtype == theirs.dtype and mine.shape == theirs.shape
    rel = float(((mine.double() - theirs.double()).abs() / theirs.double().abs().clamp_min(1e-6)).max())
    assert rel < tol

    N, bs = w.N, w.block_size
    top = N // 16
    # The top slice takes top // bs whole blocks: equal certainty sets need the
    # block ranking at that cut to be wider than the tolerance.
    srt = torch.sort(theirs.double(), descending=True).values
    nb_top = top // bs
    gap = float(srt[nb_top - 1] - srt[nb_top]) / float(srt[nb_top - 1])
    assert gap > 4 * tol, f"the top-slice cut is a near tie ({gap:.2e}); pick another budget"

    layout = budget.CacheLayout(n_layers=1, n_heads=w.Hq, seq_len=N, head_dim=w.D, item_bytes=2, block_size=bs)
    kw = dict(tail_budget=N // 8, n_sinks=4, recency=32, top_slice=top, seed=0)
    pa = reclaim.plan_reclaim(mine, bs, layout, **kw)
    pb = reclaim.plan_reclaim(theirs, bs, layout, **kw)

    da, db = pa.design, pb.design
    assert torch.equal(da.certainty, db.certainty)
    tail = ~db.certainty
    pr = ((da.pi[tail] - db.pi[tail]).abs() / db.pi[tail]).max()
    assert float(pr) < 2 * tol + 1e-12
    flips = int((da.keep != db.keep).sum())
    assert flips <= max(4, int(4 * tol * (N // 8)) + 4), flips
    for key in ("tail_budget", "top_slice", "n_sinks", "recency", "blocks_total", "bytes_full"):
        assert pa.card[key] == pb.card[key], key
    assert abs(pa.kept_tokens - pb.kept_tokens) <= flips
    assert abs(pa.card["blocks_kept"] - pb.card["blocks_kept"]) <= flips

    # the layer under plan_reclaim, called directly with a caller's generator
    sa = evict.expand_block_scores(mine, N, bs)
    sb = evict.expand_block_scores(theirs, N, bs)
    ea = evict.design_from_scores(sa, N // 8, n_sinks=4, recency=32, top_slice=top,
                                  generator=torch.Generator().manual_seed(3))
    eb = evict.design_from_scores(sb, N // 8, n_sinks=4, recency=32, top_slice=top,
                                  generator=torch.Generator().manual_seed(3))
    assert torch.equal(ea.certainty, eb.certainty)
    assert int((ea.keep != eb.keep).sum()) <= max(4, int(4 * tol * (N // 8)) + 4)
    off_a, off_b = evict.hajek_log_offsets(ea.pi), evict.hajek_log_offsets(eb.pi)
    assert np.allclose(off_a.numpy(), off_b.numpy(), rtol=0, atol=2 * tol + 1e-12)
