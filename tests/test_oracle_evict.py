"""Pins the consumers' oracle (``oracle/evict_np.py``) to the reference's own
outputs (``tests/golden/evict_cases.json``, made by ``gen_evict_golden.py``).

Where a case's top slice ends inside a run of equal scores, the reference's
choice among the tied tokens is ``torch.topk``'s and not reproducible; there
the comparison is exact outside the tied run and by counts and values inside.
"""

import base64
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import evict_np as ev

GOLDEN = Path(__file__).resolve().parent / "golden" / "evict_cases.json"


def f64(s):
    return np.frombuffer(base64.b64decode(s), dtype="<f8").copy()


def bits(s, n):
    return np.unpackbits(np.frombuffer(base64.b64decode(s), dtype=np.uint8), bitorder="little")[:n].astype(bool)


def load_cases():
    return json.loads(GOLDEN.read_text())["cases"]


def case_arrays(c):
    n = c["seq_len"]
    return (f64(c["mass"]), f64(c["uniforms"]), f64(c["pi"]), bits(c["keep"], n), bits(c["certainty"], n))


def tied_run(scores, k):
    """Token range whose score equals the k-th largest (where the top slice may split a tie)."""
    if k <= 0 or k >= scores.size:
        return np.zeros(scores.size, dtype=bool)
    t = np.sort(scores)[::-1][k - 1]
    return scores == t


def compare_design(c, keep, pi, cert, mass, ref_pi, ref_keep, ref_cert, rtol=1e-13):
    n, bs = c["seq_len"], c["block_size"]
    scores = ev.expand_block_scores(mass, n, bs)
    run = tied_run(scores, min(c["top_slice"], n)) if c["ties_at_boundary"] else np.zeros(n, dtype=bool)
    out = ~run
    fixed = np.zeros(n, dtype=bool)
    fixed[:min(c["n_sinks"], n)] = True
    if c["recency"]:
        fixed[max(0, n - c["recency"]):] = True
    assert np.all(cert[fixed]) and np.all(pi[cert] == 1.0)
    assert np.all((pi >= c["eps"]) & (pi <= 1.0))
    assert np.array_equal(cert[out], ref_cert[out])
    if (run & fixed).any():
        # the tied run reaches the sinks / recency window: which tied tokens the
        # top slice takes changes how many are certain, hence the tail total
        return
    assert np.allclose(pi[out], ref_pi[out], rtol=rtol, atol=0)
    assert int(cert.sum()) == c["n_certain"]
    # inside a tied run: the same number of certain tokens and the same tail value
    assert int(cert[run].sum()) == int(ref_cert[run].sum())
    assert np.allclose(np.sort(pi[run]), np.sort(ref_pi[run]), rtol=rtol, atol=0)
    # tail draws are assigned in ascending order: tokens after the run see the same draw
    after = np.zeros(n, dtype=bool)
    if run.any():
        after[np.nonzero(run)[0][-1] + 1:] = True
    else:
        after[:] = True
    assert np.array_equal(keep[after], ref_keep[after])
    if not c["ties_at_boundary"]:
        assert np.array_equal(keep, ref_keep)
        assert int(keep.sum()) == c["n_kept"]
        assert ev.block_retention(keep, n, bs) == c["blocks_kept"]


@pytest.mark.parametrize("c", load_cases(), ids=lambda c: c["name"])
def test_oracle_matches_reference_designs(c):
    mass, u, ref_pi, ref_keep, ref_cert = case_arrays(c)
    scores = ev.expand_block_scores(mass, c["seq_len"], c["block_size"])
    keep, pi, cert = ev.design_from_scores(scores, c["tail_budget"], n_sinks=c["n_sinks"], recency=c["recency"],
                                           top_slice=c["top_slice"], eps=c["eps"], uniforms=u,
                                           uniform_tail=c["uniform_tail"])
    compare_design(c, keep, pi, cert, mass, ref_pi, ref_keep, ref_cert)


def test_oracle_reference_unit_cases():
    """The reference's own known answers (tests/test_evict.py of kv-block-mass)."""
    assert np.array_equal(ev.expand_block_scores(np.array([1.0, 2.0]), 5, 3), [1, 1, 1, 2, 2])
    with pytest.raises(ValueError):
        ev.expand_block_scores(np.array([1.0, 2.0]), 9, 3)
    _, pi, _ = ev.design_from_scores(np.array([4.0, 1.0, 1.0]), 2, n_sinks=0, recency=0)
    assert np.allclose(pi, [1.0, 1 / 3, 1 / 3], atol=1e-12)
    _, pi, _ = ev.design_from_scores(np.array([10.0, 1, 1, 1]), 1, n_sinks=0, recency=0, uniform_tail=True)
    assert np.allclose(pi, 0.25)
    _, pi, cert = ev.design_from_scores(np.zeros(16), 4, n_sinks=1, recency=1)
    assert np.all(pi[~cert] > 0) and np.all(pi[~cert] <= 1)
    assert np.allclose(ev.hajek_log_offsets(np.array([1.0, 0.5, 0.25])), [0, np.log(2), np.log(4)])
    with pytest.raises(ValueError):
        ev.design_from_scores(np.array([1.0]), 1, eps=0.0)
    with pytest.raises(ValueError):
        ev.design_from_scores(np.array([-1.0, 2.0]), 1)


def test_top_slice_ties_go_to_lower_index():
    s = np.array([1.0, 3.0, 3.0, 2.0, 3.0, 3.0])
    assert np.array_equal(ev.top_slice_mask(s, 3), [0, 1, 1, 0, 1, 0])
    assert np.array_equal(ev.top_slice_mask(s, 10), np.ones(6, dtype=bool))


# ---------------------------------------------------------------- mutation gate
# Each mutant plants one mistake in a copy of the oracle's design; the golden
# comparison above must catch every one, and the unmutated control must pass.

def _mutant_design(kind):
    def design(scores, tail_budget, *, n_sinks=4, recency=32, top_slice=0, eps=1e-6, uniforms=None,
               uniform_tail=False):
        if kind == "recency_off_by_one" and recency:
            recency -= 1
        if kind == "sinks_dropped":
            n_sinks = 0
        if kind == "top_slice_dropped":
            top_slice = 0
        keep, pi, cert = ev.design_from_scores(scores, tail_budget, n_sinks=n_sinks, recency=recency,
                                               top_slice=top_slice, eps=eps, uniforms=uniforms,
                                               uniform_tail=uniform_tail)
        tail = ~cert
        if kind == "no_eps_floor" and tail.any() and tail_budget > 0:
            s = np.asarray(scores, dtype=np.float64)
            w = np.ones(tail.sum()) if uniform_tail else s[tail]
            if not w.sum() > 0:
                w = np.ones(tail.sum())
            pi[tail] = np.minimum(tail_budget * w / w.sum(), 1.0)
        if kind == "keep_threshold_loose" and tail.any():
            u = np.asarray(uniforms)[: int(tail.sum())]
            keep = cert.copy()
            keep[tail] = u <= 1.5 * pi[tail]
        return keep, pi, cert
    return design


def _caught(design):
    for c in load_cases():
        mass, u, ref_pi, ref_keep, ref_cert = case_arrays(c)
        sc = ev.expand_block_scores(mass, c["seq_len"], c["block_size"])
        keep, pi, cert = design(sc, c["tail_budget"], n_sinks=c["n_sinks"], recency=c["recency"],
                                top_slice=c["top_slice"], eps=c["eps"], uniforms=u, uniform_tail=c["uniform_tail"])
        try:
            compare_design(c, keep, pi, cert, mass, ref_pi, ref_keep, ref_cert)
        except AssertionError:
            return True
    return False


@pytest.mark.parametrize("kind", ["recency_off_by_one", "sinks_dropped", "top_slice_dropped", "no_eps_floor",
                                  "keep_threshold_loose"])
def test_mutants_are_caught(kind):
    assert _caught(_mutant_design(kind)), f"mutant {kind} passed every golden design"


def test_mutation_gate_control_passes():
    assert not _caught(_mutant_design("none"))
