"""Generate golden eviction designs by running the reference's consumers.

Runs kv-block-mass's own ``expand_block_scores`` and ``design_from_scores``
(``src/kvblockmass/evict.py``) and ``plan_reclaim``'s block retention count
(``src/kvblockmass/reclaim.py:46-55``) on seeded block-mass vectors and writes
``evict_cases.json`` next to this script.  Every case stores its block mass,
the arguments, the uniforms the reference drew for the tail (the reference uses the first ``n_tail`` of
``torch.rand(seq_len, float64, generator=seed)``, which equal its own
``torch.rand(n_tail, ...)``) and the
reference's ``pi``, ``keep`` and ``certainty``, as base64 of little-endian
float64 / packed bits.

``ties_at_boundary`` marks cases whose top slice ends inside a run of equal
scores: there the reference's choice among the tied tokens is whatever
``torch.topk`` returns (not a documented order), so only tie-insensitive
properties are compared for them.

Usage (needs the reference sources; the fixtures do not)::

    KVBM_REF=/root/reference python tests/golden/gen_evict_golden.py
"""

from __future__ import annotations

import base64
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("KVBM_REF", "/root/reference"))
sys.path.insert(0, str(REF / "src"))

from kvblockmass.evict import design_from_scores, expand_block_scores  # noqa: E402


def b64f(a) -> str:
    return base64.b64encode(np.ascontiguousarray(np.asarray(a, dtype="<f8")).tobytes()).decode()


def b64bits(a) -> str:
    return base64.b64encode(np.packbits(np.asarray(a, dtype=bool), bitorder="little").tobytes()).decode()


def block_retention(keep, seq_len, block_size):
    nb = -(-seq_len // block_size)
    return sum(bool(keep[b * block_size:min(seq_len, (b + 1) * block_size)].any()) for b in range(nb))


# (name, num_blocks, seq_len, block_size, tail_budget, n_sinks, recency, top_slice, eps, uniform_tail,
#  mass recipe, seed)
CASES = [
    ("typical", 16, 1000, 64, 100, 4, 32, 50, 1e-6, False, "distinct", 1),
    ("top_on_block_edge", 16, 1024, 64, 128, 4, 32, 128, 1e-6, False, "distinct", 2),
    ("no_top", 8, 512, 64, 40, 4, 32, 0, 1e-6, False, "distinct", 3),
    ("ragged_last_block", 10, 601, 64, 60, 1, 7, 30, 1e-4, False, "distinct", 4),
    ("budget_clips", 12, 700, 64, 500, 2, 8, 0, 1e-6, False, "skewed", 5),
    ("uniform_tail", 8, 500, 64, 50, 4, 32, 20, 1e-6, True, "distinct", 6),
    ("zero_mass", 8, 400, 64, 30, 1, 1, 0, 1e-6, False, "zeros", 7),
    ("zero_budget", 8, 400, 64, 0, 4, 16, 10, 1e-3, False, "distinct", 8),
    ("all_certain", 4, 100, 32, 10, 60, 60, 0, 1e-6, False, "distinct", 9),
    ("block_size_1", 300, 300, 1, 25, 2, 5, 17, 1e-6, False, "distinct", 10),
    ("extra_blocks", 20, 900, 64, 90, 4, 32, 40, 1e-6, False, "distinct", 11),
    ("top_covers_all", 4, 200, 64, 20, 0, 0, 500, 1e-6, False, "distinct", 12),
    ("tied_blocks", 16, 1000, 64, 100, 4, 32, 100, 1e-6, False, "tied", 13),
    ("causal_like", 32, 2048, 64, 256, 4, 32, 128, 1e-6, False, "causal", 14),
    ("eps_floor_binds", 16, 1024, 64, 64, 4, 32, 64, 1e-4, False, "tiny", 15),
]


def mass_for(recipe: str, nb: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if recipe == "distinct":
        return rng.permutation(nb).astype(np.float64) * 0.37 + rng.random(nb) * 0.01 + 0.05
    if recipe == "skewed":
        return np.exp(rng.standard_normal(nb) * 3.0)
    if recipe == "zeros":
        return np.zeros(nb)
    if recipe == "tied":
        return rng.integers(1, 4, nb).astype(np.float64)
    if recipe == "tiny":  # half the blocks ~1e-9 of the others: their pi falls under eps
        return np.where(rng.random(nb) < 0.5, 1e-9, 1.0) * (1.0 + rng.random(nb))
    if recipe == "causal":  # fp32-valued, decaying like a causal mass vector
        return (np.arange(nb, 0, -1) * (1.0 + 0.1 * rng.random(nb))).astype(np.float32).astype(np.float64)
    raise ValueError(recipe)


def main():
    out = []
    for (name, nb, n, bs, m, sinks, rec, top, eps, uni, recipe, seed) in CASES:
        mass = mass_for(recipe, nb, seed)
        scores = expand_block_scores(torch.from_numpy(mass), n, bs)
        d = design_from_scores(scores, m, n_sinks=sinks, recency=rec, top_slice=top, eps=eps,
                               generator=torch.Generator().manual_seed(seed), uniform_tail=uni)
        # the reference drew torch.rand(n_tail) from this generator; rand(n)[:k] == rand(k) for
        # this generator, so seq_len draws cover any tail length a restatement may find
        u = torch.rand(n, dtype=torch.float64, generator=torch.Generator().manual_seed(seed))
        k = min(top, n)
        s_sorted = np.sort(scores.numpy())[::-1]
        ties = bool(0 < k < n and s_sorted[k - 1] == s_sorted[k])
        out.append({
            "name": name, "num_blocks": nb, "seq_len": n, "block_size": bs, "tail_budget": m,
            "n_sinks": sinks, "recency": rec, "top_slice": top, "eps": eps, "uniform_tail": uni,
            "seed": seed, "mass": b64f(mass), "uniforms": b64f(u.numpy()),
            "pi": b64f(d.pi.numpy()), "keep": b64bits(d.keep.numpy()), "certainty": b64bits(d.certainty.numpy()),
            "n_kept": int(d.keep.sum()), "n_certain": int(d.certainty.sum()),
            "blocks_kept": block_retention(d.keep.numpy(), n, bs), "ties_at_boundary": ties,
        })
    path = HERE / "evict_cases.json"
    path.write_text(json.dumps({"generator": "tests/golden/gen_evict_golden.py",
                                "reference": "src/kvblockmass/evict.py (expand_block_scores, design_from_scores)",
                                "torch": torch.__version__, "cases": out}, indent=1))
    print(f"wrote {path} ({len(out)} cases)")


if __name__ == "__main__":
    main()
