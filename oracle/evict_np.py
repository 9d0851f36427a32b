"""CPU oracle for the block-mass consumers — TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may import this module; the CUDA design kernels never fall
back to it.  It restates, in numpy and float64, the reference's consumers of
the mass vector (kv-block-mass ``src/kvblockmass/evict.py``):

* ``expand_block_scores`` (``evict.py:64-83``): token ``i`` gets the score of
  block ``i // block_size``;
* ``design_from_scores`` (``evict.py:95-171``): certainty set = the first
  ``n_sinks`` tokens, the last ``recency`` tokens and the ``top_slice``
  highest scores; tail probabilities ``clip(m * w_i / sum_tail w, eps, 1)``
  with ``w`` the scores (all ones for ``uniform_tail``, and a uniform design
  when the tail's scores sum to 0); with ``m == 0`` every tail token gets
  ``eps``; a tail token is kept when its uniform draw ``u < pi``;
* ``hajek_log_offsets`` (``evict.py:174-187``): ``-log(pi)``;
* the block retention count of ``plan_reclaim`` (``reclaim.py:46-55``).

Two choices are explicit here where the reference leaves them to torch:

* the tail draws are an argument: ``uniforms[t]`` is the draw of the ``t``-th
  tail token in ascending index order, which is what the reference's
  ``torch.rand(n_tail, dtype=float64, generator=g)`` produces;
* the top slice breaks ties by index, lower index first, as the reference's
  ``_top_slice`` docstring states (``evict.py:86-87``); ``torch.topk`` itself
  does not promise an order among equal scores, so the reference's own choice
  inside a tied run is not reproducible and the parity tests compare only
  tie-insensitive properties there.

Pinned against the reference's outputs in ``tests/golden/evict_cases.json``
(``tests/golden/gen_evict_golden.py``).
"""

from __future__ import annotations

import numpy as np

__all__ = ["expand_block_scores", "top_slice_mask", "design_from_scores", "hajek_log_offsets",
           "block_retention"]


def expand_block_scores(block_scores, seq_len: int, block_size: int) -> np.ndarray:
    """``evict.py:64-83``: per-token float64 scores from per-block scores."""
    bs = np.asarray(block_scores)
    if bs.ndim != 1:
        raise ValueError(f"block_scores must be 1-D, got {bs.shape}")
    if bs.shape[0] * block_size < seq_len:
        raise ValueError(f"{bs.shape[0]} blocks of {block_size} cannot cover seq_len={seq_len}")
    return bs.astype(np.float64)[np.arange(seq_len) // block_size]


def top_slice_mask(scores: np.ndarray, n: int) -> np.ndarray:
    """``evict.py:86-92``: the ``n`` highest scores, ties to the lower index."""
    mask = np.zeros(scores.shape[0], dtype=bool)
    if n > 0:
        order = np.argsort(-scores, kind="stable")
        mask[order[:min(n, scores.shape[0])]] = True
    return mask


def design_from_scores(scores, tail_budget: int, *, n_sinks: int = 4, recency: int = 32, top_slice: int = 0,
                       eps: float = 1e-6, uniforms=None, uniform_tail: bool = False):
    """``evict.py:95-171``; returns ``(keep, pi, certainty)``.

    ``uniforms``: the draws of the tail tokens in ascending index order (at
    least ``n_tail`` values); ``None`` keeps no tail token (the draw is 1).
    """
    s = np.asarray(scores, dtype=np.float64)
    if s.ndim != 1:
        raise ValueError(f"scores must be 1-D, got {s.shape}")
    if eps <= 0:
        raise ValueError("eps must be > 0 (the design needs a positive floor)")
    if tail_budget < 0:
        raise ValueError("tail_budget must be >= 0")
    if np.any(s < 0):
        raise ValueError("scores must be non-negative")
    n = s.shape[0]
    certainty = np.zeros(n, dtype=bool)
    if n_sinks:
        certainty[:min(n_sinks, n)] = True
    if recency:
        certainty[max(0, n - recency):] = True
    if top_slice:
        certainty |= top_slice_mask(s, top_slice)
    tail_idx = np.nonzero(~certainty)[0]
    pi = np.ones(n, dtype=np.float64)
    if tail_idx.size and tail_budget > 0:
        w = np.ones(tail_idx.size) if uniform_tail else s[tail_idx]
        total = w.sum()
        if total <= 0:
            w = np.ones(tail_idx.size)
            total = w.sum()
        pi[tail_idx] = np.clip(tail_budget * w / total, eps, 1.0)
    elif tail_idx.size:
        pi[tail_idx] = eps
    keep = certainty.copy()
    if tail_idx.size:
        u = np.ones(tail_idx.size) if uniforms is None else np.asarray(uniforms, dtype=np.float64)[:tail_idx.size]
        keep[tail_idx] = u < pi[tail_idx]
    return keep, pi, certainty


def hajek_log_offsets(pi) -> np.ndarray:
    """``evict.py:174-187``: ``-log(pi)``; every ``pi`` must be > 0."""
    pi = np.asarray(pi, dtype=np.float64)
    if np.any(pi <= 0):
        raise ValueError("inclusion probabilities must be > 0")
    return -np.log(pi)


def block_retention(keep, seq_len: int, block_size: int) -> int:
    """``reclaim.py:46-55``: blocks with at least one kept token."""
    keep = np.asarray(keep, dtype=bool)
    nb = -(-seq_len // block_size)
    return int(sum(bool(keep[b * block_size:min(seq_len, (b + 1) * block_size)].any()) for b in range(nb)))
