"""CPU oracle for block-granular attention mass — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline / reference legs of
``bench.py`` may import it.  The CUDA path never falls back to it.

It is a numpy restatement of the reference's streaming algorithm
(kv-block-mass ``src/kvblockmass/reference.py:35-126``):

* GQA by repeat_interleave semantics: q-head ``h`` reads kv-head ``h // G``
  (``reference.py:23-31``; ``H_q % H_kv != 0`` raises ``ValueError`` with the
  reference's message, ``reference.py:29-30``);
* keep matrix = ``tril`` if causal, ``&`` the mask (``reference.py:83-87``),
  built here per query chunk instead of once as an ``[N, N]`` matrix so that
  long sequences fit in memory;
* query chunks of ``query_chunk`` rows with the causal key bound
  ``n_lim = stop`` (the chunk's LAST row + 1) when ``causal and causal_skip``
  (``reference.py:96-103``);
* ``scores = (q @ k^T) * scale`` in the accumulation dtype (fp64 iff the
  input is fp64, else fp32; ``reference.py:77``, ``:108-111``);
* masked entries -> -inf, softmax over keys, fully-masked rows -> 0
  (``reference.py:113-119``);
* column sums pooled into ``ceil(N / block_size)`` buckets
  (``reference.py:121-124``).

Extensions beyond the reference's mask shapes (per-batch masks and a query
row mask) are defined by linearity over the batch: the result equals the
sum over ``b`` of the reference run on batch ``b`` alone with that batch's
mask, and a row with ``query_mask`` False behaves like a pair-mask row that
keeps nothing.

Ragged batches (sequence ``b`` has its own length ``L_b <= N``) are defined
the same way, by linearity over the batch: sequence ``b`` contributes the
reference run on its first ``L_b`` positions alone (``block_mass_ragged``).

A paged key cache (``[num_pages, page_size, H_kv, D]`` plus a block table
``[B, max_pages]`` of page ids, the layout of the paged KV managers that
consume block mass) is another extension; it is defined by the dense keys it
names (``dense_keys_from_pages``), on which the reference algorithm runs.

The restatement is pinned against outputs of the reference itself, stored
under ``tests/golden/`` by ``tests/golden/gen_golden.py``.
"""

from __future__ import annotations

import math
from concurrent.futures import ThreadPoolExecutor

import numpy as np

__all__ = ["block_mass_stream", "normalize_masks", "num_blocks", "dense_keys_from_pages", "block_mass_ragged",
           "block_mass_segment_lse"]


def num_blocks(n: int, block_size: int) -> int:
    """Bucket count ``ceil(N / block_size)`` (``reference.py:89``)."""
    return (n + block_size - 1) // block_size


def _as_bool(a):
    if a is None:
        return None
    a = np.asarray(a)
    return a.astype(bool, copy=False)


def normalize_masks(attn_mask, query_mask, B: int, N: int):
    """Split the supported mask shapes into (key, pair, query) masks.

    Returns ``(key_mask [Bk, N] | None, pair_mask [Bp, N, N] | None,
    query_mask [Bq, N] | None)`` with leading batch extent 1 or ``B``.
    ``attn_mask`` shapes: ``[N]`` (key/column mask, ``reference.py:86-87``
    broadcasting), ``[N, N]`` (pair mask), ``[B, 1, N]`` (per-batch key mask),
    ``[B, N, N]`` (per-batch pair mask).  ``query_mask``: ``[N]`` or ``[B, N]``.
    """
    key = pair = None
    m = _as_bool(attn_mask)
    if m is not None:
        if m.ndim == 1:
            if m.shape[0] != N:
                raise ValueError(f"attn_mask of shape {m.shape} does not match N={N}")
            key = m.reshape(1, N)
        elif m.ndim == 2:
            if m.shape != (N, N):
                raise ValueError(f"attn_mask of shape {m.shape} does not match [N, N] with N={N}")
            pair = m.reshape(1, N, N)
        elif m.ndim == 3:
            if m.shape[0] not in (1, B) or m.shape[2] != N or m.shape[1] not in (1, N):
                raise ValueError(f"attn_mask of shape {m.shape} is not [B|1, 1|N, N]")
            if m.shape[1] == 1:
                key = m[:, 0, :]
            else:
                pair = m
        else:
            raise ValueError(f"attn_mask must be 1-D, 2-D or 3-D, got {m.ndim}-D")
    qm = _as_bool(query_mask)
    if qm is not None:
        if qm.ndim == 1:
            qm = qm.reshape(1, -1)
        if qm.ndim != 2 or qm.shape[0] not in (1, B) or qm.shape[1] != N:
            raise ValueError(f"query_mask of shape {qm.shape} is not [N] or [B, N]")
    return key, pair, qm


def _keep_rows(b, start, stop, n_lim, causal, key, pair, qm):
    """``keep[start:stop, :n_lim]`` for batch ``b`` (``reference.py:83-87``, ``:101``)."""
    rows = np.arange(start, stop)
    cols = np.arange(n_lim)
    if causal:
        keep = rows[:, None] >= cols[None, :]
    else:
        keep = np.ones((stop - start, n_lim), dtype=bool)
    if key is not None:
        keep = keep & key[b if key.shape[0] > 1 else 0, :n_lim][None, :]
    if pair is not None:
        keep = keep & pair[b if pair.shape[0] > 1 else 0, start:stop, :n_lim]
    if qm is not None:
        keep = keep & qm[b if qm.shape[0] > 1 else 0, start:stop][:, None]
    return keep


def _chunk_contrib(qc, kfull, keep, scale, acc):
    """Softmax weights of one query chunk summed over heads and rows.

    ``qc``: [H, C, D]; ``kfull``: [H, n_lim, D]; ``keep``: [C, n_lim].
    Follows ``reference.py:108-124`` for a single batch entry.
    """
    scores = np.matmul(qc.astype(acc, copy=False), np.swapaxes(kfull.astype(acc, copy=False), -1, -2))
    scores *= acc(scale)
    scores = np.where(keep[None], scores, -np.inf)
    row_has_any = keep.any(axis=-1)
    with np.errstate(invalid="ignore", over="ignore"):
        m = scores.max(axis=-1, keepdims=True)
        e = np.exp(scores - m)
        w = e / e.sum(axis=-1, keepdims=True)
    w = np.where(row_has_any[None, :, None], w, acc(0))
    w = np.nan_to_num(w, nan=0.0)
    return w.sum(axis=(0, 1))  # [n_lim]


def block_mass_stream(
    q,
    k,
    attn_mask=None,
    causal: bool = False,
    block_size: int = 64,
    scale: float | None = None,
    query_chunk: int = 256,
    causal_skip: bool = True,
    query_mask=None,
    heads: slice | None = None,
    rows: tuple[int, int] | None = None,
    threads: int = 1,
    split_rows: bool = False,
):
    """Block mass ``[ceil(N / block_size)]`` of ``q [B,H_q,N,D]``, ``k [B,H_kv,N,D]``.

    Arguments mirror ``block_mass_reference`` (``reference.py:35-45``);
    ``query_mask`` is the additive row-mask extension (see module docstring).
    ``heads`` (a slice of q-heads) and ``rows`` (a ``[start, stop)`` range of
    query rows, aligned to ``query_chunk``) restrict the sum to a sample of the
    workload; the CPU baseline uses them to time a bounded part of a large
    shape.  ``threads`` > 1 splits (batch, head) work over a thread pool
    (numpy releases the GIL inside its kernels); ``split_rows`` also splits
    each (batch, head) into its query chunks.

    The result dtype is float64 for float64 inputs and float32 otherwise
    (``reference.py:77``).
    """
    q = np.asarray(q)
    k = np.asarray(k)
    if q.ndim != 4 or k.ndim != 4:
        raise ValueError("q and k must be 4-D [B, H, N, D]")
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    if Hq % Hkv != 0:
        raise ValueError(f"GQA requires H_q % H_kv == 0, got H_q={Hq}, H_kv={Hkv}")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    G = Hq // Hkv
    if scale is None:
        scale = 1.0 / D ** 0.5
    acc = np.float64 if q.dtype == np.float64 else np.float32
    key, pair, qm = normalize_masks(attn_mask, query_mask, B, N)

    nb = num_blocks(N, block_size)
    col_block = np.arange(N) // block_size
    hsel = range(Hq)[heads] if heads is not None else range(Hq)
    r0, r1 = rows if rows is not None else (0, N)

    def one(item):
        b, h, lo, hi = item
        part = np.zeros(nb, dtype=np.float64 if acc is np.float64 else np.float32)
        for start in range(lo, hi, query_chunk):
            stop = min(start + query_chunk, N)
            n_lim = stop if (causal and causal_skip) else N
            keep = _keep_rows(b, start, stop, n_lim, causal, key, pair, qm)
            c = _chunk_contrib(q[b, h:h + 1, start:stop], k[b, (h // G):(h // G) + 1, :n_lim],
                               keep, scale, acc)
            part += np.bincount(col_block[:n_lim], weights=c, minlength=nb).astype(part.dtype)
        return part

    if split_rows:
        work = [(b, h, s, min(s + query_chunk, r1)) for b in range(B) for h in hsel
                for s in range(r0, r1, query_chunk)]
    else:
        work = [(b, h, r0, r1) for b in range(B) for h in hsel]
    mass = np.zeros(nb, dtype=np.float64 if acc is np.float64 else np.float32)
    if threads > 1 and len(work) > 1:
        with ThreadPoolExecutor(max_workers=threads) as ex:
            for part in ex.map(one, work):
                mass += part
    else:
        for bh in work:
            mass += one(bh)
    return mass


def pairs_count(B: int, Hq: int, N: int, causal: bool) -> int:
    """Algorithmic QK pairs of the full problem: causal triangle or N^2 per (b, h)."""
    per = N * (N + 1) // 2 if causal else N * N
    return B * Hq * per


def sample_pairs(Hq_sel: int, B_sel: int, N: int, rows: tuple[int, int], causal: bool) -> int:
    """QK pairs inside a ``rows`` sample over ``B_sel * Hq_sel`` (b, h) pairs."""
    r0, r1 = rows
    if causal:
        per = (r1 * (r1 + 1) - r0 * (r0 + 1)) // 2
    else:
        per = (r1 - r0) * N
    return B_sel * Hq_sel * per


def dense_block_mass(q, k, attn_mask=None, causal=False, block_size=64, scale=None):
    """Materialised ``[B, H, N, N]`` oracle for small shapes.

    Restates the reference's test oracle ``tests/naive.py:10-59``: full
    softmax with masked entries at -inf, NaN rows -> 0, then a zero-padded
    reshape-pool into buckets.  ``[N]`` masks broadcast over query rows here
    (the reference's ``naive.py:40`` reshape accepts only ``[N, N]``).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    if Hq % Hkv != 0:
        raise ValueError(f"GQA requires H_q % H_kv == 0, got H_q={Hq}, H_kv={Hkv}")
    if scale is None:
        scale = 1.0 / D ** 0.5
    kf = np.repeat(k, Hq // Hkv, axis=1)
    s = np.matmul(q, np.swapaxes(kf, -1, -2)) * scale
    keep = np.tril(np.ones((N, N), dtype=bool)) if causal else np.ones((N, N), dtype=bool)
    if attn_mask is not None:
        m = np.asarray(attn_mask).astype(bool)
        keep = keep & (m[None, :] if m.ndim == 1 else m)
    s = np.where(keep, s, -np.inf)
    with np.errstate(invalid="ignore"):
        m = s.max(axis=-1, keepdims=True)
        e = np.exp(s - m)
        w = e / e.sum(axis=-1, keepdims=True)
    w = np.nan_to_num(w, nan=0.0)
    nb = num_blocks(N, block_size)
    pad = nb * block_size - N
    if pad:
        w = np.pad(w, [(0, 0)] * 3 + [(0, pad)])
    return w.reshape(B, Hq, N, nb, block_size).sum(axis=-1).sum(axis=(0, 1, 2))


def causal_skip_extents(N: int, query_chunk: int, causal: bool, causal_skip: bool) -> list[int]:
    """Key extent handed to the score GEMM per query chunk (``reference.py:100``).

    The reference's engagement test records exactly this list
    (``tests/test_reference.py:189-215``).
    """
    out = []
    for start in range(0, N, query_chunk):
        stop = min(start + query_chunk, N)
        out.append(stop if (causal and causal_skip) else N)
    return out


if __name__ == "__main__":  # pragma: no cover - manual smoke
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 4, 100, 16))
    k = rng.standard_normal((1, 2, 100, 16))
    a = block_mass_stream(q, k, causal=True, block_size=32)
    d = dense_block_mass(q, k, causal=True, block_size=32)
    print(a, d, float(np.abs(a - d).max()), math.isclose(a.sum(), 400.0))


def dense_keys_from_pages(k_cache, block_table, n: int):
    """Dense ``k [B, H_kv, N, D]`` named by a paged cache.

    Key ``c`` of sequence ``b`` is slot ``c % P`` of page
    ``block_table[b, c // P]`` of ``k_cache [num_pages, P, H_kv, D]``.  The
    reference takes dense keys only; this defines the paged input by them.
    """
    k_cache = np.asarray(k_cache)
    table = np.asarray(block_table).astype(np.int64)
    p = k_cache.shape[1]
    c = np.arange(n)
    pages = table[:, c // p]                     # [B, N]
    rows = k_cache[pages, (c % p)[None, :]]      # [B, N, H_kv, D]
    return np.ascontiguousarray(rows.transpose(0, 2, 1, 3))


def _batch_slice(m, b, length, pair_ok=True):
    """Batch ``b``'s part of a mask of the supported shapes, cut to ``length`` positions."""
    if m is None:
        return None
    m = np.asarray(m)
    if m.ndim == 1:
        return m[:length]
    if m.ndim == 2:
        if m.shape[0] == m.shape[1] and pair_ok and m.shape[0] != 1:
            return m[:length, :length]          # [N, N] pair mask shared by the batch
        return m[b if m.shape[0] > 1 else 0, :length]   # [B, N] row mask
    mb = m[b if m.shape[0] > 1 else 0]
    if mb.shape[0] == 1:
        return mb[None, :, :length]             # [1, 1, N] key mask of batch b
    return mb[:length, :length]                 # [N, N] pair mask of batch b


def block_mass_ragged(q, k, lens, attn_mask=None, causal=False, block_size=64, scale=None, query_mask=None,
                      per_sequence=False):
    """Block mass of a ragged batch: ``q [B,H_q,N,D]``, ``k [B,H_kv,N,D]``,
    sequence ``b`` being its first ``lens[b] <= N`` positions.

    Each sequence is the reference's computation on ``q[b:b+1, :, :L]``,
    ``k[b:b+1, :, :L]`` with its slice of the masks (``reference.py:35-126``);
    its ``ceil(L / block_size)`` buckets land in the first buckets of the
    ``ceil(N / block_size)``-long output.  Returns the sum over sequences, or
    ``[B, num_blocks]`` with ``per_sequence``.  Positions past ``L`` are never
    read, so they may hold anything.
    """
    q = np.asarray(q)
    k = np.asarray(k)
    B, _, N, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    nb = num_blocks(N, block_size)
    acc = np.float64 if q.dtype == np.float64 else np.float32
    out = np.zeros((B, nb), dtype=acc)
    for b in range(B):
        L = int(min(max(int(lens[b]), 0), N))
        if L == 0:
            continue
        m = block_mass_stream(q[b:b + 1, :, :L], k[b:b + 1, :, :L],
                              attn_mask=_batch_slice(attn_mask, b, L),
                              query_mask=_batch_slice(query_mask, b, L, pair_ok=False),
                              causal=causal, block_size=block_size, scale=scale)
        out[b, :m.shape[0]] = m
    return out if per_sequence else out.sum(axis=0, dtype=np.float64).astype(acc)


def block_mass_segment_lse(q, k, attn_mask=None, causal=False, block_size=64, scale=None, query_mask=None,
                           seg=64, tile=128):
    """The mass from per-row segment log-sums: the identity the library's
    one-pass method computes, checked here against the reference's outputs.

    For query row ``i`` the reference's softmax summed over the keys of bucket
    ``j`` (``reference.py:113-124``) is ``2^(L_ij - lse2_i)``, where
    ``L_ij = log2 sum_{c in j} 2^(t_ic)`` over the kept keys (``t`` the scores
    times ``log2 e``) and ``lse2_i`` the row's log2-sum-exp2 over all kept
    keys.  This walks each row's keys in tiles of ``tile`` keys, as the kernel
    does: it keeps a running max ``m`` and, for every piece of ``seg`` keys
    (cut at bucket edges too), the sum of ``2^(t - m)`` rescaled when ``m``
    grows, and records ``L = m + log2(sum)`` when the piece ends.  The mass is
    ``sum_i sum_pieces 2^(L - lse2_i)``.  Float64; small shapes only.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    if Hq % Hkv != 0:
        raise ValueError(f"GQA requires H_q % H_kv == 0, got H_q={Hq}, H_kv={Hkv}")
    G = Hq // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    key, pair, qm = normalize_masks(attn_mask, query_mask, B, N)
    nb = num_blocks(N, block_size)
    out = np.zeros(nb, dtype=np.float64)
    log2e = 1.0 / math.log(2.0)
    # piece boundaries: every multiple of seg and of block_size
    edges = sorted(set(range(0, N, seg)) | set(range(0, N, block_size)) | {N})
    for b in range(B):
        keep = _keep_rows(b, 0, N, N, causal, key, pair, qm)
        for h in range(Hq):
            t = (q[b, h] @ k[b, h // G].T) * (scale * log2e)
            t = np.where(keep, t, -np.inf)
            for i in range(N):
                m, l = -np.inf, 0.0
                pieces = []  # (bucket, L)
                for c0 in range(0, N, tile):
                    row = t[i, c0:c0 + tile]
                    tmax = row.max()
                    if tmax > m:  # rescale only when the running max grows
                        if pieces:
                            pass  # recorded pieces are absolute (m + log2 sum): nothing to rescale
                        l = l * (2.0 ** (m - tmax)) if np.isfinite(m) else 0.0
                        m = tmax
                    for p0, p1 in zip(edges[:-1], edges[1:]):
                        if p0 < c0 or p1 > c0 + tile:
                            continue
                        sub = row[p0 - c0:p1 - c0]
                        ssum = float(np.exp2(sub - m).sum()) if np.isfinite(m) else 0.0
                        l += ssum
                        with np.errstate(divide="ignore"):
                            pieces.append((p0 // block_size, m + math.log2(ssum) if ssum > 0 else -np.inf))
                if not np.isfinite(m) or l == 0.0:
                    continue  # a row that keeps no key contributes 0 (reference.py:117-119)
                lse2 = m + math.log2(l)
                for j, L in pieces:
                    if np.isfinite(L):
                        out[j] += 2.0 ** (L - lse2)
    return out
