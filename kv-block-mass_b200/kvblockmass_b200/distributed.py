"""Multi-GPU block mass: shard (batch, kv-head) units over ranks, reduce once.

Mass is a sum over independent units u = b * H_kv + g (q-heads
[g*G, (g+1)*G) with kv-head g of batch entry b), so a problem splits across
ranks with no exchange inside the computation.  Each rank keeps only its own
units' q/k in HBM, runs the kernels on them, and one collective sums the
``num_blocks``-long mass vectors:

* ``reduce`` (default): one NCCL reduce to ``dst`` over NVLink;
* ``deterministic=True``: all-gather of the vectors, then every rank adds
  them in rank order in float64, so the bits do not depend on NCCL's choice
  of algorithm.

The reference has no multi-GPU path (kv-block-mass README.md:138-140); the
split follows from the sum over (b, h) in ``reference.py:121-124``.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

__all__ = ["partition_units", "unit_segments", "shard_inputs", "block_mass_sharded"]


def partition_units(n_units: int, world: int) -> list[tuple[int, int]]:
    """Contiguous, balanced ``[begin, end)`` unit ranges, one per rank (some may be empty)."""
    if n_units < 0 or world < 1:
        raise ValueError("n_units >= 0 and world >= 1 required")
    base, extra = divmod(n_units, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((start, start + n))
        start += n
    return out


def unit_segments(begin: int, end: int, Hkv: int) -> list[tuple[int, int, int]]:
    """Split units ``[begin, end)`` into per-batch ``(b, g0, g1)`` kv-head ranges."""
    segs = []
    u = begin
    while u < end:
        b, g0 = divmod(u, Hkv)
        g1 = min(Hkv, g0 + (end - u))
        segs.append((b, g0, g1))
        u += g1 - g0
    return segs


def _slice_mask_batch(m, b):
    if m is None:
        return None
    if m.dim() == 3:           # [B|1, 1|N, N]
        return m[b:b + 1] if m.shape[0] > 1 else m
    return m                   # [N] or [N, N]: shared by every batch entry


def _slice_query_mask(qm, b):
    if qm is None:
        return None
    if qm.dim() == 2 and qm.shape[0] > 1:
        return qm[b:b + 1]
    return qm


def shard_inputs(q, k, rank: int, world: int, attn_mask=None, query_mask=None):
    """This rank's shards of full ``q``/``k``: a list of per-segment dicts.

    Each segment is a contiguous kv-head range of one batch entry with the
    matching q-heads (views, no copies), plus that batch entry's masks.  Move
    them to the rank's device (``.to(dev)``) so each GPU holds only its part.
    """
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    if Hq % Hkv != 0:
        raise ValueError(f"GQA requires H_q % H_kv == 0, got H_q={Hq}, H_kv={Hkv}")
    G = Hq // Hkv
    begin, end = partition_units(B * Hkv, world)[rank]
    out = []
    for b, g0, g1 in unit_segments(begin, end, Hkv):
        out.append({
            "q": q[b:b + 1, g0 * G:g1 * G],
            "k": k[b:b + 1, g0:g1],
            "attn_mask": _slice_mask_batch(attn_mask, b),
            "query_mask": _slice_query_mask(query_mask, b),
        })
    return out


def block_mass_sharded(shards, causal=False, block_size=64, scale=None, causal_skip=True, *,
                       num_blocks: int, group=None, dst: int = 0, deterministic: bool = False,
                       all_ranks: bool = False, local_fn: Callable | None = None,
                       device: torch.device | None = None):
    """Global block mass from this rank's ``shards`` (see ``shard_inputs``).

    Every rank must call this with the same ``num_blocks`` and options.  The
    result is complete on ``dst`` (on every rank with ``all_ranks`` or
    ``deterministic``); other ranks get their local partial sum.  ``local_fn``
    replaces the per-shard kernel call (tests use it to run the host logic
    with the CPU oracle over ``gloo``); by default it is ``block_mass_b200``.
    """
    if local_fn is None:
        from .ops import block_mass_b200 as local_fn  # noqa: N813
    acc = None
    out_dtype = torch.float32
    for sh in shards:
        kw = {k: v for k, v in sh.items() if k not in ("q", "k") and v is not None}
        m = local_fn(sh["q"], sh["k"], causal=causal, block_size=block_size, scale=scale,
                     causal_skip=causal_skip, **kw)
        if m.dtype == torch.float64:  # fp64 inputs give an fp64 mass (reference.py:77)
            out_dtype = torch.float64
        acc = m.to(torch.float64) if acc is None else acc + m.to(torch.float64)
    if acc is None:  # a rank without units still takes part in the collective
        if device is None and dist.get_backend(group) == "nccl":
            device = torch.device("cuda", torch.cuda.current_device())  # NCCL needs a CUDA tensor
        acc = torch.zeros(num_blocks, dtype=torch.float64, device=device)
    if acc.numel() != num_blocks:
        raise ValueError(f"local mass has {acc.numel()} buckets, expected {num_blocks}")
    # The result dtype must agree across ranks; a rank without units cannot
    # see the inputs' dtype, so it follows the others'.
    flag = torch.tensor([1.0 if out_dtype == torch.float64 else 0.0], dtype=torch.float64, device=acc.device)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
    out_dtype = torch.float64 if float(flag.item()) > 0 else torch.float32
    if deterministic:
        world = dist.get_world_size(group)
        parts = [torch.empty_like(acc) for _ in range(world)]
        dist.all_gather(parts, acc, group=group)
        total = torch.zeros_like(acc)
        for p in parts:          # rank order: bit-stable for a fixed world size
            total += p
        return total.to(out_dtype)
    red = acc.to(out_dtype)
    if all_ranks:
        dist.all_reduce(red, op=dist.ReduceOp.SUM, group=group)
    else:
        dist.reduce(red, dst=dst, op=dist.ReduceOp.SUM, group=group)
    return red
