"""Seeded synthetic workloads for block-mass parity tests and benchmarks.

The reference measures on synthetic Gaussian q/k only (kv-block-mass
``bench/bench_block_mass.py:80-82``: a CPU ``torch.Generator`` seeded per
shape, ``q`` drawn before ``k``).  The five shapes below follow that
protocol.  Each draws, from one CPU generator seeded with ``seed``:

1. ``q = randn(B, H_q, N, D)`` then ``k = randn(B, H_kv, N, D)`` in fp32;
2. the shape's extra draws, in this order: per-q-head scales
   ``U(0.5, 2.0)`` (``rand(H_q) * 1.5 + 0.5``), the key mask
   (``rand(N) >= 0.1``), the attention-sink key rows
   (``randperm(N)[:N // 100]``, scaled by 8 in every kv head);
3. a cast to the shape's dtype.

The oracle is fed exactly those values upcast to fp32.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

__all__ = ["Workload", "WORKLOADS", "make_inputs", "make_unit_inputs", "pairs"]


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    Hq: int
    Hkv: int
    D: int
    N: int
    block_size: int
    causal: bool
    dtype: torch.dtype
    seed: int
    head_scale: bool = False       # per-q-head U(0.5, 2) multiplier on q
    key_mask_frac: float = 0.0     # i.i.d. fraction of masked key columns
    dead_tail_rows: int = 0        # last rows of the last batch entry keep no key
    sink_frac: float = 0.0         # fraction of key rows scaled by sink_gain
    sink_gain: float = 8.0
    notes: str = field(default="", compare=False)

    @property
    def num_blocks(self) -> int:
        return (self.N + self.block_size - 1) // self.block_size

    @property
    def G(self) -> int:
        return self.Hq // self.Hkv

    @property
    def units(self) -> int:
        """Independent (batch, kv-head group) units the problem shards into."""
        return self.B * self.Hkv


WORKLOADS = {
    "cpu_ref_n2048": Workload(
        "cpu_ref_n2048", B=1, Hq=8, Hkv=2, D=64, N=2048, block_size=64, causal=True,
        dtype=torch.float32, seed=0,
        notes="the reference's own benchmark shape (bench/bench_block_mass.py:29) at N=2048"),
    "gqa_n8192_fp32": Workload(
        "gqa_n8192_fp32", B=1, Hq=8, Hkv=2, D=64, N=8192, block_size=64, causal=True,
        dtype=torch.float32, seed=1),
    "llama3_8b_n32k": Workload(
        "llama3_8b_n32k", B=1, Hq=32, Hkv=8, D=128, N=32768, block_size=64, causal=True,
        dtype=torch.bfloat16, seed=2, head_scale=True,
        notes="Llama-3-8B attention shape; per-head scale U(0.5,2) varies softmax sharpness"),
    "batched_masked_n16k": Workload(
        "batched_masked_n16k", B=4, Hq=32, Hkv=8, D=128, N=16384, block_size=128, causal=False,
        dtype=torch.bfloat16, seed=3, key_mask_frac=0.1, dead_tail_rows=64,
        notes="10% i.i.d. masked key columns; last 64 query rows of batch 3 keep nothing"),
    "llama3_70b_n128k": Workload(
        "llama3_70b_n128k", B=1, Hq=64, Hkv=8, D=128, N=131072, block_size=256, causal=True,
        dtype=torch.bfloat16, seed=4, sink_frac=0.01,
        notes="Llama-3-70B long context; 1% of key rows x8 (attention sinks)"),
}


def pairs(w: Workload) -> int:
    """Algorithmic QK pairs: ``B*H_q*N(N+1)/2`` causal, ``B*H_q*N^2`` otherwise."""
    per = w.N * (w.N + 1) // 2 if w.causal else w.N * w.N
    return w.B * w.Hq * per


def make_inputs(w: Workload, N: int | None = None, device: str | torch.device = "cpu"):
    """Draw ``(q, k, key_mask, query_mask)`` for ``w`` (``N`` overrides the length).

    ``key_mask`` is ``[N]`` bool or None; ``query_mask`` is ``[B, N]`` bool or
    None (False rows keep no key).  q/k come back in ``w.dtype`` on ``device``.
    """
    n = w.N if N is None else N
    g = torch.Generator().manual_seed(w.seed)
    q = torch.randn(w.B, w.Hq, n, w.D, generator=g, dtype=torch.float32)
    k = torch.randn(w.B, w.Hkv, n, w.D, generator=g, dtype=torch.float32)
    key_mask = query_mask = None
    if w.head_scale:
        s = torch.rand(w.Hq, generator=g, dtype=torch.float32) * 1.5 + 0.5
        q.mul_(s.view(1, w.Hq, 1, 1))
    if w.key_mask_frac > 0:
        key_mask = torch.rand(n, generator=g, dtype=torch.float32) >= w.key_mask_frac
    if w.dead_tail_rows > 0:
        query_mask = torch.ones(w.B, n, dtype=torch.bool)
        query_mask[w.B - 1, max(0, n - w.dead_tail_rows):] = False
    if w.sink_frac > 0:
        rows = torch.randperm(n, generator=g)[: max(1, int(n * w.sink_frac))]
        k[:, :, rows, :] *= w.sink_gain
    q = q.to(w.dtype)
    k = k.to(w.dtype)
    if device != "cpu":
        q = q.to(device)
        k = k.to(device)
        key_mask = key_mask.to(device) if key_mask is not None else None
        query_mask = query_mask.to(device) if query_mask is not None else None
    return q, k, key_mask, query_mask


def make_unit_inputs(w: Workload, unit_begin: int, unit_end: int, device="cpu", N: int | None = None):
    """Inputs of the (batch, kv-head) units ``[unit_begin, unit_end)`` only.

    Per-unit protocol for shards of large shapes, so that a rank draws just
    the q/k it owns (on its own device): unit ``u`` draws its ``G`` q-heads and
    then its kv-head from a generator seeded ``seed * 1_000_003 + u``.  The
    per-q-head scales and the sink rows are drawn from a generator seeded
    ``seed`` and shared by every unit.  Same shapes and distributions as
    ``make_inputs``; different values.  The units must lie in one batch
    entry.  Returns ``(q [1, (u1-u0)*G, N, D], k [1, u1-u0, N, D])`` in
    ``w.dtype``.
    """
    n = w.N if N is None else N
    G = w.G
    if unit_begin // w.Hkv != (unit_end - 1) // w.Hkv:
        raise ValueError("units must belong to one batch entry")
    dev = torch.device(device)
    shared = torch.Generator().manual_seed(w.seed)
    head_scale = (torch.rand(w.Hq, generator=shared) * 1.5 + 0.5) if w.head_scale else None
    sink_rows = None
    if w.sink_frac > 0:
        sink_rows = torch.randperm(n, generator=shared)[: max(1, int(n * w.sink_frac))].to(dev)
    qs, ks = [], []
    for u in range(unit_begin, unit_end):
        g = torch.Generator(device=dev).manual_seed(w.seed * 1_000_003 + u)
        q = torch.randn(1, G, n, w.D, generator=g, device=dev, dtype=torch.float32)
        k = torch.randn(1, 1, n, w.D, generator=g, device=dev, dtype=torch.float32)
        if head_scale is not None:
            h0 = (u % w.Hkv) * G
            q.mul_(head_scale[h0:h0 + G].to(dev).view(1, G, 1, 1))
        if sink_rows is not None:
            k[:, :, sink_rows, :] *= w.sink_gain
        qs.append(q.to(w.dtype))
        ks.append(k.to(w.dtype))
    return torch.cat(qs, dim=1), torch.cat(ks, dim=1)
