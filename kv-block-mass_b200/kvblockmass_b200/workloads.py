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

import base64
import json
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from pathlib import Path

import torch

__all__ = ["Workload", "WORKLOADS", "make_inputs", "make_unit_inputs", "unit_states", "compute_unit_states",
           "pairs"]

_STATES_FILE = Path(__file__).resolve().parent / "workload_states.json"


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


def _unit_piece_ok(w: Workload, n: int) -> bool:
    """Whether per-unit draws can restart the stream at unit boundaries.

    torch's CPU normal sampler fills a tensor in blocks of 16 values (a tail
    that is not a whole block is redrawn), so a draw split into pieces equals
    the draw of the whole only if every piece is a whole number of blocks.
    """
    return (w.G * n * w.D) % 16 == 0 and (n * w.D) % 16 == 0


def _encode_state(st: torch.Tensor) -> str:
    return base64.b64encode(st.numpy().tobytes()).decode("ascii")


def _decode_state(s: str) -> torch.Tensor:
    return torch.frombuffer(bytearray(base64.b64decode(s)), dtype=torch.uint8).clone()


def compute_unit_states(w: Workload, N: int | None = None) -> dict:
    """Generator states of ``make_inputs``' stream at every unit boundary.

    ``q`` holds the state before the q-heads of each unit u = b * H_kv + g
    (heads ``[g*G, (g+1)*G)`` of batch ``b``: contiguous in the draw order),
    ``k`` the state before each unit's kv-head, and ``extra`` the state after
    ``k``, where the per-head scales, the key mask and the sink rows are
    drawn.  Costs one sequential draw of the whole stream.
    """
    n = w.N if N is None else N
    g = torch.Generator().manual_seed(w.seed)
    qs, ks = [], []
    for _ in range(w.units):
        qs.append(g.get_state().clone())
        torch.randn(1, w.G, n, w.D, generator=g, dtype=torch.float32)
    for _ in range(w.units):
        ks.append(g.get_state().clone())
        torch.randn(1, 1, n, w.D, generator=g, dtype=torch.float32)
    return {"q": qs, "k": ks, "extra": g.get_state().clone()}


def _stored_states(w: Workload, n: int):
    p = _STATES_FILE
    if not p.exists():
        return None
    rec = json.loads(p.read_text()).get(w.name)
    if rec is None or rec["N"] != n or rec["seed"] != w.seed or rec["torch"] != torch.__version__.split("+")[0]:
        return None
    return {"q": [_decode_state(x) for x in rec["q"]], "k": [_decode_state(x) for x in rec["k"]],
            "extra": _decode_state(rec["extra"])}


def unit_states(w: Workload, N: int | None = None) -> dict:
    """The stream's states at the unit boundaries: stored ones when this file's
    companion ``workload_states.json`` has them (the Llama-3-70B N=131072 shape,
    whose full draw takes a minute of CPU), else computed."""
    n = w.N if N is None else N
    st = _stored_states(w, n)
    return st if st is not None else compute_unit_states(w, n)


def write_unit_states(names) -> None:
    """Record ``unit_states`` of the named workloads (full length) in ``workload_states.json``."""
    out = json.loads(_STATES_FILE.read_text()) if _STATES_FILE.exists() else {}
    for name in names:
        w = WORKLOADS[name]
        st = compute_unit_states(w)
        out[name] = {"N": w.N, "seed": w.seed, "torch": torch.__version__.split("+")[0],
                     "q": [_encode_state(x) for x in st["q"]], "k": [_encode_state(x) for x in st["k"]],
                     "extra": _encode_state(st["extra"])}
    _STATES_FILE.write_text(json.dumps(out, indent=0))


def _draw(state: torch.Tensor, shape) -> torch.Tensor:
    g = torch.Generator()
    g.set_state(state)
    return torch.randn(*shape, generator=g, dtype=torch.float32)


def make_unit_inputs(w: Workload, unit_begin: int, unit_end: int, device="cpu", N: int | None = None,
                     threads: int | None = None):
    """q/k of the (batch, kv-head) units ``[unit_begin, unit_end)`` only.

    The values are exactly ``make_inputs(w)``'s slices ``q[b, g0*G:g1*G]`` and
    ``k[b, g0:g1]``: each unit's q-heads and kv-head are redrawn from the
    generator state at its place in the stream (``unit_states``), units in
    parallel threads, so a rank of a multi-GPU run draws only what it owns.
    The per-head scales and sink rows come from the state after ``k``, as in
    ``make_inputs``.  The units must lie in one batch entry.  Returns
    ``(q [1, (u1-u0)*G, N, D], k [1, u1-u0, N, D])`` in ``w.dtype`` on ``device``.
    """
    n = w.N if N is None else N
    G = w.G
    if not (0 <= unit_begin < unit_end <= w.units):
        raise ValueError(f"unit range [{unit_begin}, {unit_end}) outside [0, {w.units})")
    if unit_begin // w.Hkv != (unit_end - 1) // w.Hkv:
        raise ValueError("units must belong to one batch entry")
    b, g0 = divmod(unit_begin, w.Hkv)
    g1 = g0 + (unit_end - unit_begin)
    if not _unit_piece_ok(w, n):  # the stream cannot restart at unit boundaries: draw it all
        q, k, _, _ = make_inputs(w, N=n)
        q, k = q[b:b + 1, g0 * G:g1 * G].contiguous(), k[b:b + 1, g0:g1].contiguous()
        return q.to(device), k.to(device)
    st = unit_states(w, n)
    gx = torch.Generator()
    gx.set_state(st["extra"])
    head_scale = (torch.rand(w.Hq, generator=gx, dtype=torch.float32) * 1.5 + 0.5) if w.head_scale else None
    if w.key_mask_frac > 0:
        torch.rand(n, generator=gx, dtype=torch.float32)  # the key mask: drawn before the sink rows
    sink_rows = None
    if w.sink_frac > 0:
        sink_rows = torch.randperm(n, generator=gx)[: max(1, int(n * w.sink_frac))]

    def one(u):
        q = _draw(st["q"][u], (1, G, n, w.D))
        k = _draw(st["k"][u], (1, 1, n, w.D))
        if head_scale is not None:
            h0 = (u % w.Hkv) * G
            q.mul_(head_scale[h0:h0 + G].view(1, G, 1, 1))
        if sink_rows is not None:
            k[:, :, sink_rows, :] *= w.sink_gain
        return q.to(w.dtype), k.to(w.dtype)

    units = list(range(unit_begin, unit_end))
    nthr = max(1, min(len(units), threads or (os.cpu_count() or 1)))
    with ThreadPoolExecutor(nthr) as ex:
        parts = list(ex.map(one, units))
    q = torch.cat([p[0] for p in parts], dim=1)
    k = torch.cat([p[1] for p in parts], dim=1)
    return q.to(device), k.to(device)


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description="record the unit-boundary generator states of workloads")
    ap.add_argument("names", nargs="+", choices=sorted(WORKLOADS))
    write_unit_states(ap.parse_args().names)
