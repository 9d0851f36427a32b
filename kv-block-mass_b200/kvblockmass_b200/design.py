"""Device-side consumers of the mass vector: the reference's eviction design
(kv-block-mass ``src/kvblockmass/evict.py``) computed on the GPU, so the mass
never leaves the device.

``design_from_mass`` = ``design_from_scores(expand_block_scores(mass, seq_len,
block_size), ...)`` (``evict.py:64-171``) plus ``hajek_log_offsets``
(``evict.py:174-187``) and the block retention count of ``plan_reclaim``
(``reclaim.py:46-55``), for one sequence (``mass [num_blocks]``) or many
(``mass [rows, num_blocks]``, e.g. ``per_sequence`` block mass), in three
kernel launches (``kvbm_design`` in ``include/kvbm.h``).

Argument errors raise ``ValueError`` with the reference's messages.  A
negative or NaN mass, which the reference rejects, is only seen on the
device: ``DeviceDesign.check()`` raises for it.

Tail draws: ``generator`` (a CPU ``torch.Generator``) draws the reference's
uniforms, ``torch.rand(n, float64, generator)``, on the host; with the same
generator state the design matches the reference's (up to the order among
tied scores at the top slice's edge, where this implementation takes the
lower index, as ``_top_slice``'s docstring states).  ``uniforms`` passes the
draws explicitly; otherwise a Philox stream keyed by ``seed`` runs on the
device (no host work).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

__all__ = ["DeviceDesign", "design_from_mass", "design_workspace_bytes"]


@dataclass
class DeviceDesign:
    """A realized design on the device (rows x seq_len; 1-D for one sequence)."""

    keep: torch.Tensor            # bool
    pi: torch.Tensor              # float64
    certainty: torch.Tensor       # bool
    counts: torch.Tensor          # int64 [rows, 5]: kept, certain, tail, blocks kept, flags
    tail_budget: int
    eps: float
    scores: torch.Tensor | None = None
    log_offsets: torch.Tensor | None = None

    @property
    def tail(self) -> torch.Tensor:
        return ~self.certainty

    def n_expected(self):
        return self.pi.sum(-1)

    def n_kept(self):
        """Kept tokens per row (device tensor; ``int()`` of it synchronises)."""
        c = self.counts[:, 0]
        return c[0] if self.keep.dim() == 1 else c

    def blocks_kept(self):
        c = self.counts[:, 3]
        return c[0] if self.keep.dim() == 1 else c

    def check(self) -> "DeviceDesign":
        """Raise ``ValueError`` as the reference would for a negative / NaN mass (synchronises)."""
        if bool((self.counts[:, 4] != 0).any()):
            raise ValueError("scores must be non-negative")
        return self


def _args(mass, seq_len, block_size, tail_budget, n_sinks, recency, top_slice, eps, uniform_tail):
    if not isinstance(mass, torch.Tensor) or mass.dim() not in (1, 2):
        raise ValueError(f"block mass must be 1-D [num_blocks] or 2-D [rows, num_blocks], got "
                         f"{tuple(mass.shape) if isinstance(mass, torch.Tensor) else type(mass)}")
    if eps <= 0:
        raise ValueError("eps must be > 0 (the design needs a positive floor)")
    if tail_budget < 0:
        raise ValueError("tail_budget must be >= 0")
    nb = mass.shape[-1]
    if nb * block_size < seq_len:
        raise ValueError(f"{nb} blocks of {block_size} cannot cover seq_len={seq_len}")
    if mass.dtype not in (torch.float32, torch.float64):
        mass = mass.float()
    m2 = mass.reshape(-1, nb)
    if m2.stride(-1) != 1:
        m2 = m2.contiguous()
    a = _lib.DesignArgs()
    a.mass = m2.data_ptr()
    a.mass_dtype = _lib.KVBM_F64 if m2.dtype == torch.float64 else _lib.KVBM_F32
    a.rows = m2.shape[0]
    a.mass_row_stride = m2.stride(0)
    a.num_blocks = nb
    a.seq_len = int(seq_len)
    a.block_size = int(block_size)
    a.n_sinks = int(n_sinks)
    a.recency = int(recency)
    a.top_slice = int(top_slice)
    a.tail_budget = int(tail_budget)
    a.eps = float(eps)
    a.uniform_tail = int(bool(uniform_tail))
    return a, m2


def design_workspace_bytes(mass, seq_len, block_size) -> int:
    a, _ = _args(mass, seq_len, block_size, 0, 0, 0, 0, 1.0, False)
    return int(_lib.load().kvbm_design_workspace_bytes(ctypes.byref(a)))


def design_from_mass(mass: torch.Tensor, seq_len: int, block_size: int, tail_budget: int, *, n_sinks: int = 4,
                     recency: int = 32, top_slice: int = 0, eps: float = 1e-6, uniform_tail: bool = False,
                     generator: torch.Generator | None = None, uniforms: torch.Tensor | None = None,
                     seed: int | None = None, with_scores: bool = False, with_log_offsets: bool = False,
                     workspace: torch.Tensor | None = None) -> DeviceDesign:
    """Eviction design(s) from block mass on its CUDA device (see the module docstring)."""
    if not mass.is_cuda:
        raise ValueError("design_from_mass runs on the device of a CUDA mass tensor")
    a, m2 = _args(mass, seq_len, block_size, tail_budget, n_sinks, recency, top_slice, eps, uniform_tail)
    rows, n, dev = a.rows, a.seq_len, mass.device
    keep_alive = [m2]
    if generator is not None and uniforms is None:
        # the reference's draws: torch.rand(n_tail, float64, generator) per row; rand(n)[:k] == rand(k)
        uniforms = torch.stack([torch.rand(n, dtype=torch.float64, generator=generator) for _ in range(rows)])
    if uniforms is not None:
        u = uniforms.to(device=dev, dtype=torch.float64).reshape(rows, -1)
        if u.shape[1] < n:
            raise ValueError(f"uniforms must hold seq_len={n} draws per row, got {u.shape[1]}")
        u = u.contiguous()
        keep_alive.append(u)
        a.uniforms = ctypes.cast(u.data_ptr(), ctypes.POINTER(ctypes.c_double))
        a.uniforms_row_stride = u.stride(0)
    else:
        if seed is None:
            seed = int(torch.randint(0, 2**62, (1,)).item())
        a.seed = int(seed) & (2**64 - 1)
    with torch.cuda.device(dev):
        keep = torch.empty(rows, n, dtype=torch.bool, device=dev)
        pi = torch.empty(rows, n, dtype=torch.float64, device=dev)
        cert = torch.empty(rows, n, dtype=torch.bool, device=dev)
        counts = torch.empty(rows, 5, dtype=torch.int64, device=dev)
        scores = torch.empty(rows, n, dtype=torch.float64, device=dev) if with_scores else None
        logo = torch.empty(rows, n, dtype=torch.float64, device=dev) if with_log_offsets else None
        o = _lib.DesignOut()
        o.pi = ctypes.cast(pi.data_ptr(), ctypes.POINTER(ctypes.c_double))
        o.keep = ctypes.cast(keep.data_ptr(), ctypes.POINTER(ctypes.c_uint8))
        o.certainty = ctypes.cast(cert.data_ptr(), ctypes.POINTER(ctypes.c_uint8))
        o.counts = ctypes.cast(counts.data_ptr(), ctypes.POINTER(ctypes.c_int64))
        if scores is not None:
            o.scores = ctypes.cast(scores.data_ptr(), ctypes.POINTER(ctypes.c_double))
        if logo is not None:
            o.log_offsets = ctypes.cast(logo.data_ptr(), ctypes.POINTER(ctypes.c_double))
        lib = _lib.load()
        need = int(lib.kvbm_design_workspace_bytes(ctypes.byref(a)))
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
        code = lib.kvbm_design(ctypes.byref(a), ctypes.byref(o), workspace.data_ptr(), workspace.numel(),
                               torch.cuda.current_stream(dev).cuda_stream)
        for t in keep_alive:
            t.record_stream(torch.cuda.current_stream(dev))
    if code != _lib.KVBM_OK:
        raise ValueError(f"kvbm_design error {code}: {_lib.status_string(code)}")
    squeeze = mass.dim() == 1

    def sq(t):
        return None if t is None else (t[0] if squeeze else t)

    return DeviceDesign(keep=sq(keep), pi=sq(pi), certainty=sq(cert), counts=counts, tail_budget=int(tail_budget),
                        eps=float(eps), scores=sq(scores), log_offsets=sq(logo))
