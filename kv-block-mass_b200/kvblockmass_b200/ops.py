"""Python entry points for the B200 block-mass kernels.

Drop-in for the reference's GPU path (kv-block-mass):

* ``block_mass_b200`` accepts every argument of ``block_mass_reference``
  (``src/kvblockmass/reference.py:35-45``) and of ``block_mass_triton``
  (``src/kvblockmass/triton_kernel.py:148-158``); ``BLOCK_M``/``BLOCK_N``/
  ``query_chunk`` are accepted and ignored (tiling is the kernel's choice),
  ``device`` moves CPU inputs to that CUDA device first (``reference.py:74-76``).
* ``block_mass_triton`` keeps the reference kernel wrapper's exact signature.
* ``block_mass`` is the dispatcher of ``reference.py:129-135`` for CUDA tensors.

Errors follow the reference: ``H_q % H_kv != 0`` raises ``ValueError`` with
the reference's message (``reference.py:29-30``, ``triton_kernel.py:161-162``).
There is no CPU path: CPU tensors without a CUDA ``device`` raise ``ValueError``.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

__all__ = ["block_mass_b200", "block_mass_triton", "block_mass", "kernel_path", "make_problem",
           "workspace_bytes", "launches_per_call", "block_mass_paged", "make_paged_problem",
           "paged_workspace_bytes", "run_paged", "check_device_errors"]

_DTYPES = {
    torch.float32: _lib.KVBM_F32,
    torch.bfloat16: _lib.KVBM_BF16,
    torch.float16: _lib.KVBM_F16,
    torch.float64: _lib.KVBM_F64,
}

_VALUE_ERRORS = {
    _lib.KVBM_ERR_GQA, _lib.KVBM_ERR_SHAPE, _lib.KVBM_ERR_DTYPE, _lib.KVBM_ERR_HEAD_DIM,
    _lib.KVBM_ERR_BLOCK_SIZE, _lib.KVBM_ERR_UNITS, _lib.KVBM_ERR_NULL,
}


def _raise(code: int, prob: "_lib.Problem"):
    if code == _lib.KVBM_ERR_GQA:
        raise ValueError(f"GQA requires H_q % H_kv == 0, got H_q={prob.Hq}, H_kv={prob.Hkv}")
    msg = f"kvbm error {code}: {_lib.status_string(code)}"
    if code in _VALUE_ERRORS:
        raise ValueError(msg)
    raise RuntimeError(msg)


def _as_mask(m: torch.Tensor, device) -> torch.Tensor:
    m = m.to(device=device)
    if m.dtype != torch.bool:
        m = m != 0
    return m


class _Prepared:
    """A filled ``kvbm_problem`` plus the tensors it points into (kept alive)."""

    def __init__(self, prob, keep, out_dtype, nb):
        self.prob = prob
        self.keep = keep
        self.out_dtype = out_dtype
        self.nb = nb


def make_problem(q, k, attn_mask=None, causal=False, block_size=64, scale=None,
                 causal_skip=True, query_mask=None, units=None) -> _Prepared:
    """Validate arguments and build the C ``kvbm_problem`` for ``q``/``k``.

    Mask shapes (True = keep; combined with ``causal`` by AND):
    ``attn_mask``: ``[N]`` key mask, ``[N, N]`` pair mask (the reference's two
    forms), ``[B|1, 1, N]`` per-batch key mask, ``[B|1, N, N]`` per-batch pair
    mask; ``query_mask``: ``[N]`` or ``[B, N]`` rows to keep (a dropped row
    contributes exactly 0, as a pair-mask row that keeps nothing would).
    """
    if not (isinstance(q, torch.Tensor) and isinstance(k, torch.Tensor)):
        raise TypeError("q and k must be torch tensors")
    if q.dim() != 4 or k.dim() != 4:
        raise ValueError(f"q and k must be 4-D [B, H, N, D], got {tuple(q.shape)} and {tuple(k.shape)}")
    B, Hq, N, D = q.shape
    if k.shape[0] != B or k.shape[2] != N or k.shape[3] != D:
        raise ValueError(f"k shape {tuple(k.shape)} does not match q shape {tuple(q.shape)}")
    Hkv = k.shape[1]
    if Hkv == 0 or Hq % Hkv != 0:
        raise ValueError(f"GQA requires H_q % H_kv == 0, got H_q={Hq}, H_kv={Hkv}")
    if q.device != k.device:
        raise ValueError(f"q and k are on different devices ({q.device}, {k.device})")
    if q.dtype != k.dtype:
        common = torch.promote_types(q.dtype, k.dtype)
        q, k = q.to(common), k.to(common)
    if q.dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {q.dtype}; expected float32, bfloat16, float16 or float64")
    if N == 0:
        raise ValueError("N must be >= 1")
    if block_size is None or int(block_size) < 1:
        raise ValueError("block_size must be >= 1")
    if scale is None:
        scale = 1.0 / D ** 0.5
    dev = q.device
    keep = [q, k]
    prob = _lib.Problem()
    prob.q = q.data_ptr()
    prob.k = k.data_ptr()
    for i in range(4):
        prob.q_stride[i] = q.stride(i)
        prob.k_stride[i] = k.stride(i)
    prob.dtype = _DTYPES[q.dtype]
    prob.B, prob.Hq, prob.Hkv, prob.N, prob.D = B, Hq, Hkv, N, D

    if attn_mask is not None:
        m = _as_mask(attn_mask, dev)
        if m.dim() == 1:
            if m.shape[0] != N:
                raise ValueError(f"attn_mask of shape {tuple(m.shape)} does not match N={N}")
            m = m.contiguous()
            prob.key_mask, prob.key_mask_bstride = m.data_ptr(), 0
        elif m.dim() == 2:
            if tuple(m.shape) != (N, N):
                raise ValueError(f"attn_mask of shape {tuple(m.shape)} is not [N, N] with N={N}")
            if m.stride(1) != 1:
                m = m.contiguous()
            prob.pair_mask, prob.pair_mask_bstride, prob.pair_mask_rstride = m.data_ptr(), 0, m.stride(0)
        elif m.dim() == 3:
            if m.shape[0] not in (1, B) or m.shape[1] not in (1, N) or m.shape[2] != N:
                raise ValueError(f"attn_mask of shape {tuple(m.shape)} is not [B|1, 1|N, N]")
            if m.stride(2) != 1:
                m = m.contiguous()
            bstride = m.stride(0) if m.shape[0] > 1 else 0
            if m.shape[1] == 1:
                prob.key_mask, prob.key_mask_bstride = m.data_ptr(), bstride
            else:
                prob.pair_mask = m.data_ptr()
                prob.pair_mask_bstride, prob.pair_mask_rstride = bstride, m.stride(1)
        else:
            raise ValueError(f"attn_mask must be 1-D, 2-D or 3-D, got {m.dim()}-D")
        keep.append(m)
    if query_mask is not None:
        qm = _as_mask(query_mask, dev)
        if qm.dim() == 1:
            qm = qm.reshape(1, -1)
        if qm.dim() != 2 or qm.shape[0] not in (1, B) or qm.shape[1] != N:
            raise ValueError(f"query_mask of shape {tuple(qm.shape)} is not [N] or [B, N]")
        qm = qm.contiguous()
        prob.query_mask = qm.data_ptr()
        prob.query_mask_bstride = qm.stride(0) if qm.shape[0] > 1 else 0
        keep.append(qm)

    prob.scale = float(scale)
    prob.block_size = int(block_size)
    prob.causal = int(bool(causal))
    prob.causal_skip = int(bool(causal_skip))
    ub, ue = (0, B * Hkv) if units is None else (int(units[0]), int(units[1]))
    prob.unit_begin, prob.unit_end = ub, ue
    code = _lib.load().kvbm_validate(ctypes.byref(prob))
    if code != _lib.KVBM_OK:
        _raise(code, prob)
    nb = (N + int(block_size) - 1) // int(block_size)
    out_dtype = torch.float64 if q.dtype == torch.float64 else torch.float32
    return _Prepared(prob, keep, out_dtype, nb)


def workspace_bytes(prep: _Prepared) -> int:
    return int(_lib.load().kvbm_workspace_bytes(ctypes.byref(prep.prob)))


def kernel_path(prep: _Prepared) -> int:
    """0 = SIMT kernels, 1 = tcgen05 tensor-core kernels (on the current device)."""
    return int(_lib.load().kvbm_kernel_path(ctypes.byref(prep.prob)))


def launches_per_call(prep: _Prepared) -> int:
    return int(_lib.load().kvbm_launches_per_call(ctypes.byref(prep.prob)))


def run_prepared(prep: _Prepared, out: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None,
                 stream: torch.cuda.Stream | None = None,
                 lse: torch.Tensor | None = None) -> torch.Tensor:
    """Launch the kernels of a prepared problem on ``stream`` (default: current).

    With ``lse`` ([B, H_q, N] natural-log row log-sum-exp) pass 1 is skipped.
    """
    q = prep.keep[0]
    dev = q.device
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws_need = int(lib.kvbm_workspace_bytes(ctypes.byref(prep.prob)))
        if workspace is None or workspace.numel() < ws_need:
            workspace = torch.empty(max(ws_need, 256), dtype=torch.uint8, device=dev)
        if out is None:
            out = torch.empty(prep.nb, dtype=prep.out_dtype, device=dev)
        elif out.dtype != prep.out_dtype or out.numel() != prep.nb or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous {prep.out_dtype} tensor of {prep.nb} elements")
        s = stream if stream is not None else torch.cuda.current_stream(dev)
        if lse is None:
            code = lib.kvbm_block_mass(ctypes.byref(prep.prob), out.data_ptr(), workspace.data_ptr(),
                                       workspace.numel(), s.cuda_stream)
        else:
            B, Hq, N = prep.prob.B, prep.prob.Hq, prep.prob.N
            if tuple(lse.shape) != (B, Hq, N):
                raise ValueError(f"lse must be [B, H_q, N] = {(B, Hq, N)}, got {tuple(lse.shape)}")
            lse = lse.to(device=dev, dtype=torch.float32)
            prep.keep.append(lse)
            st = (ctypes.c_int64 * 3)(*lse.stride())
            code = lib.kvbm_block_mass_lse(ctypes.byref(prep.prob), lse.data_ptr(), st, out.data_ptr(),
                                           workspace.data_ptr(), workspace.numel(), s.cuda_stream)
    if code != _lib.KVBM_OK:
        _raise(code, prep.prob)
    return out


def block_mass_b200(q, k, attn_mask=None, causal=False, block_size=64, scale=None,
                    causal_skip=True, query_mask=None, *, BLOCK_M=None, BLOCK_N=None,
                    query_chunk=None, device=None, units=None, out=None, workspace=None, lse=None):
    """Block-pooled column sums of the softmax attention matrix on a B200.

    Returns ``mass [ceil(N / block_size)]`` (float32; float64 for float64
    inputs) on the CUDA device of ``q``.  ``units=(begin, end)`` restricts the
    sum to the (batch, kv-head) units ``[begin, end)`` of ``B * H_kv`` (used by
    the multi-GPU shards); ``out``/``workspace`` let callers reuse buffers.
    ``lse`` ([B, H_q, N], natural log of sum_c exp(scale * q.k_c) over the kept
    keys, e.g. the softmax LSE an attention forward returns) skips the row
    statistics pass: about half the work.
    """
    del BLOCK_M, BLOCK_N, query_chunk  # tiling is fixed by the kernels
    if device is not None:
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError(f"block_mass_b200 computes on CUDA devices only, got device={device}")
        if (not q.is_cuda and not k.is_cuda and q.is_pinned() and k.is_pinned() and units is None
                and lse is None and out is None and q.dim() == 4 and k.dim() == 4):
            return _from_pinned_host(q, k, dev, attn_mask=attn_mask, causal=causal, block_size=block_size,
                                     scale=scale, causal_skip=causal_skip, query_mask=query_mask,
                                     workspace=workspace)
        q, k = q.to(dev), k.to(dev)
    if not (q.is_cuda and k.is_cuda):
        raise ValueError("block_mass_b200 needs CUDA tensors (there is no CPU path); "
                         "pass device='cuda' or use the reference's block_mass_reference")
    prep = make_problem(q, k, attn_mask=attn_mask, causal=causal, block_size=block_size,
                        scale=scale, causal_skip=causal_skip, query_mask=query_mask, units=units)
    return run_prepared(prep, out=out, workspace=workspace, lse=lse)


_COPY_STREAMS: dict = {}


def _copy_stream(dev: torch.device) -> torch.cuda.Stream:
    if dev not in _COPY_STREAMS:
        _COPY_STREAMS[dev] = torch.cuda.Stream(device=dev)
    return _COPY_STREAMS[dev]


def _from_pinned_host(q, k, dev, attn_mask, causal, block_size, scale, causal_skip, query_mask, workspace,
                      target_units: int = 2):
    """Pinned host q/k: overlap the host-to-device copy with the kernels.

    The (batch, kv-head) units are cut into contiguous segments; a side
    stream copies segment i + 1 while segment i runs on the caller's stream,
    and the per-segment mass vectors are added in segment order (deterministic;
    the grouping of the final sum differs from one call over all units, so the
    bits can differ from it in the last place).
    """
    from .distributed import unit_segments

    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    if Hkv == 0 or Hq % Hkv != 0:
        raise ValueError(f"GQA requires H_q % H_kv == 0, got H_q={Hq}, H_kv={Hkv}")
    G = Hq // Hkv
    with torch.cuda.device(dev):
        qd = torch.empty(q.shape, dtype=q.dtype, device=dev)
        kd = torch.empty(k.shape, dtype=k.dtype, device=dev)
        compute = torch.cuda.current_stream(dev)
        copy = _copy_stream(dev)
        copy.wait_stream(compute)  # qd/kd may reuse memory the compute stream still reads
        am = None if attn_mask is None else attn_mask.to(dev, non_blocking=True)
        qm = None if query_mask is None else query_mask.to(dev, non_blocking=True)
        U = B * Hkv
        step = max(1, min(target_units, U))
        bounds = [(u, min(U, u + step)) for u in range(0, U, step)]
        parts = []
        for ub, ue in bounds:
            with torch.cuda.stream(copy):
                for b, g0, g1 in unit_segments(ub, ue, Hkv):
                    qd[b, g0 * G:g1 * G].copy_(q[b, g0 * G:g1 * G], non_blocking=True)
                    kd[b, g0:g1].copy_(k[b, g0:g1], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy)
            compute.wait_event(ev)
            prep = make_problem(qd, kd, attn_mask=am, causal=causal, block_size=block_size, scale=scale,
                                causal_skip=causal_skip, query_mask=qm, units=(ub, ue))
            parts.append(run_prepared(prep, workspace=workspace))
        # qd/kd were written on the copy stream: tell the allocator before they are freed
        qd.record_stream(copy)
        kd.record_stream(copy)
        total = parts[0].clone()
        for m in parts[1:]:
            total += m
        return total


def block_mass_triton(q, k, attn_mask=None, causal=False, block_size=64, scale=None,
                      BLOCK_M=64, BLOCK_N=64, causal_skip=True):
    """Same signature as the reference's ``block_mass_triton`` (``triton_kernel.py:148-158``)."""
    return block_mass_b200(q, k, attn_mask=attn_mask, causal=causal, block_size=block_size,
                           scale=scale, causal_skip=causal_skip, BLOCK_M=BLOCK_M, BLOCK_N=BLOCK_N)


def block_mass(q, k, **kwargs):
    """Dispatcher of ``reference.py:129-135``: CUDA tensors run the B200 kernels."""
    if q.is_cuda or kwargs.get("device") not in (None, "cpu"):
        return block_mass_b200(q, k, **kwargs)
    raise ValueError("kvblockmass_b200.block_mass handles CUDA tensors; CPU tensors belong to "
                     "the reference's block_mass_reference")


class _PagedPrepared:
    """A dense ``kvbm_problem`` (its k ignored) plus the ``kvbm_paged_kv`` of the cache."""

    def __init__(self, prep: _Prepared, kv, keep):
        self.prep = prep
        self.kv = kv
        self.keep = keep


def make_paged_problem(q, k_cache, block_table, attn_mask=None, causal=False, block_size=64, scale=None,
                       causal_skip=True, query_mask=None, units=None) -> _PagedPrepared:
    """Validate a paged call and build its C structs.

    ``k_cache`` is ``[num_pages, page_size, H_kv, D]`` (any strides, the dtype
    of ``q``); ``block_table`` is ``[B, max_pages]`` of page ids (converted to
    int32): key ``n`` of sequence ``b`` is ``k_cache[block_table[b, n // P], n % P]``.
    Every sequence has ``N = q.shape[2]`` keys.
    """
    if not all(isinstance(t, torch.Tensor) for t in (q, k_cache, block_table)):
        raise TypeError("q, k_cache and block_table must be torch tensors")
    if q.dim() != 4 or k_cache.dim() != 4:
        raise ValueError(f"q must be [B, H_q, N, D] and k_cache [num_pages, page_size, H_kv, D], "
                         f"got {tuple(q.shape)} and {tuple(k_cache.shape)}")
    B, Hq, N, D = q.shape
    num_pages, page_size, Hkv, Dk = k_cache.shape
    if Dk != D:
        raise ValueError(f"k_cache head dim {Dk} != q head dim {D}")
    if block_table.dim() != 2 or block_table.shape[0] != B:
        raise ValueError(f"block_table must be [B={B}, max_pages], got {tuple(block_table.shape)}")
    if block_table.dtype.is_floating_point or block_table.dtype == torch.bool:
        raise ValueError(f"block_table must hold integer page ids, got {block_table.dtype}")
    if k_cache.dtype != q.dtype:
        raise ValueError(f"k_cache dtype {k_cache.dtype} != q dtype {q.dtype}")
    if not (q.device == k_cache.device == block_table.device):
        raise ValueError("q, k_cache and block_table must be on one device")
    if num_pages == 0 or page_size == 0:
        raise ValueError("k_cache has no pages")
    if block_table.shape[1] * page_size < N:
        raise ValueError(f"block_table covers {block_table.shape[1] * page_size} keys < N={N}")
    table = block_table.to(torch.int32)
    if table.stride(1) != 1:
        table = table.contiguous()
    # stand-in dense k: make_problem checks shapes and masks; the C call ignores it
    k_shape = torch.empty((), dtype=q.dtype, device=q.device).expand(B, Hkv, N, D)
    prep = make_problem(q, k_shape, attn_mask=attn_mask, causal=causal, block_size=block_size, scale=scale,
                        causal_skip=causal_skip, query_mask=query_mask, units=units)
    kv = _lib.PagedKV()
    kv.k_cache = k_cache.data_ptr()
    for i in range(4):
        kv.cache_stride[i] = k_cache.stride(i)
    kv.num_pages, kv.page_size = num_pages, page_size
    kv.block_table = table.data_ptr()
    kv.block_table_stride = table.stride(0)
    kv.max_pages = table.shape[1]
    code = _lib.load().kvbm_validate_paged(ctypes.byref(prep.prob), ctypes.byref(kv))
    if code != _lib.KVBM_OK:
        _raise(code, prep.prob)
    return _PagedPrepared(prep, kv, [k_cache, table])


def paged_workspace_bytes(pp: _PagedPrepared) -> int:
    return int(_lib.load().kvbm_paged_workspace_bytes(ctypes.byref(pp.prep.prob), ctypes.byref(pp.kv)))


def run_paged(pp: _PagedPrepared, out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
              stream: torch.cuda.Stream | None = None, lse: torch.Tensor | None = None) -> torch.Tensor:
    """Launch a prepared paged problem (page gather, then the dense kernels) on ``stream``."""
    prep = pp.prep
    dev = prep.keep[0].device
    lib = _lib.load()
    with torch.cuda.device(dev):
        need = paged_workspace_bytes(pp)
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
        if out is None:
            out = torch.empty(prep.nb, dtype=prep.out_dtype, device=dev)
        elif out.dtype != prep.out_dtype or out.numel() != prep.nb or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous {prep.out_dtype} tensor of {prep.nb} elements")
        s = stream if stream is not None else torch.cuda.current_stream(dev)
        lse_ptr, st = None, None
        if lse is not None:
            B, Hq, N = prep.prob.B, prep.prob.Hq, prep.prob.N
            if tuple(lse.shape) != (B, Hq, N):
                raise ValueError(f"lse must be [B, H_q, N] = {(B, Hq, N)}, got {tuple(lse.shape)}")
            lse = lse.to(device=dev, dtype=torch.float32)
            pp.keep.append(lse)
            lse_ptr, st = lse.data_ptr(), (ctypes.c_int64 * 3)(*lse.stride())
        code = lib.kvbm_block_mass_paged(ctypes.byref(prep.prob), ctypes.byref(pp.kv), lse_ptr, st,
                                         out.data_ptr(), workspace.data_ptr(), workspace.numel(), s.cuda_stream)
    if code != _lib.KVBM_OK:
        _raise(code, prep.prob)
    return out


def block_mass_paged(q, k_cache, block_table, attn_mask=None, causal=False, block_size=64, scale=None,
                     causal_skip=True, query_mask=None, *, units=None, out=None, workspace=None, lse=None):
    """``block_mass_b200`` with keys read from a paged KV cache.

    ``k_cache [num_pages, page_size, H_kv, D]`` and ``block_table [B,
    max_pages]`` (page ids) on the device of ``q [B, H_q, N, D]``; the other
    arguments as ``block_mass_b200``.  ``block_size == page_size`` gives one
    bucket per page.  The result has the same bits as ``block_mass_b200`` on
    the dense keys the table names.  A page id outside ``[0, num_pages)`` is
    not read (its keys count as zero vectors); ``check_device_errors()``
    reports it.
    """
    if not (q.is_cuda and k_cache.is_cuda):
        raise ValueError("block_mass_paged needs CUDA tensors (there is no CPU path)")
    pp = make_paged_problem(q, k_cache, block_table, attn_mask=attn_mask, causal=causal, block_size=block_size,
                            scale=scale, causal_skip=causal_skip, query_mask=query_mask, units=units)
    return run_paged(pp, out=out, workspace=workspace, lse=lse)


def check_device_errors(device=None) -> None:
    """Raise ``RuntimeError`` if a kernel on ``device`` recorded an error since the last check.

    Two conditions are recorded on the device instead of faulting: a bounded
    wait in a tensor-core kernel that ran out (``KVBM_ERR_TIMEOUT``) and a
    block-table entry outside the cache (``KVBM_ERR_PAGE``).  Synchronises the
    current stream; both words are cleared.
    """
    dev = torch.device("cuda") if device is None else torch.device(device)
    with torch.cuda.device(dev):
        code = _lib.load().kvbm_check_device_errors(torch.cuda.current_stream(dev).cuda_stream)
    if code != _lib.KVBM_OK:
        raise RuntimeError(f"kvbm error {code}: {_lib.status_string(code)}")
