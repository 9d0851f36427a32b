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
           "paged_workspace_bytes", "run_paged", "check_device_errors", "block_mass_varlen",
           "make_varlen_problem", "run_prepared", "run_staged", "method_of"]

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
    """A filled ``kvbm_problem`` (+ ``kvbm_options``) and the tensors they point into."""

    def __init__(self, prob, keep, out_dtype, nb):
        self.prob = prob
        self.keep = keep
        self.out_dtype = out_dtype
        self.nb = nb
        self.opts = None          # _lib.Options when any extension is used
        self.per_sequence = False
        self.packed = False       # q rows addressed through cu_seqlens
        self.total = 0            # rows of a packed q

    @property
    def out_shape(self):
        return (self.prob.B, self.nb) if self.per_sequence else (self.nb,)

    def options(self) -> "_lib.Options":
        if self.opts is None:
            self.opts = _lib.Options()
        return self.opts


def _int32_on(t: torch.Tensor, dev, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or t.dim() != 1:
        raise ValueError(f"{name} must be a 1-D integer tensor")
    if t.dtype.is_floating_point or t.dtype == torch.bool:
        raise ValueError(f"{name} must hold integers, got {t.dtype}")
    return t.to(device=dev, dtype=torch.int32).contiguous()


def _fill_problem(q_ptr, q_strides, k_ptr, k_strides, dtype, B, Hq, Hkv, N, D, dev, keep, attn_mask, causal,
                  block_size, scale, causal_skip, query_mask, units) -> _Prepared:
    """Shared tail of the make_*_problem functions: masks, scalars, validation."""
    if Hkv == 0 or Hq % Hkv != 0:
        raise ValueError(f"GQA requires H_q % H_kv == 0, got H_q={Hq}, H_kv={Hkv}")
    if dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {dtype}; expected float32, bfloat16, float16 or float64")
    if N == 0:
        raise ValueError("N must be >= 1")
    if block_size is None or int(block_size) < 1:
        raise ValueError("block_size must be >= 1")
    if scale is None:
        scale = 1.0 / D ** 0.5
    prob = _lib.Problem()
    prob.q = q_ptr
    prob.k = k_ptr
    for i in range(4):
        prob.q_stride[i] = q_strides[i]
        prob.k_stride[i] = k_strides[i]
    prob.dtype = _DTYPES[dtype]
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
    out_dtype = torch.float64 if dtype == torch.float64 else torch.float32
    return _Prepared(prob, keep, out_dtype, nb)


def _set_ragged(prep: _Prepared, dev, seq_lens=None, cu_seqlens=None, total=0, per_sequence=False):
    if seq_lens is not None and cu_seqlens is not None:
        raise ValueError("seq_lens and cu_seqlens are exclusive")
    B = prep.prob.B
    if seq_lens is not None:
        lens = _int32_on(seq_lens, dev, "seq_lens")
        if lens.shape[0] != B:
            raise ValueError(f"seq_lens must have B={B} entries, got {lens.shape[0]}")
        prep.keep.append(lens)
        prep.options().seq_lens = lens.data_ptr()
    if cu_seqlens is not None:
        cu = _int32_on(cu_seqlens, dev, "cu_seqlens")
        if cu.shape[0] != B + 1:
            raise ValueError(f"cu_seqlens must have B + 1 = {B + 1} entries, got {cu.shape[0]}")
        prep.keep.append(cu)
        o = prep.options()
        o.cu_seqlens = cu.data_ptr()
        o.total_tokens = int(total)
        prep.packed = True
        prep.total = int(total)
    if per_sequence:
        prep.per_sequence = True
        prep.options().per_sequence = 1


def _validate_ex(prep: _Prepared):
    if prep.opts is None:
        return
    code = _lib.load().kvbm_validate_ex(ctypes.byref(prep.prob), ctypes.byref(prep.opts))
    if code != _lib.KVBM_OK:
        _raise(code, prep.prob)


_METHODS = {None: 0, "auto": 0, "two_pass": 1, "one_pass": 2}


def _set_method(prep: _Prepared, method) -> None:
    if method not in _METHODS:
        raise ValueError(f"method must be one of 'auto', 'two_pass', 'one_pass', got {method!r}")
    if _METHODS[method]:
        prep.options().method = _METHODS[method]


def make_problem(q, k, attn_mask=None, causal=False, block_size=64, scale=None,
                 causal_skip=True, query_mask=None, units=None, seq_lens=None,
                 per_sequence=False, method=None) -> _Prepared:
    """Validate arguments and build the C ``kvbm_problem`` for ``q``/``k``.

    Mask shapes (True = keep; combined with ``causal`` by AND):
    ``attn_mask``: ``[N]`` key mask, ``[N, N]`` pair mask (the reference's two
    forms), ``[B|1, 1, N]`` per-batch key mask, ``[B|1, N, N]`` per-batch pair
    mask; ``query_mask``: ``[N]`` or ``[B, N]`` rows to keep (a dropped row
    contributes exactly 0, as a pair-mask row that keeps nothing would).
    ``seq_lens`` ``[B]``: sequence ``b`` is its first ``seq_lens[b] <= N``
    positions (ragged batch in the padded layout); ``per_sequence``: the
    output is ``[B, num_blocks]``, one row per sequence.  ``method``:
    ``"two_pass"`` (row statistics, then a second pass over the scores),
    ``"one_pass"`` (pass 1 keeps per-segment log-sums and forms the mass
    itself; tensor-core paths, block_size a multiple of 64) or ``"auto"``
    (None: one pass where it applies).
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
    prep = _fill_problem(q.data_ptr(), q.stride(), k.data_ptr(), k.stride(), q.dtype, B, Hq, Hkv, N, D,
                         q.device, [q, k], attn_mask, causal, block_size, scale, causal_skip, query_mask, units)
    _set_ragged(prep, q.device, seq_lens=seq_lens, per_sequence=per_sequence)
    _set_method(prep, method)
    _validate_ex(prep)
    return prep


def make_varlen_problem(q, k, cu_seqlens, max_seqlen=None, attn_mask=None, causal=False, block_size=64,
                        scale=None, causal_skip=True, query_mask=None, units=None,
                        per_sequence=False, method=None) -> _Prepared:
    """Packed (varlen) batch: ``q [T, H_q, D]``, ``k [T, H_kv, D]``, sequence ``b``
    is rows ``[cu_seqlens[b], cu_seqlens[b + 1])``.  ``max_seqlen`` (host int,
    read from ``cu_seqlens`` when omitted) is the bucket extent ``N``; masks
    index positions inside a sequence, as for ``[B, N]`` tensors."""
    if not all(isinstance(t, torch.Tensor) for t in (q, k, cu_seqlens)):
        raise TypeError("q, k and cu_seqlens must be torch tensors")
    if q.dim() != 3 or k.dim() != 3:
        raise ValueError(f"packed q and k must be 3-D [T, H, D], got {tuple(q.shape)} and {tuple(k.shape)}")
    T, Hq, D = q.shape
    if k.shape[0] != T or k.shape[2] != D:
        raise ValueError(f"k shape {tuple(k.shape)} does not match q shape {tuple(q.shape)}")
    if q.device != k.device:
        raise ValueError(f"q and k are on different devices ({q.device}, {k.device})")
    if q.dtype != k.dtype:
        raise ValueError(f"q dtype {q.dtype} != k dtype {k.dtype}")
    if cu_seqlens.dim() != 1 or cu_seqlens.shape[0] < 2:
        raise ValueError("cu_seqlens must be [B + 1] with B >= 1")
    if max_seqlen is None:
        cu_h = cu_seqlens.detach().to("cpu", torch.int64)
        max_seqlen = int((cu_h[1:] - cu_h[:-1]).max())
    B, Hkv = cu_seqlens.shape[0] - 1, k.shape[1]
    qs = (0, q.stride(1), q.stride(0), q.stride(2))
    ks = (0, k.stride(1), k.stride(0), k.stride(2))
    prep = _fill_problem(q.data_ptr(), qs, k.data_ptr(), ks, q.dtype, B, Hq, Hkv, int(max_seqlen), D, q.device,
                         [q, k], attn_mask, causal, block_size, scale, causal_skip, query_mask, units)
    _set_ragged(prep, q.device, cu_seqlens=cu_seqlens, total=T, per_sequence=per_sequence)
    _set_method(prep, method)
    _validate_ex(prep)
    return prep


def workspace_bytes(prep: _Prepared) -> int:
    lib = _lib.load()
    if prep.opts is not None:
        return int(lib.kvbm_workspace_bytes_ex(ctypes.byref(prep.prob), ctypes.byref(prep.opts)))
    return int(lib.kvbm_workspace_bytes(ctypes.byref(prep.prob)))


def kernel_path(prep: _Prepared) -> int:
    """0 = SIMT kernels, 1 = tcgen05 tensor-core kernels, 2 = tcgen05 3xTF32 (current device)."""
    return int(_lib.load().kvbm_kernel_path(ctypes.byref(prep.prob)))


def method_of(prep: _Prepared) -> str:
    """``"one_pass"`` or ``"two_pass"``: how the current device runs ``prep``."""
    opts = ctypes.byref(prep.opts) if prep.opts is not None else None
    code = int(_lib.load().kvbm_method(ctypes.byref(prep.prob), opts))
    if code < 0:
        _raise(-code, prep.prob)
    return "one_pass" if code == _lib.KVBM_METHOD_ONE_PASS else "two_pass"


def launches_per_call(prep: _Prepared) -> int:
    return int(_lib.load().kvbm_launches_per_call(ctypes.byref(prep.prob)))


def _lse_strides(prep: _Prepared, lse: torch.Tensor):
    B, Hq, N = prep.prob.B, prep.prob.Hq, prep.prob.N
    if prep.packed:
        if tuple(lse.shape) != (Hq, prep.total):
            raise ValueError(f"packed lse must be [H_q, T] = {(Hq, prep.total)}, got {tuple(lse.shape)}")
        return (0, lse.stride(0), lse.stride(1))
    if tuple(lse.shape) != (B, Hq, N):
        raise ValueError(f"lse must be [B, H_q, N] = {(B, Hq, N)}, got {tuple(lse.shape)}")
    return tuple(lse.stride())


def run_prepared(prep: _Prepared, out: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None,
                 stream: torch.cuda.Stream | None = None,
                 lse: torch.Tensor | None = None) -> torch.Tensor:
    """Launch the kernels of a prepared problem on ``stream`` (default: current).

    With ``lse`` (``[B, H_q, N]`` natural-log row log-sum-exp; ``[H_q, T]`` for
    a packed batch) the row statistics are not recomputed.
    """
    q = prep.keep[0]
    dev = q.device
    lib = _lib.load()
    with torch.cuda.device(dev):
        opts = prep.opts
        if lse is not None:
            lse = lse.to(device=dev, dtype=torch.float32)
            st = _lse_strides(prep, lse)
            prep.keep.append(lse)
            opts = prep.options()
            opts.lse = lse.data_ptr()
            for i in range(3):
                opts.lse_stride[i] = st[i]
        ws_need = workspace_bytes(prep)
        if workspace is None or workspace.numel() < ws_need:
            workspace = torch.empty(max(ws_need, 256), dtype=torch.uint8, device=dev)
        if out is None:
            out = torch.empty(prep.out_shape, dtype=prep.out_dtype, device=dev)
        elif out.dtype != prep.out_dtype or tuple(out.shape) != prep.out_shape or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous {prep.out_dtype} tensor of shape {prep.out_shape}")
        s = stream if stream is not None else torch.cuda.current_stream(dev)
        if opts is None:
            code = lib.kvbm_block_mass(ctypes.byref(prep.prob), out.data_ptr(), workspace.data_ptr(),
                                       workspace.numel(), s.cuda_stream)
        else:
            code = lib.kvbm_block_mass_ex(ctypes.byref(prep.prob), ctypes.byref(opts), out.data_ptr(),
                                          workspace.data_ptr(), workspace.numel(), s.cuda_stream)
        if lse is not None:
            opts.lse = None
    if code != _lib.KVBM_OK:
        _raise(code, prep.prob)
    return out


def block_mass_b200(q, k, attn_mask=None, causal=False, block_size=64, scale=None,
                    causal_skip=True, query_mask=None, *, BLOCK_M=None, BLOCK_N=None,
                    query_chunk=None, device=None, units=None, out=None, workspace=None, lse=None,
                    seq_lens=None, per_sequence=False, method=None):
    """Block-pooled column sums of the softmax attention matrix on a B200.

    Returns ``mass [ceil(N / block_size)]`` (float32; float64 for float64
    inputs) on the CUDA device of ``q``.  ``units=(begin, end)`` restricts the
    sum to the (batch, kv-head) units ``[begin, end)`` of ``B * H_kv`` (used by
    the multi-GPU shards); ``out``/``workspace`` let callers reuse buffers.
    ``lse`` ([B, H_q, N], natural log of sum_c exp(scale * q.k_c) over the kept
    keys, e.g. the softmax LSE an attention forward returns) spares the row
    statistics (one pass: no running max; two passes: no pass 1).  ``seq_lens [B]`` makes the batch
    ragged (sequence ``b`` is its first ``seq_lens[b]`` positions; the padding
    is never read into a pair); ``per_sequence`` returns ``[B, num_blocks]``.
    ``method`` as for ``make_problem``.
    """
    del BLOCK_M, BLOCK_N, query_chunk  # tiling is fixed by the kernels
    if device is not None:
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError(f"block_mass_b200 computes on CUDA devices only, got device={device}")
        if (not q.is_cuda and not k.is_cuda and units is None and lse is None and out is None
                and q.dim() == 4 and k.dim() == 4 and q.dtype == k.dtype and seq_lens is None
                and not per_sequence and q.numel() > 0 and k.numel() > 0):
            return _from_host(q, k, dev, attn_mask=attn_mask, causal=causal, block_size=block_size,
                              scale=scale, causal_skip=causal_skip, query_mask=query_mask,
                              workspace=workspace, method=method)
        q, k = q.to(dev), k.to(dev)
    if not (q.is_cuda and k.is_cuda):
        raise ValueError("block_mass_b200 needs CUDA tensors (there is no CPU path); "
                         "pass device='cuda' or use the reference's block_mass_reference")
    prep = make_problem(q, k, attn_mask=attn_mask, causal=causal, block_size=block_size,
                        scale=scale, causal_skip=causal_skip, query_mask=query_mask, units=units,
                        seq_lens=seq_lens, per_sequence=per_sequence, method=method)
    return run_prepared(prep, out=out, workspace=workspace, lse=lse)


_COPY_STREAMS: dict = {}
_SIDE_STREAMS: dict = {}


def _copy_stream(dev: torch.device) -> torch.cuda.Stream:
    if dev not in _COPY_STREAMS:
        _COPY_STREAMS[dev] = torch.cuda.Stream(device=dev)
    return _COPY_STREAMS[dev]


def _side_stream(dev: torch.device) -> torch.cuda.Stream:
    if dev not in _SIDE_STREAMS:
        _SIDE_STREAMS[dev] = torch.cuda.Stream(device=dev)
    return _SIDE_STREAMS[dev]


def run_staged(prep: _Prepared, stages: int, workspace: torch.Tensor, out: torch.Tensor | None = None,
               units: tuple[int, int] | None = None, heads: tuple[int, int] | None = None,
               stream: torch.cuda.Stream | None = None, rows: tuple[int, int] | None = None) -> None:
    """One staged launch of a prepared problem (``kvbm_options.stages``).

    ``stages`` is a mask of ``_lib.KVBM_STAGE_*``; ``units`` is a range of the
    problem's units (relative to its unit range) that passes 1 and 2 cover,
    ``heads`` a range of q-heads of each GQA group that pass 1 covers (needs a
    one-unit ``units``), ``rows`` a range of query rows that pass 1 covers
    (begin a multiple of 128, end a multiple of 128 or N; kernel paths 0 and
    1).  Every piece writes into ``workspace``, which must be
    sized for the whole problem; the reduce stage then gives the bits of one
    whole call.
    """
    o = prep.options()
    o.stages = int(stages)
    o.run_unit_begin, o.run_unit_end = units if units is not None else (0, 0)
    o.run_head_begin, o.run_head_end = heads if heads is not None else (0, 0)
    o.run_row_begin, o.run_row_end = rows if rows is not None else (0, 0)
    s = stream if stream is not None else torch.cuda.current_stream(prep.keep[0].device)
    try:
        code = _lib.load().kvbm_block_mass_ex(ctypes.byref(prep.prob), ctypes.byref(o),
                                              None if out is None else out.data_ptr(), workspace.data_ptr(),
                                              workspace.numel(), s.cuda_stream)
    finally:
        o.stages = o.run_unit_begin = o.run_unit_end = o.run_head_begin = o.run_head_end = 0
        o.run_row_begin = o.run_row_end = 0
    if code != _lib.KVBM_OK:
        _raise(code, prep.prob)


def _host_pieces(U: int, G: int, N: int, by_rows: bool) -> list:
    """The pieces of a host-input call: (unit, (head0, head1), (row0, row1) or
    None, stages, whether the unit's k travels with it).

    With ``by_rows`` (kernel paths 0 and 1, N >= 4096) every unit is cut into
    three pieces of query rows, and the pieces go in order of work per byte:
    first rows [N/2, N) of every unit with its k, then rows [N/4, N/2) of
    every unit, then rows [0, N/4).  Under causal masking pass 1 of rows
    [r0, r1) reads k rows [0, r1), and its work per byte of q grows with r1:
    the last half of the rows carries three quarters of a unit's work in 60 %
    of its bytes (with k), the first quarter 1/16 of the work in 20 %.  So the
    kernels run ahead of the copies while the earlier rows still stream in,
    and the pieces copied last are short.
    Otherwise unit 0 goes first as q-head 0 (with the k), then its other
    q-heads, and every further unit is one piece with both passes.  A unit cut
    into pieces runs pass 2 after its last piece.
    """
    P1, P2 = _lib.KVBM_STAGE_PASS1, _lib.KVBM_STAGE_PASS2
    if by_rows and N >= 4096:
        half = (N // 2 + 127) // 128 * 128
        quarter = (N // 4 + 127) // 128 * 128
        return [(u, (0, G), (half, N), P1, True) for u in range(U)] + \
            [(u, (0, G), (quarter, half), P1, False) for u in range(U)] + \
            [(u, (0, G), (0, quarter), P1, False) for u in range(U)]
    if G > 1:
        pieces = [(0, (0, 1), None, P1, True), (0, (1, G), None, P1, False)]
    else:
        pieces = [(0, (0, 1), None, P1, True)]
    return pieces + [(u, (0, G), None, P1 | P2, True) for u in range(1, U)]


def _from_host(q, k, dev, attn_mask, causal, block_size, scale, causal_skip, query_mask, workspace, method=None):
    """Host q/k (pinned or pageable): overlap the host-to-device copies with the kernels.

    The copy stream moves the inputs one piece at a time (``_host_pieces``)
    while the kernels run the pieces that have arrived, as staged calls into
    one workspace sized for the whole problem; one bucket reduce at the end
    sums every unit, so the result has the bits of ``kvbm_block_mass`` on the
    same values.  The first piece's copies are queued before the problem is
    planned.  Consecutive pieces alternate between the caller's stream and a
    second compute stream, so one piece's pass 1 fills the SMs its
    predecessor's last CTAs leave idle.

    Pageable tensors are staged through two pinned bounce buffers of one unit
    each: the host copies piece i + 1 into one while the copy engine reads
    piece i from the other (and the GPU computes piece i - 1).
    """
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    if Hkv == 0 or Hq % Hkv != 0:
        raise ValueError(f"GQA requires H_q % H_kv == 0, got H_q={Hq}, H_kv={Hkv}")
    G = Hq // Hkv
    pinned = q.is_pinned() and k.is_pinned()
    S = _lib
    with torch.cuda.device(dev):
        qd = torch.empty(q.shape, dtype=q.dtype, device=dev)
        kd = torch.empty(k.shape, dtype=k.dtype, device=dev)
        compute = torch.cuda.current_stream(dev)
        copy = _copy_stream(dev)
        side = _side_stream(dev)
        copy.wait_stream(compute)  # qd/kd may reuse memory the compute stream still reads
        # fp32 may run the 3xTF32 path, which takes no row pieces; pageable
        # tensors keep whole-head pieces (the host copies into the bounce
        # buffers run faster in large pieces)
        pieces = _host_pieces(B * Hkv, G, N, pinned and q.dtype != torch.float32)
        bounce, bounce_ev = None, [None, None]
        if not pinned:
            unit_bytes = (G * N * D * q.element_size()) + N * D * k.element_size()
            bounce = [torch.empty(unit_bytes, dtype=torch.uint8, pin_memory=True) for _ in range(2)]

        # pinned q/k whose rows are contiguous: a piece is one 2-D copy of q
        # (the same rows of its q-heads) and one of k, with no tensor views
        direct = pinned and q.stride(3) == 1 and q.stride(2) == D and k.stride(3) == 1 and k.stride(2) == D
        lib, es = _lib.load(), q.element_size()

        def copy2d(dst, d_off, d_pitch, src, s_off, s_pitch, width, height):
            code = lib.kvbm_copy_2d_async(dst.data_ptr() + d_off * es, d_pitch * es, src.data_ptr() + s_off * es,
                                          s_pitch * es, width * es, height, copy.cuda_stream)
            if code != _lib.KVBM_OK:
                raise RuntimeError(f"kvbm error {code}: {_lib.status_string(code)}")

        def copies(i):
            """Queue piece i's host-to-device copies; the event marks their end."""
            u, (h0, h1), rows, _, with_k = pieces[i]
            b, g = divmod(u, Hkv)
            if direct:
                r0, r1 = rows if rows is not None else (0, N)
                if with_k:
                    copy2d(kd, b * kd.stride(0) + g * kd.stride(1), 0, k, b * k.stride(0) + g * k.stride(1), 0,
                           N * D, 1)
                h = g * G + h0
                copy2d(qd, b * qd.stride(0) + h * qd.stride(1) + r0 * D, qd.stride(1),
                       q, b * q.stride(0) + h * q.stride(1) + r0 * D, q.stride(1), (r1 - r0) * D, h1 - h0)
                ev = torch.cuda.Event()
                ev.record(copy)
                return ev
            cps = [(kd[b, g], k[b, g])] if with_k else []
            qu, qdu = q[b, g * G:(g + 1) * G], qd[b, g * G:(g + 1) * G]
            if rows is None:  # whole heads: one contiguous copy
                cps.append((qdu[h0:h1], qu[h0:h1]))
            else:
                cps += [(qdu[h, rows[0]:rows[1]], qu[h, rows[0]:rows[1]]) for h in range(h0, h1)]
            with torch.cuda.stream(copy):
                if pinned:
                    for dst, src in cps:
                        dst.copy_(src, non_blocking=True)
                else:
                    j = i % 2
                    if bounce_ev[j] is not None:
                        bounce_ev[j].synchronize()  # the copy engine has read this buffer
                    off = 0
                    for dst, src in cps:
                        n = src.numel() * src.element_size()
                        stage = bounce[j][off:off + n].view(src.dtype).view(src.shape)
                        stage.copy_(src)
                        dst.copy_(stage, non_blocking=True)
                        off += n
                    bounce_ev[j] = torch.cuda.Event()
                    bounce_ev[j].record(copy)
                ev = torch.cuda.Event()
                ev.record(copy)
            return ev

        first = copies(0)
        am = None if attn_mask is None else attn_mask.to(dev, non_blocking=True)
        qm = None if query_mask is None else query_mask.to(dev, non_blocking=True)
        prep = make_problem(qd, kd, attn_mask=am, causal=causal, block_size=block_size, scale=scale,
                            causal_skip=causal_skip, query_mask=qm, method=method)
        need = workspace_bytes(prep)
        ws = workspace if workspace is not None and workspace.numel() >= need else \
            torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
        out = torch.empty(prep.out_shape, dtype=prep.out_dtype, device=dev)
        if prep.prob.pair_mask or prep.prob.key_mask:
            run_staged(prep, S.KVBM_STAGE_MASKS, ws, stream=compute)
        side.wait_stream(compute)  # the masks, their bits, and anything the caller queued
        streams = [compute, side]
        # units cut into pass-1 pieces: their pass 2 follows their last piece
        last_piece = {pc[0]: i for i, pc in enumerate(pieces) if not pc[3] & S.KVBM_STAGE_PASS2}
        latest = {}  # (unit, stream index) -> event after that unit's latest piece there
        for i, (u, heads, rows, stages, _) in enumerate(pieces):
            ev = first if i == 0 else copies(i)
            st = streams[i % 2]
            st.wait_event(ev)
            run_staged(prep, stages, ws, units=(u, u + 1), heads=heads, rows=rows, stream=st)
            if u not in last_piece:
                continue
            if i < last_piece[u]:
                latest[(u, i % 2)] = torch.cuda.Event()
                latest[(u, i % 2)].record(st)
            else:
                # pass 2 of the unit reads pass 1 of every one of its heads and rows
                other = latest.get((u, (i + 1) % 2))
                if other is not None:
                    st.wait_event(other)
                run_staged(prep, S.KVBM_STAGE_PASS2, ws, units=(u, u + 1), stream=st)
        if direct:
            # one element of each through torch on the copy stream, after every
            # piece: the host allocator then keeps the pinned blocks of q and k
            # until the copies end, as it does for its own asynchronous copies
            with torch.cuda.stream(copy):
                qd[-1, -1, -1, -1:].copy_(q[-1, -1, -1, -1:], non_blocking=True)
                kd[-1, -1, -1, -1:].copy_(k[-1, -1, -1, -1:], non_blocking=True)
        compute.wait_stream(side)
        run_staged(prep, S.KVBM_STAGE_REDUCE, ws, out=out, stream=compute)
        for t in (qd, kd, ws) + tuple(x for x in (am, qm) if x is not None):
            t.record_stream(side)
        # qd/kd were written on the copy stream: tell the allocator before they are freed
        qd.record_stream(copy)
        kd.record_stream(copy)
        return out


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
    """A prepared problem whose k comes from a paged cache (``prep.opts.paged``)."""

    def __init__(self, prep: _Prepared, kv, keep):
        self.prep = prep
        self.kv = kv
        self.keep = keep


def make_paged_problem(q, k_cache, block_table, attn_mask=None, causal=False, block_size=64, scale=None,
                       causal_skip=True, query_mask=None, units=None, seq_lens=None, cu_seqlens=None,
                       max_seqlen=None, per_sequence=False, method=None) -> _PagedPrepared:
    """Validate a paged call and build its C structs.

    ``k_cache`` is ``[num_pages, page_size, H_kv, D]`` (any strides, the dtype
    of ``q``); ``block_table`` is ``[B, max_pages]`` of page ids (converted to
    int32): key ``n`` of sequence ``b`` is ``k_cache[block_table[b, n // P], n % P]``.
    ``q`` is ``[B, H_q, N, D]`` (every sequence N long, or ``seq_lens[b]``
    long), or packed ``[T, H_q, D]`` with ``cu_seqlens`` (as ``block_mass_varlen``).
    """
    if not all(isinstance(t, torch.Tensor) for t in (q, k_cache, block_table)):
        raise TypeError("q, k_cache and block_table must be torch tensors")
    packed = cu_seqlens is not None
    if (q.dim() != (3 if packed else 4)) or k_cache.dim() != 4:
        raise ValueError(f"q must be [B, H_q, N, D] ([T, H_q, D] with cu_seqlens) and k_cache "
                         f"[num_pages, page_size, H_kv, D], got {tuple(q.shape)} and {tuple(k_cache.shape)}")
    num_pages, page_size, Hkv, Dk = k_cache.shape
    D = q.shape[-1]
    B = (cu_seqlens.shape[0] - 1) if packed else q.shape[0]
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
    if packed:
        if max_seqlen is None:
            cu_h = cu_seqlens.detach().to("cpu", torch.int64)
            max_seqlen = int((cu_h[1:] - cu_h[:-1]).max())
        N = int(max_seqlen)
        qs = (0, q.stride(1), q.stride(0), q.stride(2))
    else:
        N = q.shape[2]
        qs = q.stride()
    if block_table.shape[1] * page_size < N:
        raise ValueError(f"block_table covers {block_table.shape[1] * page_size} keys < N={N}")
    table = block_table.to(torch.int32)
    if table.stride(1) != 1:
        table = table.contiguous()
    Hq = q.shape[1]
    # k in the problem is ignored (the options carry the cache); any non-null pointer
    prep = _fill_problem(q.data_ptr(), qs, k_cache.data_ptr(), (0, 0, 0, 0), q.dtype, B, Hq, Hkv, N, D, q.device,
                         [q], attn_mask, causal, block_size, scale, causal_skip, query_mask, units)
    kv = _lib.PagedKV()
    kv.k_cache = k_cache.data_ptr()
    for i in range(4):
        kv.cache_stride[i] = k_cache.stride(i)
    kv.num_pages, kv.page_size = num_pages, page_size
    kv.block_table = table.data_ptr()
    kv.block_table_stride = table.stride(0)
    kv.max_pages = table.shape[1]
    prep.keep += [k_cache, table, kv]
    prep.options().paged = ctypes.pointer(kv)
    _set_ragged(prep, q.device, seq_lens=seq_lens, cu_seqlens=cu_seqlens, total=q.shape[0] if packed else 0,
                per_sequence=per_sequence)
    _set_method(prep, method)
    _validate_ex(prep)
    return _PagedPrepared(prep, kv, [k_cache, table])


def paged_workspace_bytes(pp: _PagedPrepared) -> int:
    return workspace_bytes(pp.prep)


def run_paged(pp: _PagedPrepared, out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
              stream: torch.cuda.Stream | None = None, lse: torch.Tensor | None = None) -> torch.Tensor:
    """Launch a prepared paged problem (page gather, then the dense kernels) on ``stream``."""
    return run_prepared(pp.prep, out=out, workspace=workspace, stream=stream, lse=lse)


def block_mass_paged(q, k_cache, block_table, attn_mask=None, causal=False, block_size=64, scale=None,
                     causal_skip=True, query_mask=None, *, seq_lens=None, cu_seqlens=None, max_seqlen=None,
                     per_sequence=False, units=None, out=None, workspace=None, lse=None, method=None):
    """``block_mass_b200`` with keys read from a paged KV cache.

    ``k_cache [num_pages, page_size, H_kv, D]`` and ``block_table [B,
    max_pages]`` (page ids) on the device of ``q``: ``[B, H_q, N, D]``
    (optionally ``seq_lens [B]``), or packed ``[T, H_q, D]`` with
    ``cu_seqlens [B + 1]``.  Other arguments as ``block_mass_b200``;
    ``block_size == page_size`` gives one bucket per page.  The result has the
    same bits as the dense call on the keys the table names.  A page id
    outside ``[0, num_pages)`` is not read (its keys count as zero vectors);
    ``check_device_errors()`` reports it.  Table entries past a sequence's
    length are never read.  ``method`` as for ``make_problem``.
    """
    if not (q.is_cuda and k_cache.is_cuda):
        raise ValueError("block_mass_paged needs CUDA tensors (there is no CPU path)")
    pp = make_paged_problem(q, k_cache, block_table, attn_mask=attn_mask, causal=causal, block_size=block_size,
                            scale=scale, causal_skip=causal_skip, query_mask=query_mask, units=units,
                            seq_lens=seq_lens, cu_seqlens=cu_seqlens, max_seqlen=max_seqlen,
                            per_sequence=per_sequence, method=method)
    return run_paged(pp, out=out, workspace=workspace, lse=lse)


def block_mass_varlen(q, k, cu_seqlens, max_seqlen=None, attn_mask=None, causal=False, block_size=64,
                      scale=None, causal_skip=True, query_mask=None, *, per_sequence=False, units=None, out=None,
                      workspace=None, lse=None, method=None):
    """Block mass of a packed (varlen) batch, as FlashAttention's varlen layout.

    ``q [T, H_q, D]``, ``k [T, H_kv, D]``; sequence ``b`` is rows
    ``[cu_seqlens[b], cu_seqlens[b + 1])`` (``cu_seqlens [B + 1]`` int32 on the
    device).  ``max_seqlen`` (host int; read from ``cu_seqlens`` when omitted,
    which synchronises) sets ``N``: the output is ``[ceil(N / block_size)]``
    summed over sequences, or ``[B, ceil(N / block_size)]`` with
    ``per_sequence``.  Each sequence contributes exactly what the reference
    computes for it alone.  ``lse`` is ``[H_q, T]``; ``method`` as for
    ``make_problem``.
    """
    if not (q.is_cuda and k.is_cuda):
        raise ValueError("block_mass_varlen needs CUDA tensors (there is no CPU path)")
    prep = make_varlen_problem(q, k, cu_seqlens, max_seqlen=max_seqlen, attn_mask=attn_mask, causal=causal,
                               block_size=block_size, scale=scale, causal_skip=causal_skip,
                               query_mask=query_mask, units=units, per_sequence=per_sequence, method=method)
    return run_prepared(prep, out=out, workspace=workspace, lse=lse)


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
