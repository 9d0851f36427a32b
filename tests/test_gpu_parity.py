"""GPU parity: the CUDA kernels (through the C ABI) against the reference's
golden outputs and the CPU oracle.

Tolerances (max relative error per bucket, |a-b| / max(|b|, 1e-6)):
  * fp64 inputs: 1e-9 against the reference's fp64 output;
  * fp32 inputs: 2e-5 against the reference's fp32 output;
  * bf16/fp16 inputs: 1e-3 against the reference fed the same values upcast
    to fp32.
Sum rule sum(mass) = B * H_q * (#rows that keep a key) to 1e-5 relative;
causal_skip on/off and repeated runs bit-identical (torch.equal).
"""

import numpy as np
import pytest
import torch

from conftest import load_golden
from _helpers import case_inputs, checksum_ok, max_rel
from oracle import block_mass_np as orc

import kvblockmass_b200 as kb
from kvblockmass_b200.workloads import WORKLOADS, make_inputs

pytestmark = pytest.mark.gpu

TOL = {torch.float64: 1e-9, torch.float32: 2e-5, torch.bfloat16: 1e-3, torch.float16: 1e-3}


def run(q, k, **kw):
    out = kb.block_mass_b200(q, k, **kw)
    torch.cuda.synchronize()
    return out


def oracle_for(q, k, **kw):
    """CPU oracle on the exact values the kernel saw (upcast to fp32/fp64)."""
    qn = q.detach().cpu()
    kn = k.detach().cpu()
    if qn.dtype in (torch.bfloat16, torch.float16):
        qn, kn = qn.float(), kn.float()
    km = kw.pop("attn_mask", None)
    qm = kw.pop("query_mask", None)
    return orc.block_mass_stream(qn.numpy(), kn.numpy(),
                                 attn_mask=None if km is None else km.cpu().numpy(),
                                 query_mask=None if qm is None else qm.cpu().numpy(), **kw)


# ------------------------------------------------------------ golden: small cases
@pytest.mark.parametrize("idx", range(22))
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32, torch.bfloat16])
def test_small_cases(cuda_device, small_cases, idx, dtype):
    c = small_cases[idx]
    q, k, mask = case_inputs(c)
    qd, kd = q.to(dtype).to(cuda_device), k.to(dtype).to(cuda_device)
    md = None if mask is None else mask.to(cuda_device)
    got = run(qd, kd, attn_mask=md, causal=c["causal"], block_size=c["block_size"])
    assert got.dtype == (torch.float64 if dtype == torch.float64 else torch.float32)
    assert got.shape == (len(c["mass_ref_fp64"]),)
    assert torch.isfinite(got).all()
    if dtype == torch.float64:
        want = c["mass_ref_fp64"]
    elif dtype == torch.float32:
        want = c["mass_ref_fp32"]
    else:
        want = oracle_for(qd, kd, attn_mask=md, causal=c["causal"], block_size=c["block_size"])
    assert max_rel(got.cpu().numpy(), want) < TOL[dtype], c["name"]
    # sum rule against the reference's fp64 total
    total = float(np.sum(c["mass_ref_fp64"]))
    assert abs(float(got.double().sum()) - total) <= 1e-5 * max(total, 1.0)


# ------------------------------------------------------------ golden: workloads
@pytest.mark.parametrize("name", ["cpu_ref_n2048", "gqa_n8192_fp32"])
def test_fp32_workloads_vs_reference(cuda_device, name):
    g = load_golden(name)
    w = WORKLOADS[name]
    q, k, _, _ = make_inputs(w)
    assert checksum_ok(q, g["q_checksum"]) and checksum_ok(k, g["k_checksum"])
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    a = run(qd, kd, causal=w.causal, block_size=w.block_size)
    b = run(qd, kd, causal=w.causal, block_size=w.block_size, causal_skip=False)
    c = run(qd, kd, causal=w.causal, block_size=w.block_size)
    assert torch.equal(a, b), "causal_skip on/off must be bit-identical"
    assert torch.equal(a, c), "repeated runs must be bit-identical"
    assert max_rel(a.cpu().numpy(), g["mass_ref_fp32"]) < 2e-5
    assert max_rel(a.cpu().numpy(), g["mass_ref_fp64"]) < 2e-5
    expect = w.B * w.Hq * w.N
    assert abs(float(a.double().sum()) - expect) <= 1e-5 * expect


@pytest.mark.parametrize("name", ["llama3_8b_n32k", "batched_masked_n16k"])
def test_bf16_workloads_vs_reference(cuda_device, name):
    g = load_golden(name)
    if g is None:
        pytest.skip(f"golden fixture {name}.json not generated")
    w = WORKLOADS[name]
    q, k, km, qm = make_inputs(w)
    assert checksum_ok(q, g["q_checksum"]) and checksum_ok(k, g["k_checksum"])
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    kmd = None if km is None else km.to(cuda_device)
    qmd = None if qm is None else qm.to(cuda_device)
    a = run(qd, kd, attn_mask=kmd, query_mask=qmd, causal=w.causal, block_size=w.block_size)
    assert max_rel(a.cpu().numpy(), g["mass_ref_fp32"]) < 1e-3
    alive = w.B * w.N if qm is None else int(qm.sum())
    expect = w.Hq * alive
    assert abs(float(a.double().sum()) - expect) <= 1e-5 * expect
    if w.causal:
        b = run(qd, kd, attn_mask=kmd, query_mask=qmd, causal=w.causal, block_size=w.block_size,
                causal_skip=False)
        assert torch.equal(a, b)


def test_dead_rows_contribute_exactly_zero(cuda_device):
    """Rows that keep nothing add exactly 0: masking them equals dropping them."""
    w = WORKLOADS["batched_masked_n16k"]
    q, k, km, qm = make_inputs(w, N=1024)
    qd, kd, kmd, qmd = q.to(cuda_device), k.to(cuda_device), km.to(cuda_device), qm.to(cuda_device)
    a = run(qd, kd, attn_mask=kmd, query_mask=qmd, block_size=w.block_size)
    # the same rows removed through an [B, N, N] pair mask
    pair = (km[None, None, :] & qm[:, :, None]).to(cuda_device)
    b = run(qd, kd, attn_mask=pair, block_size=w.block_size)
    assert max_rel(a.cpu().numpy(), b.cpu().numpy()) < 1e-5
    want = oracle_for(qd, kd, attn_mask=km, query_mask=qm, block_size=w.block_size)
    assert max_rel(a.cpu().numpy(), want) < 1e-3
    expect = w.Hq * int(qm.sum())
    assert abs(float(a.double().sum()) - expect) <= 1e-5 * expect


# ------------------------------------------------------------ masks and shapes
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("kind", ["keys", "pairs", "batch_keys", "batch_pairs", "query"])
@pytest.mark.parametrize("causal", [False, True])
def test_mask_kinds(cuda_device, dtype, kind, causal):
    g = torch.Generator().manual_seed(101)
    B, Hq, Hkv, N, D = 2, 4, 2, 333, 64
    q = torch.randn(B, Hq, N, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    kw = {}
    if kind == "keys":
        kw["attn_mask"] = torch.rand(N, generator=g) > 0.25
    elif kind == "pairs":
        kw["attn_mask"] = torch.rand(N, N, generator=g) > 0.4
    elif kind == "batch_keys":
        kw["attn_mask"] = torch.rand(B, 1, N, generator=g) > 0.25
    elif kind == "batch_pairs":
        kw["attn_mask"] = torch.rand(B, N, N, generator=g) > 0.4
    else:
        kw["query_mask"] = torch.rand(B, N, generator=g) > 0.3
    dev = {n: v.to(cuda_device) for n, v in kw.items()}
    got = run(q.to(cuda_device), k.to(cuda_device), causal=causal, block_size=48, **dev)
    want = oracle_for(q, k, causal=causal, block_size=48, **kw)
    assert max_rel(got.cpu().numpy(), want) < TOL[dtype]


@pytest.mark.parametrize("N", [1, 2, 63, 64, 65, 127, 128, 129, 255, 257, 1000])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_ragged_lengths(cuda_device, N, dtype):
    g = torch.Generator().manual_seed(N)
    q = torch.randn(1, 4, N, 128, generator=g).to(dtype)
    k = torch.randn(1, 2, N, 128, generator=g).to(dtype)
    for causal in (True, False):
        got = run(q.to(cuda_device), k.to(cuda_device), causal=causal, block_size=64)
        want = oracle_for(q, k, causal=causal, block_size=64)
        assert max_rel(got.cpu().numpy(), want) < TOL[dtype], (N, causal)


@pytest.mark.parametrize("D", [8, 16, 32, 64, 96, 128, 192, 256])
def test_head_dims(cuda_device, D):
    g = torch.Generator().manual_seed(D)
    q = torch.randn(1, 2, 300, D, generator=g)
    k = torch.randn(1, 1, 300, D, generator=g)
    for dtype in (torch.float32, torch.bfloat16):
        got = run(q.to(dtype).to(cuda_device), k.to(dtype).to(cuda_device), causal=True, block_size=32)
        want = oracle_for(q.to(dtype), k.to(dtype), causal=True, block_size=32)
        assert max_rel(got.cpu().numpy(), want) < TOL[dtype]


def test_strided_inputs_match_contiguous(cuda_device):
    """q/k as views of [B, N, H, D] storage (the common KV layout) give the same bits."""
    g = torch.Generator().manual_seed(3)
    for dtype in (torch.float32, torch.bfloat16):
        qs = torch.randn(2, 500, 8, 128, generator=g).to(dtype).to(cuda_device)
        ks = torch.randn(2, 500, 2, 128, generator=g).to(dtype).to(cuda_device)
        qv, kv = qs.transpose(1, 2), ks.transpose(1, 2)
        a = run(qv, kv, causal=True, block_size=64)
        b = run(qv.contiguous(), kv.contiguous(), causal=True, block_size=64)
        assert torch.equal(a, b)


def test_units_shard_and_sum(cuda_device):
    """Mass is a sum over (batch, kv-head) units: shards add up to the whole."""
    g = torch.Generator().manual_seed(9)
    q = torch.randn(2, 8, 700, 64, generator=g).to(torch.bfloat16).to(cuda_device)
    k = torch.randn(2, 2, 700, 64, generator=g).to(torch.bfloat16).to(cuda_device)
    full = run(q, k, causal=True, block_size=64)
    parts = [run(q, k, causal=True, block_size=64, units=(u, u + 1)) for u in range(4)]
    assert max_rel(sum(p.double() for p in parts).cpu().numpy(), full.double().cpu().numpy()) < 1e-6
    u2 = run(q, k, causal=True, block_size=64, units=(1, 3))
    assert max_rel(u2.cpu().numpy(), (parts[1].double() + parts[2].double()).cpu().numpy()) < 1e-6


def test_pass1_unit_groups_cover_every_tile(cuda_device):
    """Pass 1 runs its CTAs in groups of units whose k fits in 32 MiB: at
    N=65536, D=128 bf16 (16 MiB of k per unit) 3 units form the uneven groups
    {0, 1} and {2}.  Every (unit, head, query tile) must still get its row LSE:
    the whole call equals the sum of one-unit calls, and the sum rule holds."""
    g = torch.Generator().manual_seed(23)
    N = 65536
    q = torch.randn(1, 6, N, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    k = torch.randn(1, 3, N, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    full = run(q, k, causal=True, block_size=64)
    parts = [run(q, k, causal=True, block_size=64, units=(u, u + 1)) for u in range(3)]
    assert max_rel(sum(p.double() for p in parts).cpu().numpy(), full.double().cpu().numpy()) < 1e-6
    expect = 6 * N
    assert abs(float(full.double().sum()) - expect) <= 1e-5 * expect
    nc = run(q, k, causal=False, block_size=64)
    assert abs(float(nc.double().sum()) - expect) <= 1e-5 * expect


def test_drop_in_entry_points(cuda_device):
    g = torch.Generator().manual_seed(31)
    q = torch.randn(2, 4, 256, 32, generator=g, dtype=torch.float64).float()
    k = torch.randn(2, 2, 256, 32, generator=g, dtype=torch.float64).float()
    want = oracle_for(q, k, causal=True, block_size=64)
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    for fn in (lambda: kb.block_mass_triton(qd, kd, causal=True, block_size=64),
               lambda: kb.block_mass(qd, kd, causal=True, block_size=64),
               lambda: kb.block_mass_b200(q, k, causal=True, block_size=64, device="cuda",
                                          query_chunk=128)):
        got = fn()
        assert got.is_cuda
        assert max_rel(got.cpu().numpy(), want) < 2e-5


def test_peak_memory_n4096(cuda_device):
    """O(N) workspace: N=4096 must not allocate anything like an [N, N] matrix
    (the reference's bound, tests/test_triton.py:85-103)."""
    g = torch.Generator().manual_seed(47)
    q = torch.randn(1, 8, 4096, 64, generator=g).to(cuda_device)
    k = torch.randn(1, 2, 4096, 64, generator=g).to(cuda_device)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    run(q, k, causal=True, block_size=64)
    peak = (torch.cuda.max_memory_allocated() - base) / 2**20
    assert peak < 64, f"peak {peak:.1f} MiB"


def test_determinism_bf16(cuda_device):
    g = torch.Generator().manual_seed(77)
    q = torch.randn(1, 8, 3000, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    k = torch.randn(1, 2, 3000, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    a = run(q, k, causal=True, block_size=64)
    b = run(q, k, causal=True, block_size=64, causal_skip=False)
    c = run(q, k, causal=True, block_size=64)
    assert torch.equal(a, b) and torch.equal(a, c)


# ------------------------------------------------------------ Llama-3-70B, N=131072
def test_llama3_70b_vs_reference(cuda_device):
    """The Llama-3-70B long-context shape (N=131072, block 256, 1% x8 sink keys)
    against the reference's own output: ``block_mass_reference`` run on a GPU
    once per kv-head group (``tests/golden/gen_golden_70b.py``).  The whole
    problem, and each (batch, kv-head) unit alone as a multi-GPU shard computes
    it, within 1e-3 per bucket of the fp32 reference (and of the fp64 one);
    the sum rule, causal_skip on/off and repeats with the same bits, and the
    units adding up to the whole."""
    from kvblockmass_b200.workloads import make_unit_inputs

    g = load_golden("llama3_70b_n128k")
    if g is None:
        pytest.skip("golden fixture llama3_70b_n128k.json not generated")
    w = WORKLOADS["llama3_70b_n128k"]
    G = w.G
    q, k = make_unit_inputs(w, 0, w.units)
    for rec in g["units"]:
        u = rec["unit"]
        assert checksum_ok(q[:, u * G:(u + 1) * G], rec["q_checksum"]), u
        assert checksum_ok(k[:, u:u + 1], rec["k_checksum"]), u
    q, k = q.to(cuda_device), k.to(cuda_device)
    a = run(q, k, causal=True, block_size=w.block_size)
    assert a.shape == (w.num_blocks,) and torch.isfinite(a).all() and bool((a >= 0).all())
    assert max_rel(a.cpu().numpy(), g["mass_ref_fp32"]) < 1e-3
    if "mass_ref_fp64" in g:
        assert max_rel(a.cpu().numpy(), g["mass_ref_fp64"]) < 1e-3
    expect = w.Hq * w.N
    assert abs(float(a.double().sum()) - expect) <= 1e-5 * expect
    b = run(q, k, causal=True, block_size=w.block_size, causal_skip=False)
    c = run(q, k, causal=True, block_size=w.block_size)
    assert torch.equal(a, b) and torch.equal(a, c)
    acc = torch.zeros(w.num_blocks, dtype=torch.float64, device=cuda_device)
    for rec in g["units"]:
        u = rec["unit"]
        m = run(q, k, causal=True, block_size=w.block_size, units=(u, u + 1))
        assert max_rel(m.cpu().numpy(), rec["mass_ref_fp32"]) < 1e-3, u
        acc += m.double()
    assert max_rel(acc.cpu().numpy(), a.double().cpu().numpy()) < 1e-6


def test_llama3_70b_prefix_vs_oracle(cuda_device):
    """Numerics on the 70B data (1% x8 sink keys, block 256) against the oracle:
    under causality the first N' rows/keys form a problem of their own."""
    from kvblockmass_b200.workloads import make_unit_inputs

    w = WORKLOADS["llama3_70b_n128k"]
    q, k = make_unit_inputs(w, 3, 4, device=cuda_device, N=4096)
    got = run(q, k, causal=True, block_size=w.block_size)
    want = oracle_for(q, k, causal=True, block_size=w.block_size)
    assert max_rel(got.cpu().numpy(), want) < 1e-3


@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("shape,dtype", [((1, 32, 8, 3000, 128), torch.bfloat16),
                                         ((1, 8, 2, 9000, 128), torch.bfloat16),  # unit 0 by query rows
                                         ((2, 4, 2, 4200, 32), torch.float64),    # SIMT, rows
                                         ((3, 8, 2, 777, 64), torch.bfloat16),
                                         ((2, 8, 2, 900, 64), torch.float32),    # 3xTF32: per-piece tf32 split
                                         ((2, 4, 4, 500, 96), torch.float32),    # 3xTF32, K-block slots
                                         ((2, 4, 2, 400, 160), torch.float32)])  # SIMT
def test_host_inputs_give_the_device_call_bits(cuda_device, shape, dtype, pinned):
    """Host q/k with device='cuda' are copied piece by piece (unit 0 by query
    rows or by heads, then unit by unit) while earlier pieces compute, as staged
    calls into one workspace with one reduce: the result has the bits of the
    device-input call.  Pageable tensors go through pinned bounce buffers."""
    B, Hq, Hkv, N, D = shape
    g = torch.Generator().manual_seed(17)
    q = torch.randn(B, Hq, N, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    if pinned:
        q, k = q.pin_memory(), k.pin_memory()
    km = torch.rand(N, generator=g) > 0.1
    qm = torch.rand(B, N, generator=g) > 0.1
    a = kb.block_mass_b200(q, k, attn_mask=km, query_mask=qm, causal=True, block_size=64, device=cuda_device)
    b = run(q.to(cuda_device), k.to(cuda_device), attn_mask=km.to(cuda_device), query_mask=qm.to(cuda_device),
            causal=True, block_size=64)
    torch.cuda.synchronize()
    assert a.is_cuda
    assert torch.equal(a, b)
    c = kb.block_mass_b200(q, k, attn_mask=km, query_mask=qm, causal=True, block_size=64, device=cuda_device)
    assert torch.equal(a, c)


@pytest.mark.parametrize("N", [700, 5000])
def test_host_inputs_with_strided_rows(cuda_device, N):
    """Pinned q/k whose rows are not contiguous per head (a [B, N, H, D] buffer
    viewed as [B, H, N, D]) take the per-piece tensor copies instead of the
    2-D copies; the result is still the device-input call's bits."""
    B, Hq, Hkv, D = 1, 8, 2, 128
    g = torch.Generator().manual_seed(N)
    q = torch.randn(B, N, Hq, D, generator=g).to(torch.bfloat16).pin_memory().transpose(1, 2)
    k = torch.randn(B, N, Hkv, D, generator=g).to(torch.bfloat16).pin_memory().transpose(1, 2)
    assert q.is_pinned() and q.stride(2) != D
    a = kb.block_mass_b200(q, k, causal=True, block_size=64, device=cuda_device)
    b = run(q.to(cuda_device), k.to(cuda_device), causal=True, block_size=64)
    assert torch.equal(a, b)


@pytest.mark.parametrize("mask_kind", ["batch_pairs", "pairs", "none"])
def test_host_inputs_with_pair_masks(cuda_device, mask_kind):
    """Pair masks are packed once before the pieces run (KVBM_STAGE_MASKS); every
    mask form gives the device-input call's bits."""
    B, Hq, Hkv, N, D = 2, 8, 2, 1000, 64
    g = torch.Generator().manual_seed(29)
    q = torch.randn(B, Hq, N, D, generator=g).to(torch.bfloat16).pin_memory()
    k = torch.randn(B, Hkv, N, D, generator=g).to(torch.bfloat16).pin_memory()
    if mask_kind == "batch_pairs":
        am = torch.rand(B, N, N, generator=g) > 0.2
    elif mask_kind == "pairs":
        am = torch.rand(N, N, generator=g) > 0.2
    else:
        am = None
    qm = torch.rand(B, N, generator=g) > 0.1
    a = kb.block_mass_b200(q, k, attn_mask=am, query_mask=qm, causal=True, block_size=64, device=cuda_device)
    b = run(q.to(cuda_device), k.to(cuda_device), attn_mask=None if am is None else am.to(cuda_device),
            query_mask=qm.to(cuda_device), causal=True, block_size=64)
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float32, 64), (torch.float32, 96),
                                     (torch.float32, 160), (torch.float64, 32)])
@pytest.mark.parametrize("mask", ["none", "pairs"])
def test_staged_pieces_on_two_streams(cuda_device, dtype, D, mask):
    """kvbm_options.stages / run ranges through the C ABI: pass 1 per (unit,
    head range) and pass 2 per unit, out of order on two streams, into one
    workspace, then one reduce: the bits of one whole call, on every kernel
    path, also with the LSE input."""
    from kvblockmass_b200 import _lib
    from kvblockmass_b200.ops import run_staged

    S = _lib
    B, Hq, Hkv, N = 2, 6, 2, 700
    G = Hq // Hkv
    g = torch.Generator().manual_seed(D)
    q = torch.randn(B, Hq, N, D, generator=g).to(dtype).to(cuda_device)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype).to(cuda_device)
    am = (torch.rand(B, N, N, generator=g) > 0.3).to(cuda_device) if mask == "pairs" else None
    whole = run(q, k, attn_mask=am, causal=True, block_size=32)
    prep = kb.make_problem(q, k, attn_mask=am, causal=True, block_size=32)
    ws = torch.full((kb.workspace_bytes(prep),), 0xFF, dtype=torch.uint8, device=cuda_device)
    out = torch.empty_like(whole)
    s0 = torch.cuda.current_stream(cuda_device)
    s1 = torch.cuda.Stream(device=cuda_device)
    run_staged(prep, S.KVBM_STAGE_MASKS, ws, stream=s0)
    s1.wait_stream(s0)
    U = B * Hkv
    done = {}
    for u in reversed(range(U)):              # units in reverse, heads split in two pieces
        for i, (h0, h1) in enumerate(((0, 1), (1, G))):
            st = s0 if (u + i) % 2 else s1
            run_staged(prep, S.KVBM_STAGE_PASS1, ws, units=(u, u + 1), heads=(h0, h1), stream=st)
            e = torch.cuda.Event()
            e.record(st)
            done.setdefault(u, []).append(e)
    for u in range(U):
        st = s0 if u % 2 else s1
        for e in done[u]:
            st.wait_event(e)
        run_staged(prep, S.KVBM_STAGE_PASS2, ws, units=(u, u + 1), stream=st)
    s0.wait_stream(s1)
    run_staged(prep, S.KVBM_STAGE_REDUCE, ws, out=out, stream=s0)
    torch.cuda.synchronize()
    assert torch.equal(out, whole)
    # a staged call with every stage is the whole call
    out2 = torch.empty_like(whole)
    run_staged(prep, 0, ws, out=out2)
    torch.cuda.synchronize()
    assert torch.equal(out2, whole)


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 64), (torch.float64, 32),
                                     (torch.float32, 160)])
@pytest.mark.parametrize("causal,skip", [(True, True), (True, False), (False, True)])
def test_staged_row_pieces(cuda_device, dtype, D, causal, skip):
    """kvbm_options.run_row_begin/end: pass 1 in pieces of query rows (in any
    order, on two streams, rows of one piece ending at N or on a 128-row
    boundary), then pass 2 and the reduce: the bits of one whole call."""
    from kvblockmass_b200 import _lib
    from kvblockmass_b200.ops import run_staged

    B, Hq, Hkv, N = 2, 4, 2, 1000
    g = torch.Generator().manual_seed(D + 7)
    q = torch.randn(B, Hq, N, D, generator=g).to(dtype).to(cuda_device)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype).to(cuda_device)
    km = (torch.rand(N, generator=g) > 0.1).to(cuda_device)
    kw = dict(attn_mask=km, causal=causal, causal_skip=skip, block_size=48)
    whole = run(q, k, **kw)
    prep = kb.make_problem(q, k, **kw)
    assert kb.kernel_path(prep) in (0, 1)
    ws = torch.full((kb.workspace_bytes(prep),), 0xFF, dtype=torch.uint8, device=cuda_device)
    out = torch.empty_like(whole)
    s0 = torch.cuda.current_stream(cuda_device)
    s1 = torch.cuda.Stream(device=cuda_device)
    s1.wait_stream(s0)
    chunks = [(768, 1000), (0, 256), (256, 768)]
    for u in range(B * Hkv):
        for i, rows in enumerate(chunks):
            st = s0 if (u + i) % 2 else s1
            run_staged(prep, _lib.KVBM_STAGE_PASS1, ws, units=(u, u + 1), rows=rows, stream=st)
    s0.wait_stream(s1)
    run_staged(prep, _lib.KVBM_STAGE_PASS2, ws, stream=s0)
    run_staged(prep, _lib.KVBM_STAGE_REDUCE, ws, out=out, stream=s0)
    torch.cuda.synchronize()
    assert torch.equal(out, whole)


def test_staged_row_range_is_refused_on_the_tf32_path(cuda_device):
    """The 3xTF32 path converts whole rows of q/k to tf32 pairs in pass 1, so a
    row range there is refused before any launch."""
    from kvblockmass_b200 import _lib
    from kvblockmass_b200.ops import run_staged

    q = torch.randn(1, 4, 512, 64, device=cuda_device)
    k = torch.randn(1, 2, 512, 64, device=cuda_device)
    prep = kb.make_problem(q, k, causal=True, block_size=64)
    assert kb.kernel_path(prep) == 2
    ws = torch.empty(kb.workspace_bytes(prep), dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ValueError, match="sizes"):
        run_staged(prep, _lib.KVBM_STAGE_PASS1, ws, units=(0, 1), rows=(0, 256))


def test_causal_skip_is_engaged(cuda_device):
    """causal_skip must skip work, not only give the same bits (the reference's
    engagement test, tests/test_reference.py:148-158 and :189-215, records the
    key extents its chunks visit).  Skipping the tiles above the diagonal
    halves a causal step: the time with the skip must be well under the time
    without it, on the same inputs."""
    g = torch.Generator().manual_seed(90)
    q = torch.randn(1, 16, 8192, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    k = torch.randn(1, 4, 8192, 128, generator=g).to(torch.bfloat16).to(cuda_device)

    def timed(skip):
        prep = kb.make_problem(q, k, causal=True, block_size=64, causal_skip=skip)
        ws = torch.empty(kb.workspace_bytes(prep), dtype=torch.uint8, device=cuda_device)
        out = torch.empty(prep.nb, device=cuda_device)
        for _ in range(3):
            kb.run_prepared(prep, out=out, workspace=ws)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(10):
            kb.run_prepared(prep, out=out, workspace=ws)
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b), out.clone()

    t_off, m_off = timed(False)
    t_on, m_on = timed(True)
    assert torch.equal(m_on, m_off)
    assert t_on < 0.75 * t_off, (t_on, t_off)


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 192), (torch.bfloat16, 256), (torch.float16, 256)])
def test_wide_heads_on_tensor_cores(cuda_device, dtype, D):
    """D = 192 / 256 run the tcgen05 kernels (one CTA per SM): parity with every
    mask kind and the LSE input, causal_skip on/off with the same bits."""
    g = torch.Generator().manual_seed(D + 7)
    B, Hq, Hkv, N = 2, 8, 2, 700
    q = torch.randn(B, Hq, N, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    assert kb.kernel_path(kb.make_problem(qd, kd, causal=True)) == 1
    km = torch.rand(N, generator=g) > 0.2
    pm = torch.rand(N, N, generator=g) > 0.3
    for causal in (True, False):
        for mask in (None, km, pm):
            dm = None if mask is None else mask.to(cuda_device)
            got = run(qd, kd, attn_mask=dm, causal=causal, block_size=64)
            want = oracle_for(q, k, attn_mask=mask, causal=causal, block_size=64)
            assert max_rel(got.cpu().numpy(), want) < 1e-3, (causal, None if mask is None else mask.dim())
    a = run(qd, kd, causal=True, block_size=64)
    assert torch.equal(a, run(qd, kd, causal=True, block_size=64, causal_skip=False))
    # the LSE input gives the mass of the two-pass call
    s_ = (q.float() @ k.float().repeat_interleave(Hq // Hkv, dim=1).transpose(-1, -2)) / D ** 0.5
    lse = s_.masked_fill(~torch.ones(N, N, dtype=torch.bool).tril(), float("-inf")).logsumexp(-1)
    b = kb.block_mass_b200(qd, kd, causal=True, block_size=64, lse=lse.to(cuda_device))
    assert max_rel(b.cpu().numpy(), a.cpu().numpy()) < 2e-3
    # ragged lengths
    lens = torch.tensor([N, 333], dtype=torch.int32, device=cuda_device)
    r = kb.block_mass_b200(qd, kd, causal=True, block_size=64, seq_lens=lens, per_sequence=True)
    alone = run(qd[1:, :, :333], kd[1:, :, :333], causal=True, block_size=64)
    assert max_rel(r[1, :alone.numel()].double().cpu().numpy(), alone.double().cpu().numpy()) < 1e-6


@pytest.mark.parametrize("dtype,D,path", [
    (torch.bfloat16, 8, 1), (torch.bfloat16, 40, 1), (torch.float16, 80, 1), (torch.bfloat16, 96, 1),
    (torch.bfloat16, 112, 1), (torch.float16, 160, 1), (torch.bfloat16, 224, 1),
    (torch.float32, 4, 2), (torch.float32, 12, 2), (torch.float32, 48, 2), (torch.float32, 60, 2),
    (torch.float32, 100, 2), (torch.float32, 128, 2), (torch.float32, 132, 0),
])
def test_padded_head_dims_on_tensor_cores(cuda_device, dtype, D, path):
    """Head dims between the kernels' 64/128/192/256 (and 32/64 for fp32) run the
    next larger tensor-core configuration: the tensor map has the real extent,
    and its zero fill makes the padding columns add exact zeros."""
    g = torch.Generator().manual_seed(D + 100)
    q = torch.randn(2, 8, 500, D, generator=g).to(dtype)
    k = torch.randn(2, 2, 500, D, generator=g).to(dtype)
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    assert kb.kernel_path(kb.make_problem(qd, kd, causal=True)) == path
    for causal in (True, False):
        got = run(qd, kd, causal=causal, block_size=64)
        want = oracle_for(q, k, causal=causal, block_size=64)
        assert max_rel(got.cpu().numpy(), want) < TOL[dtype], causal


def test_head_dim_view_reads_no_padding(cuda_device):
    """A [..., :96] view of a wider tensor: the columns past 96 are never read
    (they hold NaN here), and the bits equal those of a contiguous copy."""
    g = torch.Generator().manual_seed(5)
    qw = torch.randn(1, 8, 600, 128, generator=g).to(torch.bfloat16)
    kw = torch.randn(1, 2, 600, 128, generator=g).to(torch.bfloat16)
    qw[..., 96:] = float("nan")
    kw[..., 96:] = float("nan")
    qv, kv = qw.to(cuda_device)[..., :96], kw.to(cuda_device)[..., :96]
    assert kb.kernel_path(kb.make_problem(qv, kv, causal=True)) == 1
    a = run(qv, kv, causal=True, block_size=64)
    b = run(qv.contiguous(), kv.contiguous(), causal=True, block_size=64)
    assert torch.isfinite(a).all() and torch.equal(a, b)


@pytest.mark.parametrize("mask", [None, "keys", "pairs"])
def test_fp32_d128_on_tensor_cores(cuda_device, mask):
    """fp32 at D = 128 runs the 3xTF32 tensor-core kernels (kernel path 2), the
    streamed operand one 128-byte K-block per ring slot: parity at the fp32
    tolerance with the oracle and with the reference's own fp32 golden
    (small case d128_n257), causal_skip on/off with the same bits."""
    g = torch.Generator().manual_seed(128)
    B, Hq, Hkv, N, D = 2, 8, 2, 1500, 128
    q = torch.randn(B, Hq, N, D, generator=g)
    k = torch.randn(B, Hkv, N, D, generator=g)
    qd, kd = q.to(cuda_device), k.to(cuda_device)
    assert kb.kernel_path(kb.make_problem(qd, kd, causal=True)) == 2
    m = None
    if mask == "keys":
        m = torch.rand(N, generator=g) > 0.2
    elif mask == "pairs":
        m = torch.rand(N, N, generator=g) > 0.3
    md = None if m is None else m.to(cuda_device)
    for causal in (True, False):
        got = run(qd, kd, attn_mask=md, causal=causal, block_size=64)
        want = oracle_for(q, k, attn_mask=m, causal=causal, block_size=64)
        assert max_rel(got.cpu().numpy(), want) < 2e-5, causal
    a = run(qd, kd, attn_mask=md, causal=True, block_size=64)
    assert torch.equal(a, run(qd, kd, attn_mask=md, causal=True, block_size=64, causal_skip=False))


def test_fp32_d128_reference_golden(cuda_device, small_cases):
    c = next(x for x in small_cases if x["name"] == "d128_n257")
    q, k, mask = case_inputs(c)
    qd, kd = q.float().to(cuda_device), k.float().to(cuda_device)
    assert kb.kernel_path(kb.make_problem(qd, kd, causal=True)) == 2
    got = run(qd, kd, causal=c["causal"], block_size=c["block_size"])
    assert max_rel(got.cpu().numpy(), c["mass_ref_fp32"]) < 2e-5
