"""Multi-rank host logic over ``gloo`` on CPU (world size 2), no GPU.

The per-shard kernel call is replaced by the CPU oracle, so these tests cover
the unit partition, the shard slicing (masks included), both reduction modes
and failure behaviour; the GPU kernels themselves are covered by the parity
tests and by the multi-GPU bench.
"""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent

from kvblockmass_b200.distributed import partition_units, unit_segments  # noqa: E402


def test_partition_units():
    assert partition_units(8, 8) == [(i, i + 1) for i in range(8)]
    assert partition_units(8, 3) == [(0, 3), (3, 6), (6, 8)]
    assert partition_units(2, 4) == [(0, 1), (1, 2), (2, 2), (2, 2)]
    assert partition_units(32, 8)[7] == (28, 32)


def test_unit_segments():
    assert unit_segments(0, 8, 8) == [(0, 0, 8)]
    assert unit_segments(3, 13, 8) == [(0, 3, 8), (1, 0, 5)]
    assert unit_segments(5, 5, 8) == []


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_fn(q, k, causal=False, block_size=64, scale=None, causal_skip=True, attn_mask=None,
               query_mask=None):
    from oracle.block_mass_np import block_mass_stream

    out = block_mass_stream(q.numpy(), k.numpy(), causal=causal, block_size=block_size, scale=scale,
                            causal_skip=causal_skip,
                            attn_mask=None if attn_mask is None else attn_mask.numpy(),
                            query_mask=None if query_mask is None else query_mask.numpy())
    return torch.from_numpy(np.asarray(out, dtype=np.float64))


def _inputs():
    g = torch.Generator().manual_seed(123)
    B, Hq, Hkv, N, D = 3, 6, 3, 150, 16
    q = torch.randn(B, Hq, N, D, generator=g, dtype=torch.float64)
    k = torch.randn(B, Hkv, N, D, generator=g, dtype=torch.float64)
    km = torch.rand(B, 1, N, generator=g) > 0.2
    qm = torch.rand(B, N, generator=g) > 0.1
    return q, k, km, qm


def _worker(rank, world, port, mode, out_path):
    sys.path.insert(0, str(ROOT / "kv-block-mass_b200"))
    sys.path.insert(0, str(ROOT))
    from datetime import timedelta

    import torch.distributed as dist

    from kvblockmass_b200.distributed import block_mass_sharded, shard_inputs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    q, k, km, qm = _inputs()
    if mode == "empty":  # one unit for two ranks: rank 1 has nothing to compute
        q, k, km, qm = q[:1, :2], k[:1, :1], km[:1], qm[:1]
    nb = (q.shape[2] + 31) // 32
    try:
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected rank failure before the reduce")
        shards = shard_inputs(q, k, rank, world, attn_mask=km, query_mask=qm)
        res = block_mass_sharded(shards, causal=True, block_size=32, num_blocks=nb,
                                 local_fn=_oracle_fn, deterministic=(mode == "det"),
                                 all_ranks=(mode in ("all", "empty")))
        torch.save({"rank": rank, "mass": res}, f"{out_path}.{rank}")
    except Exception as e:  # noqa: BLE001 - the test inspects the error text
        torch.save({"rank": rank, "error": f"{type(e).__name__}: {e}"}, f"{out_path}.{rank}")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(mode, tmp_path, world=2):
    port = _free_port()
    out = str(tmp_path / "res")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode is not None, "rank did not exit"
    return [torch.load(f"{out}.{r}") for r in range(world)]


def _expected():
    from oracle.block_mass_np import block_mass_stream

    q, k, km, qm = _inputs()
    return block_mass_stream(q.numpy(), k.numpy(), attn_mask=km.numpy(), query_mask=qm.numpy(),
                             causal=True, block_size=32)


@pytest.mark.parametrize("mode", ["reduce", "det", "all"])
def test_sharded_matches_full(tmp_path, mode):
    res = _run(mode, tmp_path)
    want = _expected()
    r0 = res[0]["mass"].double().numpy()
    np.testing.assert_allclose(r0, want, rtol=1e-6, atol=1e-6)
    if mode in ("det", "all"):
        assert torch.equal(res[0]["mass"], res[1]["mass"])


def test_rank_failure_surfaces_as_error(tmp_path):
    """A rank that raises before the reduce: the survivor's collective ends with an
    error within the process-group timeout instead of hanging."""
    res = _run("fail", tmp_path)
    assert "injected rank failure" in res[1]["error"]
    assert "error" in res[0], "rank 0 should see the missing peer as an error"


def test_rank_without_units_joins_the_collective(tmp_path):
    """More ranks than units: the empty rank contributes zeros, and every rank
    gets the float64 result that float64 inputs give (reference.py:77)."""
    from oracle.block_mass_np import block_mass_stream

    res = _run("empty", tmp_path)
    q, k, km, qm = _inputs()
    want = block_mass_stream(q[:1, :2].numpy(), k[:1, :1].numpy(), attn_mask=km[:1].numpy(),
                             query_mask=qm[:1].numpy(), causal=True, block_size=32)
    for r in res:
        assert "mass" in r, r.get("error")
        assert r["mass"].dtype == torch.float64
        np.testing.assert_allclose(r["mass"].numpy(), want, rtol=1e-12, atol=1e-12)
