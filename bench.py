#!/usr/bin/env python
"""Benchmark: causal block-mass QK pairs/sec on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload NAME]

A step is one pass of the hot path (pass 1 row log-sum-exp, pass 2 per-key
partials, bucket reduce) over one synthetic batch of the Llama-3-8B attention
shape (B=1, H_q=32, H_kv=8, D=128, N=32768, block 64, causal, bf16), with
inputs resident in HBM.  With N GPUs (torchrun, one rank per GPU) every rank
owns one batch entry of that shape (weak scaling: per-GPU work is fixed) and
the per-rank mass vectors are combined by one NCCL reduce to rank 0 inside
each step.

Reported beside the device-timed value:
  e2e           the same metric through the public API (block_mass_b200 on
                pinned host tensors, device="cuda"), H2D of q/k and D2H of the
                mass inside the timed region;
  lse_input     the device-resident step with the row LSE supplied (one pass
                that needs no running max, and the two-pass method's pass 2
                alone beside it);
  paged         the device-resident step with k read from a paged cache
                (16-key pages in shuffled order + block table): page gather,
                both passes, reduce;
  ragged        a packed (varlen) batch of six sequences, 32768 tokens, in one
                call, beside one dense call per sequence;
  design        the device-side eviction design of the step's mass (the
                reference's consumers, evict.py, on the GPU);
  roofline      the dominant kernel's algorithmic tensor FLOP/s against the
                measured bf16 peak, and its exp rate against the MUFU ex2
                rate measured live on this GPU (the binding unit);
  strong_70b    strong scaling of the Llama-3-70B N=131072 shape: its 8
                (batch, kv-head) units split over the ranks, NCCL reduce
                inside each step, with the whole problem on one GPU beside it;
  cpu_baseline  the reference's own CPU path (block_mass_reference from the
                package installed in baseline/_ref, torch CPU, all host
                cores) on one whole (batch, kv-head) unit, with the numpy
                restatement timed on the same unit beside it.
`--impl reference` times the reference's CPU path alone (rank 0): one q-head
of that unit per step.  `--impl reference-triton` times the reference's own
Triton kernel (installed in baseline/_ref) on the same GPU: a secondary
comparison.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "kv-block-mass_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "causal block-mass QK pairs/sec at Llama-3-8B shape N=32k; % tensor/MUFU peak"
UNIT = "QK pairs/s"
DEFAULT_WORKLOAD = "llama3_8b_n32k"
L2_BYTES = 126 * 2**20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference", "reference-triton"], default="b200",
                    help="reference: the CPU path (reference arm); reference-triton: the reference's own "
                         "Triton kernel on this GPU (secondary comparison)")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--seq-len", type=int, default=None,
                    help="override N of the workload (small cases for profiler captures)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-strong", action="store_true",
                    help="skip the strong-scaling record of the Llama-3-70B N=131072 shape")
    ap.add_argument("--strong-steps", type=int, default=5)
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="weak: every rank owns a full batch entry of the workload; strong: the "
                         "workload's (batch, kv-head) units are split across the ranks")
    return ap.parse_args()


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs"), "bf16_tflops": d.get("bf16_tflops"),
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def traffic_record(workload: str):
    """DRAM bytes per launch of each kernel from a committed ncu summary, if any."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    return d.get(workload)


# ----------------------------------------------------------------------- clocks
def rank_gpu_indices(world: int) -> list[int]:
    """nvidia-smi indices of the GPUs the ranks of this node use (local ranks
    0..world-1, through CUDA_VISIBLE_DEVICES when it is set): the clock
    record covers the GPUs under load and no idle one."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if all(x.isdigit() for x in ids) and len(ids) >= world:
            return [int(x) for x in ids[:world]]
    return list(range(world))


class ClockSampler:
    """nvidia-smi clock / throttle sampling in the background (rank 0)."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-i", ",".join(map(str, self.gpus)), "-lms", "50"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        self.t_start = time.time()
        return self

    def mark(self):
        return time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self, t0: float, t1: float):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = time.mktime(time.strptime(parts[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                frac = float("0." + parts[0].split(".")[1]) if "." in parts[0] else 0.0
                rows.append((ts + frac, parts))
            except (ValueError, IndexError):
                continue
        inside = [r for r in rows if t0 - 0.06 <= r[0] <= t1 + 0.06]
        window = "timed region"
        if len(inside) < 3:
            inside = [r for r in rows if r[0] >= t0 - 2.0]
            window = "timed region +/- neighbouring steady-state steps (short timed region)"
        os.unlink(self.file.name)
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1][2]) for r in inside if r[1][2].replace(".", "").isdigit()]
        mx = [float(r[1][3]) for r in inside if r[1][3].replace(".", "").isdigit()]
        pw = [float(r[1][4]) for r in inside if r[1][4].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in inside for n, v in zip(names, r[1][6:10]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "reasons": reasons, "samples": len(inside),
                "window": window}


# ------------------------------------------------------------------- CPU sample
REF_SITE = ROOT / "baseline" / "_ref"


def stock_reference():
    """kv-block-mass's unmodified ``block_mass_reference`` (src/kvblockmass/reference.py:35-126)
    from the package installed in baseline/_ref, or None when it is not installed."""
    if not (REF_SITE / "kvblockmass").is_dir():
        return None
    if str(REF_SITE) not in sys.path:
        sys.path.insert(0, str(REF_SITE))
    try:
        from kvblockmass.reference import block_mass_reference
    except Exception:
        return None
    return block_mass_reference


def _unit0_inputs(w, heads: int):
    """q-heads [0, heads) of unit (batch 0, kv-head 0) with kv-head 0, full length, fp32
    (the exact values of make_inputs), and batch 0's masks."""
    from kvblockmass_b200.workloads import make_inputs, make_unit_inputs

    if w.key_mask_frac > 0 or w.dead_tail_rows > 0:
        q, k, km, qm = make_inputs(w)
        q, k = q[:1, :heads], k[:1, :1]
        qm = None if qm is None else qm[0]
    else:
        q, k = make_unit_inputs(w, 0, 1)
        q, km, qm = q[:, :heads], None, None
    return q.float().contiguous(), k.float().contiguous(), km, qm


def _unit_pairs(w, heads: int) -> int:
    return heads * (w.N * (w.N + 1) // 2 if w.causal else w.N * w.N)


def time_stock_reference(fn, w, qf, kf, km, qm):
    """One call of the stock reference on all host cores (torch CPU); seconds."""
    torch.set_num_threads(os.cpu_count() or 1)
    mask = km
    if qm is not None:  # a query mask becomes the [N, N] keep matrix the reference takes
        base = km if km is not None else torch.ones(w.N, dtype=torch.bool)
        mask = base[None, :] & qm[:, None]
    t0 = time.perf_counter()
    fn(qf, kf, attn_mask=mask, causal=w.causal, block_size=w.block_size)
    return time.perf_counter() - t0


def time_port(w, qf, kf, km, qm):
    """One call of the numpy restatement (oracle/block_mass_np.py) on all host cores; seconds."""
    from threadpoolctl import threadpool_limits

    from oracle.block_mass_np import block_mass_stream

    with threadpool_limits(limits=1):
        t0 = time.perf_counter()
        block_mass_stream(qf.numpy(), kf.numpy(), attn_mask=None if km is None else km.numpy(),
                          query_mask=None if qm is None else qm.numpy()[None], causal=w.causal,
                          block_size=w.block_size, threads=os.cpu_count() or 1, split_rows=True)
        return time.perf_counter() - t0


def cpu_baseline_record(w):
    """The CPU path on one whole (batch 0, kv-head 0) unit of workload ``w``: its
    G q-heads over every query row (no extrapolation), all host cores.

    ``kind: reference`` times kv-block-mass's own ``block_mass_reference``
    (baseline/_ref, torch CPU, the reference's streaming path); the numpy
    restatement is timed on the same unit beside it (``port_value``).  Without
    the installed reference the port is the baseline (``kind: port``).
    """
    G = w.Hq // w.Hkv
    qf, kf, km, qm = _unit0_inputs(w, G)
    npairs = _unit_pairs(w, G)
    cores = os.cpu_count() or 1
    t_port = time_port(w, qf, kf, km, qm)
    rec = {"unit": UNIT, "cores": cores, "port_value": npairs / t_port, "port_seconds": round(t_port, 3)}
    fn = stock_reference()
    what = f"unit (b=0, kv-head 0) = {G} q-heads x all {w.N} query rows of {w.name}: {npairs:.3e} pairs"
    if fn is not None:
        t_ref = time_stock_reference(fn, w, qf, kf, km, qm)
        rec.update(value=npairs / t_ref, kind="reference", seconds=round(t_ref, 3),
                   sample=(f"kv-block-mass block_mass_reference (baseline/_ref, torch CPU, "
                           f"{torch.get_num_threads()} threads, causal_skip on, query_chunk 256) on {what} "
                           f"in {t_ref:.2f} s; the numpy restatement took {t_port:.2f} s on the same unit"),
                   reference_over_port=round(t_port / t_ref, 3))
    else:
        rec.update(value=npairs / t_port, kind="port", seconds=round(t_port, 3),
                   sample=(f"oracle/block_mass_np.py (numpy restatement of reference.py:35-126) on {what} "
                           f"in {t_port:.2f} s (the reference package is not installed in baseline/_ref)"))
    return rec


def reference_arm(args, w):
    """--impl reference: the reference's CPU path on this host (rank 0 only).

    Each step runs kv-block-mass's own ``block_mass_reference`` (installed in
    baseline/_ref; torch CPU on all host cores) on one q-head of unit
    (batch 0, kv-head 0) over every query row; without the installed package
    the numpy restatement runs instead.  The value is one host's CPU rate
    whatever the number of GPUs of the run (``per_host``).
    """
    steps, warm = args.steps, args.warmup
    fn = stock_reference()
    qf, kf, km, qm = _unit0_inputs(w, 1)
    npairs = _unit_pairs(w, 1)
    if fn is not None:
        one = lambda: time_stock_reference(fn, w, qf, kf, km, qm)  # noqa: E731
        kind = "reference"
        what = (f"kv-block-mass block_mass_reference (baseline/_ref, torch CPU, all host cores, causal_skip on) "
                f"on q-head 0 of unit (b=0, kv-head 0) of {w.name}, all {w.N} query rows: {npairs:.3e} pairs "
                f"per step")
    else:
        one = lambda: time_port(w, qf, kf, km, qm)  # noqa: E731
        kind = "port"
        what = (f"oracle/block_mass_np.py (numpy restatement of reference.py:35-126; the reference package is "
                f"not installed) on q-head 0 of unit (b=0, kv-head 0) of {w.name}: {npairs:.3e} pairs per step")
    for _ in range(warm):
        one()
    secs = [one() for _ in range(steps)]
    total = sum(secs)
    value = npairs * steps / total
    cores = os.cpu_count() or 1
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
        "warmup": warm, "ms_per_step": total / steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference", "per_host": True, "host_cores": cores,
        "config": workload_config(w, args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind, "sample": what},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("one host's CPU cores, whatever n_gpus is: a ratio against an N-GPU line compares N GPUs "
                 "with one host"),
    }
    print(json.dumps(line), flush=True)


def reference_triton_arm(args, w):
    """--impl reference-triton: the reference's own GPU kernel on this GPU, rank 0 only.

    A secondary, GPU-to-GPU comparison (the reference arm proper is the CPU
    path above): kv-block-mass's unmodified ``block_mass_triton``
    (src/kvblockmass/triton_kernel.py:148-196) from the package installed in
    ``baseline/_ref`` (pip install --target), called through its public API on
    the workload's inputs in HBM, each call with its own allocations as the
    API makes them.  Prints an ``unavailable`` line if the package or Triton
    is missing.
    """
    ref_dir = ROOT / "baseline" / "_ref"
    try:
        sys.path.insert(0, str(ref_dir))
        from kvblockmass.triton_kernel import block_mass_triton  # noqa: E402
    except Exception as e:  # the package is not installed on this box
        print(json.dumps({"impl": "reference-triton", "unavailable": f"{type(e).__name__}: {e}"}), flush=True)
        return
    from kvblockmass_b200.workloads import make_inputs, pairs
    import kvblockmass_b200 as kb

    dev = torch.device("cuda", 0)
    q, k, km, qm = make_inputs(w)
    q, k = q.to(dev), k.to(dev)
    mask = None if km is None else km.to(dev)
    note = None
    if qm is not None:
        note = "the reference takes no query mask: its run keeps the dead rows this workload drops"
    kw = dict(attn_mask=mask, causal=w.causal, block_size=w.block_size)
    for _ in range(max(args.warmup, 1)):
        ref = block_mass_triton(q, k, **kw)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ref = block_mass_triton(q, k, **kw)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ours = kb.block_mass_b200(q, k, **kw)
    torch.cuda.synchronize()
    rel = float(((ours.double() - ref.double()).abs() / ref.double().abs().clamp_min(1e-30)).max())
    line = {"metric": METRIC, "value": pairs(w) / (ms * 1e-3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "impl": "reference-triton",
            "dtype": str(q.dtype).replace("torch.", ""), "data": "synthetic", "config": workload_config(w, 1),
            "max_rel_vs_b200": rel, "api": "kvblockmass.triton_kernel.block_mass_triton (baseline/_ref)"}
    if note:
        line["note"] = note
    print(json.dumps(line), flush=True)


def workload_config(w, world: int, scaling: str = "weak"):
    if scaling == "weak":
        shard = "each rank owns B_per_rank batch entries (B*H_kv units); NCCL reduce of mass to rank 0"
        gb = w.B * world
    else:
        shard = (f"the {w.B * w.Hkv} (batch, kv-head) units split contiguously over {world} ranks, each "
                 "rank's inputs the exact slices of the workload's draw; NCCL reduce of mass to rank 0")
        gb = w.B
    return {
        "workload": w.name, "B_per_rank": w.B if scaling == "weak" else None, "global_batch": gb,
        "Hq": w.Hq, "Hkv": w.Hkv,
        "D": w.D, "seq_len": w.N, "block_size": w.block_size, "causal": w.causal,
        "parallelism": f"units{world}" if world > 1 else "single",
        "shard": shard,
        "inputs_exceed_l2": True, "l2_flush": "none (q+k per step exceed the 126 MB L2)",
    }


# --------------------------------------------------------- strong scaling, 70B
def strong_70b_record(args, lib, dev, rank: int, world: int):
    """Strong scaling of the Llama-3-70B N=131072 shape (B=1, H_q=64, H_kv=8,
    D=128, block 256, causal, bf16, 1% x8 sink keys) beside the headline.

    Its 8 (batch, kv-head) units are split contiguously over the ranks; each
    rank draws exactly its units' slices of the workload's inputs
    (``make_unit_inputs``, the values the reference golden pins) into its own
    HBM.  A step is every rank's kernels on its units plus the NCCL reduce of
    the 512-bucket mass to rank 0; steps are timed with CUDA events between
    barriers, max over ranks.  With more than one rank, rank 0 also times the
    whole problem alone first (the units gathered over NCCL), which gives the
    run's own ``efficiency_vs_1gpu``.
    """
    import torch.distributed as dist

    from kvblockmass_b200 import ops
    from kvblockmass_b200.distributed import partition_units
    from kvblockmass_b200.workloads import WORKLOADS, make_unit_inputs, pairs

    w5 = WORKLOADS["llama3_70b_n128k"]
    parts = partition_units(w5.units, world)
    ub, ue = parts[rank]
    if ue <= ub:
        return None if rank else {"skipped": f"more ranks ({world}) than units ({w5.units})"}
    t0 = time.time()
    q, k = make_unit_inputs(w5, ub, ue)
    q, k = q.to(dev), k.to(dev)
    draw_s = time.time() - t0
    K, warm = max(1, args.strong_steps), 2
    stream = torch.cuda.current_stream(dev)

    def timed(prep, out, ws, reduce):
        def step():
            code = lib.kvbm_block_mass(ctypes.byref(prep.prob), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                       stream.cuda_stream)
            if code != 0:
                raise RuntimeError(f"kvbm_block_mass failed: {code}")
            if reduce:
                dist.reduce(out, dst=0, op=dist.ReduceOp.SUM)
        for _ in range(warm):
            step()
        if reduce:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(K):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        if reduce:
            dist.barrier()
        return e0.elapsed_time(e1) / K

    single_ms = None
    equal_parts = len({e - b for b, e in parts}) == 1
    if world > 1 and equal_parts:
        # the whole problem on rank 0 alone: gather every rank's units there
        qa = torch.empty((world,) + tuple(q.shape), dtype=q.dtype, device=dev)
        ka = torch.empty((world,) + tuple(k.shape), dtype=k.dtype, device=dev)
        dist.all_gather_into_tensor(qa, q.unsqueeze(0).contiguous())
        dist.all_gather_into_tensor(ka, k.unsqueeze(0).contiguous())
        if rank == 0:
            qf = qa.permute(1, 0, 2, 3, 4).reshape(1, w5.Hq, w5.N, w5.D)
            kf = ka.permute(1, 0, 2, 3, 4).reshape(1, w5.Hkv, w5.N, w5.D)
            pf = ops.make_problem(qf, kf, causal=True, block_size=w5.block_size)
            wsf = torch.empty(ops.workspace_bytes(pf), dtype=torch.uint8, device=dev)
            of = torch.empty(pf.nb, dtype=torch.float32, device=dev)
            single_ms = timed(pf, of, wsf, False)
            del qf, kf, pf, wsf, of
        del qa, ka
        torch.cuda.empty_cache()
        dist.barrier()
    prep = ops.make_problem(q, k, causal=True, block_size=w5.block_size)
    ws = torch.empty(ops.workspace_bytes(prep), dtype=torch.uint8, device=dev)
    out = torch.empty(prep.nb, dtype=torch.float32, device=dev)
    ms = timed(prep, out, ws, world > 1)
    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    if lib.kvbm_check_device_errors(stream.cuda_stream) != 0:
        raise RuntimeError("a device-side wait timed out in the strong-scaling run")
    total_pairs = pairs(w5)
    rec = {"workload": w5.name, "n_gpus": world, "units_per_rank": [e - b for b, e in parts], "steps": K,
           "warmup": warm, "ms_per_step": ms, "value": total_pairs / (ms * 1e-3), "unit": UNIT,
           "scaling": "strong", "pairs_per_step": total_pairs,
           "timing": "CUDA events per rank between barriers, max over ranks; NCCL reduce inside each step",
           "inputs": "exact slices of make_inputs(llama3_70b_n128k) per rank (make_unit_inputs), in HBM",
           "input_draw_s": round(draw_s, 1)}
    if world == 1:
        rec["single_gpu_ms"] = ms
        rec["efficiency_vs_1gpu"] = 1.0
    elif single_ms is not None:
        rec["single_gpu_ms"] = single_ms
        rec["speedup_vs_1gpu"] = single_ms / ms
        rec["efficiency_vs_1gpu"] = single_ms / ms / world
    del q, k, ws, out, prep
    torch.cuda.empty_cache()
    return rec if rank == 0 else None


# ------------------------------------------------------------------- B200 arm
def b200_arm(args, w):
    import torch.distributed as dist

    import kvblockmass_b200 as kb
    from kvblockmass_b200 import _lib, ops
    from kvblockmass_b200.workloads import make_inputs, pairs

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    lib = _lib.load()

    if args.scaling == "weak":
        # Rank r owns batch entry r of the weak-scaled problem (seed offset by rank).
        from dataclasses import replace
        wr = replace(w, seed=w.seed + 1000 * rank) if rank else w
        q_cpu, k_cpu, km, qm = make_inputs(wr)
        pairs_total_per_step = pairs(w) * world
    else:
        # Rank r owns a contiguous range of the workload's (batch, kv-head) units and
        # draws only those (exact slices of make_inputs' stream).
        from kvblockmass_b200.distributed import partition_units
        from kvblockmass_b200.workloads import make_unit_inputs
        if w.key_mask_frac > 0 or w.dead_tail_rows > 0:
            raise SystemExit("--scaling strong supports unmasked workloads only")
        ub, ue = partition_units(w.B * w.Hkv, world)[rank]
        if ue <= ub:
            raise SystemExit(f"rank {rank} has no units: use at most {w.B * w.Hkv} GPUs")
        q_cpu, k_cpu = make_unit_inputs(w, ub, ue)
        km = qm = None
        pairs_total_per_step = pairs(w)
    q_pin, k_pin = q_cpu.pin_memory(), k_cpu.pin_memory()
    q = q_pin.to(dev)
    k = k_pin.to(dev)
    kmd = None if km is None else km.to(dev)
    qmd = None if qm is None else qm.to(dev)
    prep = ops.make_problem(q, k, attn_mask=kmd, query_mask=qmd, causal=w.causal, block_size=w.block_size)
    path = ops.kernel_path(prep)
    method = ops.method_of(prep)
    # sized for this call and for the two-pass layout the LSE-input leg below takes
    prep_two = ops.make_problem(q, k, attn_mask=kmd, query_mask=qmd, causal=w.causal, block_size=w.block_size,
                                method="two_pass")
    ws = torch.empty(max(ops.workspace_bytes(prep), ops.workspace_bytes(prep_two), 256), dtype=torch.uint8,
                     device=dev)
    out = torch.empty(prep.nb, dtype=prep.out_dtype, device=dev)
    stream = torch.cuda.current_stream(dev)
    per_head = w.N * (w.N + 1) // 2 if w.causal else w.N * w.N
    pairs_rank = q.shape[0] * q.shape[1] * per_head
    launches = ops.launches_per_call(prep)

    def step(events=None):
        if events is None:
            code = lib.kvbm_block_mass(ctypes.byref(prep.prob), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                       stream.cuda_stream)
        else:
            arr = (ctypes.c_void_p * 4)(*[e.cuda_event for e in events])
            code = lib.kvbm_block_mass_events(ctypes.byref(prep.prob), out.data_ptr(), ws.data_ptr(),
                                              ws.numel(), stream.cuda_stream, arr)
        if code != 0:
            raise RuntimeError(f"kvbm_block_mass failed: {_lib.status_string(code)}")
        if world > 1:
            dist.reduce(out, dst=0, op=dist.ReduceOp.SUM)

    # MUFU ex2 rate of this GPU, measured before any heavy work so that the
    # peak is the unthrottled one (the roofline denominator of the exp unit).
    ex2 = ctypes.c_double(0.0)
    if lib.kvbm_measure_ex2_rate(stream.cuda_stream, ctypes.byref(ex2)) != 0:
        ex2.value = float("nan")

    # Warm-up (also creates the NCCL communicator).
    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()
    if lib.kvbm_check_device_errors(stream.cuda_stream) != 0:
        raise RuntimeError("a device-side wait timed out during warm-up")

    # Timed region: K steps, CUDA events on the launching stream, per-pass events inside.
    K = args.steps
    pass_events = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K)]
    # torch creates the CUDA event lazily at its first record(); record each once
    # so that the raw handles exist before the library records them in-call.
    for evs in pass_events:
        for e in evs:
            e.record(stream)
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(rank_gpu_indices(world)) if rank == 0 else None
    if sampler:
        sampler.__enter__()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_wall0 = time.time()
    e_start.record(stream)
    for i in range(K):
        step(pass_events[i])
    e_end.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    if world > 1:
        dist.barrier()
    ms_local = e_start.elapsed_time(e_end)
    ms_t = torch.tensor([ms_local], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_total = float(ms_t.item())
    p1 = [ev[0].elapsed_time(ev[1]) for ev in pass_events]
    p2 = [ev[1].elapsed_time(ev[2]) for ev in pass_events]
    p3 = [ev[2].elapsed_time(ev[3]) for ev in pass_events]
    if lib.kvbm_check_device_errors(stream.cuda_stream) != 0:
        raise RuntimeError("a device-side wait timed out in the timed region")

    # End to end through the public API: pinned host q/k in, mass back on the host.
    # The same K steps and the same idle lead-in (0.3 s) as the device-timed
    # steps, so that both start from the same power state.
    e2e = None
    if not args.no_e2e:
        Ke = args.e2e_steps or K
        kb.block_mass_b200(q_pin, k_pin, attn_mask=kmd, query_mask=qmd, causal=w.causal,
                           block_size=w.block_size, device=dev).cpu()
        torch.cuda.synchronize()
        time.sleep(0.3)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(Ke):
            m = kb.block_mass_b200(q_pin, k_pin, attn_mask=kmd, query_mask=qmd, causal=w.causal,
                                   block_size=w.block_size, device=dev)
            if world > 1:
                dist.reduce(m, dst=0, op=dist.ReduceOp.SUM)
            m_host = m.cpu()
        a1.record(stream)
        torch.cuda.synchronize()
        e_ms = torch.tensor([a0.elapsed_time(a1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        e2e = {"value": pairs_total_per_step * Ke / (float(e_ms.item()) * 1e-3), "unit": UNIT,
               "h2d_bytes_per_step": int(q_pin.numel() * q_pin.element_size() + k_pin.numel() * k_pin.element_size()),
               "d2h_bytes_per_step": int(m_host.numel() * m_host.element_size()),
               "steps": Ke, "api": "kvblockmass_b200.block_mass_b200(pinned host q/k, device='cuda').cpu()",
               "lead_in": "0.3 s idle after one untimed call, as before the device-timed steps",
               "bits_equal_device_call": None}
        # the same call on pageable host tensors (staged through pinned bounce buffers)
        q_pg, k_pg = q_pin.clone(), k_pin.clone()
        assert not q_pg.is_pinned()
        Ke = max(3, min(Ke, 10))
        kb.block_mass_b200(q_pg, k_pg, attn_mask=kmd, query_mask=qmd, causal=w.causal,
                           block_size=w.block_size, device=dev).cpu()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a0.record(stream)
        for _ in range(Ke):
            m = kb.block_mass_b200(q_pg, k_pg, attn_mask=kmd, query_mask=qmd, causal=w.causal,
                                   block_size=w.block_size, device=dev)
            if world > 1:
                dist.reduce(m, dst=0, op=dist.ReduceOp.SUM)
            m_host_pg = m.cpu()
        a1.record(stream)
        torch.cuda.synchronize()
        p_ms = torch.tensor([a0.elapsed_time(a1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(p_ms, op=dist.ReduceOp.MAX)
        e2e["pageable"] = {"value": pairs_total_per_step * Ke / (float(p_ms.item()) * 1e-3), "unit": UNIT,
                           "ms_per_step": float(p_ms.item()) / Ke,
                           "api": "block_mass_b200(pageable host q/k, device='cuda'): pinned bounce buffers"}
        del q_pg, k_pg
        if world == 1:
            dev_out = ops.run_prepared(prep, workspace=ws)
            torch.cuda.synchronize()
            e2e["bits_equal_device_call"] = bool(torch.equal(m_host.to(dev), dev_out)
                                                 and torch.equal(m_host_pg.to(dev), dev_out))

    # Caller-provided LSE (pass 1 skipped): the path an attention forward can feed.
    lse_input = None
    if not args.no_e2e:
        lse_buf = torch.empty(q.shape[0], q.shape[1], q.shape[2], dtype=torch.float32, device=dev)
        # the LSE of these inputs, from the library's own pass 1 (the values an attention
        # forward would return): run once, read back negated base-2 lse2, convert to natural log
        ops.run_prepared(prep, out=out, workspace=ws)
        torch.cuda.synchronize()
        if path == 1:
            # tensor-core layout: -lse2 over 128-row tiles, rows permuted inside each
            # 64-row half (row 8m + 2p + e at p*16 + 2m + e; kvbm_internal.cuh)
            npad = (w.N + 127) // 128 * 128
            nl = ws[: q.shape[0] * q.shape[1] * npad * 4].view(torch.float32).view(q.shape[0], q.shape[1], npad)
            rr = torch.arange(w.N, device=dev)
            ii = rr & 63
            slot = (rr & ~63) | (((ii >> 1) & 3) << 4) | ((ii >> 3) << 1) | (ii & 1)
            lse_buf.copy_(-nl[:, :, slot] / 1.4426950408889634)
        else:
            nl = ws[: q.shape[0] * q.shape[1] * w.N * 4].view(torch.float32).view(q.shape[0], q.shape[1], w.N)
            lse_buf.copy_(nl / 1.4426950408889634)
        st3 = (ctypes.c_int64 * 3)(*lse_buf.stride())

        def lse_call(method):
            o = _lib.Options()
            o.lse = lse_buf.data_ptr()
            for i in range(3):
                o.lse_stride[i] = st3[i]
            o.method = method
            return lambda: lib.kvbm_block_mass_ex(ctypes.byref(prep.prob), ctypes.byref(o), out.data_ptr(),
                                                  ws.data_ptr(), ws.numel(), stream.cuda_stream)

        def lse_ms_of(call):
            for _ in range(2):
                if call() != 0:
                    raise RuntimeError("kvbm_block_mass_ex with an LSE failed")
            torch.cuda.synchronize()
            l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            l0.record(stream)
            for _ in range(K):
                call()
            l1.record(stream)
            torch.cuda.synchronize()
            return l0.elapsed_time(l1) / K

        lse_ms = lse_ms_of(lse_call(_lib.KVBM_METHOD_AUTO))
        lse2_ms = lse_ms_of(lse_call(_lib.KVBM_METHOD_TWO_PASS))
        lse_input = {"value": pairs_rank / (lse_ms * 1e-3), "unit": UNIT,
                     "ms_per_step": lse_ms, "per_gpu": True, "method": ops.method_of(prep),
                     "api": "kvbm_block_mass_ex with kvbm_options.lse (row LSE supplied, as an attention "
                            "forward returns it; the same as kvbm_block_mass_lse)",
                     # one exp2 per pair against the live-measured MUFU rate
                     "mufu_frac_of_bound": (pairs_rank / ex2.value) / (lse_ms * 1e-3),
                     "two_pass": {"value": pairs_rank / (lse2_ms * 1e-3), "ms_per_step": lse2_ms,
                                  "note": "the two-pass method's pass 2 alone (plus the LSE import and the reduce)",
                                  "pass2_mufu_frac_of_bound": (pairs_rank / ex2.value) / (lse2_ms * 1e-3)}}
        del lse_buf

    # Paged key cache (16-key pages, shuffled page ids): page gather + both passes.
    paged = None
    if not args.no_e2e:
        P = 16
        B_, Hkv_, N_, D_ = k.shape
        npg = -(-N_ // P)
        gen = torch.Generator().manual_seed(7)
        table = torch.randperm(B_ * npg, generator=gen).reshape(B_, npg).to(torch.int32).to(dev)
        kp = torch.zeros(B_, Hkv_, npg * P, D_, dtype=k.dtype, device=dev)
        kp[:, :, :N_] = k
        cache = torch.empty(B_ * npg, P, Hkv_, D_, dtype=k.dtype, device=dev)
        cache[table.flatten().long()] = kp.reshape(B_, Hkv_, npg, P, D_).permute(0, 2, 3, 1, 4).reshape(
            B_ * npg, P, Hkv_, D_)
        del kp
        pp = ops.make_paged_problem(q, cache, table, attn_mask=kmd, query_mask=qmd, causal=w.causal,
                                    block_size=w.block_size)
        ws_p = torch.empty(ops.paged_workspace_bytes(pp), dtype=torch.uint8, device=dev)
        out_p = torch.empty_like(out)

        def paged_step():
            code = lib.kvbm_block_mass_paged(ctypes.byref(pp.prep.prob), ctypes.byref(pp.kv), None, None,
                                             out_p.data_ptr(), ws_p.data_ptr(), ws_p.numel(), stream.cuda_stream)
            if code != 0:
                raise RuntimeError(f"kvbm_block_mass_paged failed: {_lib.status_string(code)}")

        for _ in range(2):
            paged_step()
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(K):
            paged_step()
        g1.record(stream)
        torch.cuda.synchronize()
        if lib.kvbm_check_device_errors(stream.cuda_stream) != 0:
            raise RuntimeError("device error in the paged run")
        ms_p = g0.elapsed_time(g1) / K
        dense_out = ops.run_prepared(prep, workspace=ws)
        torch.cuda.synchronize()
        paged = {"value": pairs_rank / (ms_p * 1e-3), "unit": UNIT, "ms_per_step": ms_p, "per_gpu": True,
                 "page_size": P, "pages": B_ * npg, "bits_equal_dense": bool(torch.equal(out_p, dense_out)),
                 "gathered_bytes_per_step": int(2 * k.numel() * k.element_size()),
                 "api": "kvbm_block_mass_paged (k from a [pages, 16, H_kv, D] cache + block table)"}
        del cache, ws_p, table, dense_out

    # Ragged serving batch (packed varlen layout, the workload's heads, 32768 tokens in
    # six sequences): one call against one dense call per sequence.
    ragged = None
    if not args.no_e2e and path == 1:
        lens_r = [16384, 8192, 4096, 2048, 1024, 1024]
        T = sum(lens_r)
        gen = torch.Generator(device=dev).manual_seed(11)
        qp = torch.randn(T, q.shape[1], q.shape[3], device=dev, generator=gen).to(q.dtype)
        kp = torch.randn(T, k.shape[1], k.shape[3], device=dev, generator=gen).to(k.dtype)
        cu = torch.tensor([0] + list(np.cumsum(lens_r)), dtype=torch.int32, device=dev)
        vprep = ops.make_varlen_problem(qp, kp, cu, max_seqlen=max(lens_r), causal=w.causal,
                                        block_size=w.block_size)
        ws_r = torch.empty(ops.workspace_bytes(vprep), dtype=torch.uint8, device=dev)
        out_r = torch.empty(vprep.out_shape, dtype=torch.float32, device=dev)
        singles = []
        for i, L in enumerate(lens_r):
            s0 = int(cu[i])
            singles.append(ops.make_problem(qp[s0:s0 + L].transpose(0, 1).unsqueeze(0),
                                            kp[s0:s0 + L].transpose(0, 1).unsqueeze(0), causal=w.causal,
                                            block_size=w.block_size))

        def timed(fn, reps):
            for _ in range(2):
                fn()
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for _ in range(reps):
                fn()
            t1.record(stream)
            torch.cuda.synchronize()
            return t0.elapsed_time(t1) / reps

        ms_r = timed(lambda: ops.run_prepared(vprep, out=out_r, workspace=ws_r), K)
        ms_loop = timed(lambda: [ops.run_prepared(sp, workspace=ws_r) for sp in singles], K)
        per_head_r = sum(L * (L + 1) // 2 if w.causal else L * L for L in lens_r)
        pairs_r = q.shape[1] * per_head_r
        ragged = {"value": pairs_r / (ms_r * 1e-3), "unit": UNIT, "ms_per_step": ms_r, "per_gpu": True,
                  "seq_lens": lens_r, "tokens": T,
                  "one_call_per_sequence_ms": ms_loop,
                  "api": "kvbm_block_mass_ex (packed q/k + cu_seqlens), vs one kvbm_block_mass per sequence"}
        del qp, kp, ws_r, singles

    # Device-side consumer: the eviction design of the step's mass (kvbm_design), as
    # plan_reclaim sets it up (tail budget N/8, top slice half of it, 4 sinks, 32 recent).
    design = None
    design_mass_host = None
    if not args.no_e2e:
        from kvblockmass_b200 import design as dsg
        Nd, bsd = q.shape[2], w.block_size
        mass_d = ops.run_prepared(prep, workspace=ws)
        a_d, m2 = dsg._args(mass_d, Nd, bsd, Nd // 8, 4, 32, Nd // 16, 1e-6, False)
        a_d.seed = 1
        outs = {n: torch.empty(Nd, dtype=dt, device=dev) for n, dt in
                (("pi", torch.float64), ("keep", torch.bool), ("cert", torch.bool))}
        counts = torch.empty(1, 5, dtype=torch.int64, device=dev)
        o_d = _lib.DesignOut()
        o_d.pi = ctypes.cast(outs["pi"].data_ptr(), ctypes.POINTER(ctypes.c_double))
        o_d.keep = ctypes.cast(outs["keep"].data_ptr(), ctypes.POINTER(ctypes.c_uint8))
        o_d.certainty = ctypes.cast(outs["cert"].data_ptr(), ctypes.POINTER(ctypes.c_uint8))
        o_d.counts = ctypes.cast(counts.data_ptr(), ctypes.POINTER(ctypes.c_int64))
        ws_d = torch.empty(max(256, lib.kvbm_design_workspace_bytes(ctypes.byref(a_d))), dtype=torch.uint8,
                           device=dev)

        def design_step():
            if lib.kvbm_design(ctypes.byref(a_d), ctypes.byref(o_d), ws_d.data_ptr(), ws_d.numel(),
                               stream.cuda_stream) != 0:
                raise RuntimeError("kvbm_design failed")

        for _ in range(3):
            design_step()
        torch.cuda.synchronize()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record(stream)
        for _ in range(50):
            design_step()
        d1.record(stream)
        torch.cuda.synchronize()
        design_mass_host = mass_d.cpu().numpy()
        design = {"ms_per_design": d0.elapsed_time(d1) / 50, "tokens": Nd, "block_size": bsd,
                  "tail_budget": Nd // 8, "top_slice": Nd // 16, "kept_tokens": int(counts[0, 0]),
                  "launches": 3, "api": "kvbm_design (expand_block_scores + design_from_scores + block retention)"}
        del mass_d, m2, outs, ws_d

    clocks = None
    if sampler:
        sampler.__exit__(None, None, None)
        clocks = sampler.summary(t_wall0, t_wall1)

    strong = None
    if not args.no_strong:
        strong = strong_70b_record(args, lib, dev, rank, world)

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks = measured_peaks()
    fma_frac = float(lib.kvbm_exp2_fma_fraction()) if path >= 1 else 0.0
    t1, t2, t3 = statistics.mean(p1), statistics.mean(p2), statistics.mean(p3)
    dom_name, dom_ms = ("pass2_mass", t2) if t2 >= t1 else ("pass1_lse", t1)
    if method == "one_pass":  # pass 1 also forms the mass: its own traffic record
        dom_name, dom_ms = "pass1_one_pass", t1
    flops = pairs_rank * 2 * w.D                      # algorithmic tensor FLOPs per launch
    achieved_tflops = flops / (dom_ms * 1e-3) / 1e12
    exp_rate = pairs_rank / (dom_ms * 1e-3)           # one ex2 per pair per pass
    tensor_peak = peaks["bf16_tflops"]
    bound_time = max(flops / (tensor_peak * 1e12), pairs_rank / ex2.value)
    binding = "mufu_ex2" if pairs_rank / ex2.value >= flops / (tensor_peak * 1e12) else "tensor"
    tr = traffic_record(w.name)
    traffic = None
    if tr and dom_name in tr:
        traffic = tr[dom_name]
    value = pairs_total_per_step * K / (ms_total * 1e-3)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms_total / K, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(w, world, args.scaling),
        "kernel_path": "tcgen05" if path == 1 else "simt",
        "method": method,
        "kernel_ms": {"pass1_lse": t1, "pass2_mass": t2, "reduce": t3},
        "kernel_mcycles": (None if not clocks or not clocks.get("sm_mhz") else
                           {"pass1_lse": t1 * clocks["sm_mhz"] / 1e3, "pass2_mass": t2 * clocks["sm_mhz"] / 1e3,
                            "reduce": t3 * clocks["sm_mhz"] / 1e3,
                            "note": "kernel ms x median SM MHz of the timed region: cycles at the clock the "
                                    "power state allowed"}),
        "roofline": {
            "bound": "tensor", "achieved": achieved_tflops, "peak": tensor_peak, "unit": "TFLOP/s",
            "frac": achieved_tflops / tensor_peak, "traffic": traffic, "kernel": dom_name,
            "peak_source": ("measured bf16_tflops (burst) of MEASURED_PEAKS.json" if peaks["source"] == "measured"
                            else "fallback 1590 TFLOP/s bf16 burst (MEASURED_PEAKS.json absent)"),
            "binding_unit": binding,
            "mufu": {"achieved_ex2_per_s": exp_rate, "peak_ex2_per_s": ex2.value,
                     "frac": exp_rate / ex2.value, "peak_source": "measured live (kvbm_measure_ex2_rate)",
                     "note": "achieved counts every exp2 of the algorithm (one per pair); fma_pipe_fraction "
                             "of them run on the FMA pipe, so the MUFU unit itself is at mufu_unit_frac",
                     "fma_pipe_fraction": fma_frac,
                     "mufu_unit_frac": exp_rate * (1.0 - fma_frac) / ex2.value},
            "frac_of_binding": (bound_time / (dom_ms * 1e-3)),
            "algorithmic_per_launch": {"pairs": pairs_rank, "tensor_flops": flops, "ex2": pairs_rank},
        },
        "gpu_launches": K * launches,
        "clocks": clocks,
    }
    if e2e:
        line["e2e"] = e2e
    if lse_input:
        line["lse_input"] = lse_input
    if paged:
        line["paged"] = paged
    if ragged:
        line["ragged"] = ragged
    if design:
        line["design"] = design
    if strong:
        line["strong_70b"] = strong
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_record(w)
        if design is not None and design_mass_host is not None:
            # the same design on the host: the oracle's restatement of evict.py (float64 numpy)
            from oracle import evict_np as ev
            Nd = design["tokens"]
            t0 = time.perf_counter()
            reps = 20
            for _ in range(reps):
                sc = ev.expand_block_scores(design_mass_host, Nd, design["block_size"])
                ev.design_from_scores(sc, design["tail_budget"], n_sinks=4, recency=32,
                                      top_slice=design["top_slice"], uniforms=np.zeros(Nd))
            line["cpu_baseline"]["design_ms"] = (time.perf_counter() - t0) * 1e3 / reps
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    from kvblockmass_b200.workloads import WORKLOADS

    w = WORKLOADS[args.workload]
    if args.seq_len:
        from dataclasses import replace
        w = replace(w, N=args.seq_len, name=f"{w.name}@N={args.seq_len}")
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return 0
        reference_arm(args, w)
        return 0
    if args.impl == "reference-triton":
        if int(os.environ.get("RANK", "0")) != 0:
            return 0
        reference_triton_arm(args, w)
        return 0
    b200_arm(args, w)
    return 0


if __name__ == "__main__":
    sys.exit(main())
