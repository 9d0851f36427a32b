"""Golden block mass of the Llama-3-70B long-context shape, from the reference run on a GPU.

Shape: B=1, H_q=64, H_kv=8, D=128, N=131072, block 256, causal, bf16 q/k drawn
by ``kvblockmass_b200.workloads.make_inputs`` (seed 4: ``q`` then ``k`` from
one CPU generator, then 1% of key rows x8 as attention sinks, then the cast to
bf16).  The reference's keep matrix alone is 16 GiB at this N and its CPU run
takes hours, so the unmodified ``block_mass_reference``
(kv-block-mass ``src/kvblockmass/reference.py:35-126``) runs on a CUDA device
(its ``device=`` argument, ``reference.py:74-76``) once per kv-head group:
mass is a sum over (batch, head), so the eight group vectors add up to the
whole.  Each group runs on the bf16 values upcast to fp32 (TF32 matmuls off),
and once more upcast to fp64 as an error-free yardstick.  The inputs are drawn
per group (``make_unit_inputs``: exactly ``make_inputs``' slices).

Usage, on a machine with a CUDA GPU and the reference package::

    KVBM_REF=<reference checkout, or a pip --target dir holding kvblockmass> \\
        python tests/golden/gen_golden_70b.py --out tests/golden/llama3_70b_n128k.json
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "kv-block-mass_b200"))

from kvblockmass_b200.workloads import WORKLOADS, make_unit_inputs  # noqa: E402


def reference_module():
    ref = os.environ.get("KVBM_REF")
    if not ref:
        raise SystemExit("set KVBM_REF to the reference checkout (with src/kvblockmass) or to a directory "
                         "that holds the installed kvblockmass package")
    ref = Path(ref)
    sys.path.insert(0, str(ref / "src" if (ref / "src" / "kvblockmass").is_dir() else ref))
    from kvblockmass import reference  # noqa: E402

    return reference


def checksum(t: torch.Tensor) -> dict:
    t64 = t.to(torch.float64).reshape(-1)
    return {"sum": float(t64.sum()), "abs_sum": float(t64.abs().sum()),
            "first": [float(x) for x in t64[:4]], "last": [float(x) for x in t64[-4:]]}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--no-fp64", action="store_true")
    args = ap.parse_args()
    ref = reference_module()
    assert torch.cuda.is_available(), "the reference runs on a CUDA device at this size"
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    w = WORKLOADS["llama3_70b_n128k"]
    dev = torch.device("cuda", 0)
    units = []
    tot32 = torch.zeros(w.num_blocks, dtype=torch.float64)
    tot64 = torch.zeros(w.num_blocks, dtype=torch.float64)
    for u in range(w.units):
        q, k = make_unit_inputs(w, u, u + 1)
        rec = {"unit": u, "q_checksum": checksum(q), "k_checksum": checksum(k)}
        qf, kf = q.float(), k.float()
        torch.cuda.synchronize()
        t0 = time.time()
        m32 = ref.block_mass_reference(qf, kf, causal=True, block_size=w.block_size, device=dev)
        torch.cuda.synchronize()
        rec["seconds_fp32"] = round(time.time() - t0, 2)
        rec["mass_ref_fp32"] = [float(x) for x in m32.cpu()]
        tot32 += m32.cpu().double()
        if not args.no_fp64:
            t0 = time.time()
            m64 = ref.block_mass_reference(q.double(), k.double(), causal=True, block_size=w.block_size,
                                           device=dev)
            torch.cuda.synchronize()
            rec["seconds_fp64"] = round(time.time() - t0, 2)
            rec["mass_ref_fp64"] = [float(x) for x in m64.cpu()]
            tot64 += m64.cpu()
        units.append(rec)
        print(f"unit {u}: sum fp32 {sum(rec['mass_ref_fp32']):.3f} ({rec['seconds_fp32']} s)", flush=True)
        del q, k, qf, kf, m32
        torch.cuda.empty_cache()
    out = {
        "meta": {"generator": "tests/golden/gen_golden_70b.py", "torch": torch.__version__,
                 "device": torch.cuda.get_device_name(dev),
                 "reference": "kv-block-mass src/kvblockmass/reference.py (block_mass_reference), "
                              "device=cuda, one call per kv-head group, TF32 off"},
        "name": w.name, "workload": w.name, "N": w.N, "block_size": w.block_size,
        "input_protocol": "kvblockmass_b200.workloads.make_inputs (drawn per unit by make_unit_inputs)",
        "units": units,
        "mass_ref_fp32": [float(x) for x in tot32],
        "mass_ref_fp32_note": "sum over the eight kv-head groups (fp64 adds of the reference's fp32 vectors)",
    }
    if not args.no_fp64:
        out["mass_ref_fp64"] = [float(x) for x in tot64]
    Path(args.out).write_text(json.dumps(out))
    print(f"total fp32 {float(tot32.sum()):.3f} (expected {w.Hq * w.N})", flush=True)


if __name__ == "__main__":
    main()
