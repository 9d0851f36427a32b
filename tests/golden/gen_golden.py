"""Generate golden block-mass vectors by running the reference itself.

Runs kv-block-mass's own ``block_mass_reference`` (and its dense test oracle
``tests/naive.py``) on seeded inputs and writes the outputs as JSON fixtures
next to this script.  Inputs are not stored: every case records the recipe
(shape, seed, generator protocol) plus input checksums, and the tests
regenerate the inputs with the same CPU ``torch.Generator`` and check the
checksums before comparing.

Usage (needs the reference sources; they are not needed to *use* the
fixtures)::

    KVBM_REF=/root/reference python tests/golden/gen_golden.py [--big]

``--big`` adds the Llama-3-8B N=32768 and the batched masked N=16384 shapes
(minutes of CPU and ~4 GiB of RAM each).
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
REF = Path(os.environ.get("KVBM_REF", "/root/reference"))
sys.path.insert(0, str(REF / "src"))
sys.path.insert(0, str(REF))
sys.path.insert(0, str(ROOT / "kv-block-mass_b200"))

from kvblockmass.reference import block_mass_reference  # noqa: E402
from tests.naive import block_mass_naive  # noqa: E402  (the reference's tests/naive.py)

from kvblockmass_b200.workloads import WORKLOADS, make_inputs  # noqa: E402


def checksum(t: torch.Tensor) -> dict:
    t64 = t.to(torch.float64).reshape(-1)
    return {
        "sum": float(t64.sum()),
        "abs_sum": float(t64.abs().sum()),
        "first": [float(x) for x in t64[:4]],
        "last": [float(x) for x in t64[-4:]],
    }


def qk_test(B, H_q, H_kv, N, D, seed, dtype=torch.float64):
    """Input protocol of the reference's tests (``tests/test_reference.py:10-14``)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H_q, N, D, generator=g, dtype=dtype)
    k = torch.randn(B, H_kv, N, D, generator=g, dtype=dtype)
    return q, k


def mask_recipe(kind, N, seed=None):
    """Masks used by the reference's tests, rebuilt from a recipe."""
    if kind is None:
        return None
    if kind == "keys_first_half":               # test_reference.py:155-157
        m = torch.ones(N, dtype=torch.bool)
        m[N // 2:] = False
        return m
    if kind == "row0_dead":                      # test_reference.py:110-111
        m = torch.ones(N, N, dtype=torch.bool)
        m[0, :] = False
        return m
    if kind == "rows_from_64_dead":              # eval/cases.jsonl KVBM-03
        m = torch.ones(N, N, dtype=torch.bool)
        m[64:, :] = False
        return m
    if kind == "rand_pairs":                     # test_reference.py:180
        return torch.rand(N, N, generator=torch.Generator().manual_seed(seed)) > 0.5
    if kind == "rand_keys":
        return torch.rand(N, generator=torch.Generator().manual_seed(seed)) > 0.3
    raise ValueError(kind)


# (name, B, H_q, H_kv, N, D, seed, causal, block_size, mask kind, mask seed)
SMALL_CASES = [
    ("sum_rule_noncausal", 2, 4, 2, 128, 32, 0, False, 64, None, None),
    ("sum_rule_causal", 2, 4, 2, 128, 32, 0, True, 64, None, None),
    ("naive_noncausal_s7", 2, 4, 2, 128, 32, 7, False, 64, None, None),
    ("naive_causal_s7", 2, 4, 2, 128, 32, 7, True, 64, None, None),
    ("gqa_8_2_n96", 1, 8, 2, 96, 16, 3, True, 32, None, None),
    ("ragged_n1", 2, 2, 1, 1, 8, 11, True, 64, None, None),
    ("ragged_n5", 2, 2, 1, 5, 8, 11, True, 64, None, None),
    ("ragged_n64", 2, 2, 1, 64, 8, 11, True, 64, None, None),
    ("ragged_n65", 2, 2, 1, 65, 8, 11, True, 64, None, None),
    ("ragged_n100", 2, 2, 1, 100, 8, 11, True, 64, None, None),
    ("ragged_n129", 2, 2, 1, 129, 8, 11, True, 64, None, None),
    ("n_lt_block", 1, 1, 1, 16, 8, 5, False, 64, None, None),
    ("key_mask_half", 2, 2, 2, 128, 16, 13, False, 64, "keys_first_half", None),
    ("row0_dead", 1, 1, 1, 64, 8, 17, False, 32, "row0_dead", None),
    ("rows_from_64_dead", 2, 4, 2, 128, 32, 0, False, 64, "rows_from_64_dead", None),
    ("n600_chunked", 1, 2, 1, 600, 16, 59, True, 64, None, None),
    ("skip_n600_gqa", 1, 4, 2, 600, 16, 71, True, 64, None, None),
    ("skip_n129_pairs", 2, 2, 1, 129, 8, 72, True, 32, "rand_pairs", 5),
    ("keys_rand_causal", 2, 4, 1, 300, 24, 19, True, 48, "rand_keys", 9),
    ("gqa_n100_d16_bs64", 1, 8, 2, 100, 16, 37, True, 64, None, None),
    ("d128_n257", 1, 4, 2, 257, 128, 23, True, 64, None, None),
    ("d64_n1000_noncausal", 1, 2, 1, 1000, 64, 29, False, 100, None, None),
]


def small_cases():
    out = []
    for (name, B, Hq, Hkv, N, D, seed, causal, bs, mk, ms) in SMALL_CASES:
        q, k = qk_test(B, Hq, Hkv, N, D, seed)
        mask = mask_recipe(mk, N, ms)
        ref64 = block_mass_reference(q, k, attn_mask=mask, causal=causal, block_size=bs)
        noskip64 = block_mass_reference(q, k, attn_mask=mask, causal=causal, block_size=bs,
                                        causal_skip=False)
        ref32 = block_mass_reference(q.float(), k.float(), attn_mask=mask, causal=causal,
                                     block_size=bs)
        naive = None
        if mk is None or mask is not None and mask.dim() == 2:
            naive = block_mass_naive(q, k, attn_mask=mask, causal=causal, block_size=bs)
        out.append({
            "name": name, "B": B, "Hq": Hq, "Hkv": Hkv, "N": N, "D": D, "seed": seed,
            "causal": causal, "block_size": bs, "mask": mk, "mask_seed": ms,
            "input_protocol": "tests/test_reference.py:_qk (fp64 randn, q then k)",
            "q_checksum": checksum(q), "k_checksum": checksum(k),
            "mass_ref_fp64": [float(x) for x in ref64],
            "mass_ref_fp64_noskip_identical": bool(torch.equal(ref64, noskip64)),
            "mass_ref_fp32": [float(x) for x in ref32],
            "mass_naive_fp64": None if naive is None else [float(x) for x in naive],
        })
        print(f"  {name}: sum={float(ref64.sum()):.6f}", flush=True)
    return out


def workload_case(name: str, per_batch: bool = False, fp64: bool = True):
    w = WORKLOADS[name]
    q, k, key_mask, query_mask = make_inputs(w)
    qf, kf = q.float(), k.float()
    t0 = time.time()
    if not per_batch:
        mass = block_mass_reference(qf, kf, attn_mask=key_mask, causal=w.causal,
                                    block_size=w.block_size)
    else:
        # mass is linear over the batch: run the reference per batch entry with that
        # entry's [N, N] keep matrix (key mask & query-row mask).
        mass = torch.zeros(w.num_blocks, dtype=torch.float32)
        for b in range(w.B):
            m = key_mask
            if query_mask is not None and not bool(query_mask[b].all()):
                m = (key_mask if key_mask is not None else torch.ones(w.N, dtype=torch.bool))
                m = m[None, :] & query_mask[b][:, None]
            mass += block_mass_reference(qf[b:b + 1], kf[b:b + 1], attn_mask=m,
                                         causal=w.causal, block_size=w.block_size)
    t_ref = time.time() - t0
    rec = {
        "name": name, "workload": name, "N": w.N,
        "input_protocol": "kvblockmass_b200.workloads.make_inputs",
        "q_checksum": checksum(q), "k_checksum": checksum(k),
        "key_mask_count": None if key_mask is None else int(key_mask.sum()),
        "query_mask_count": None if query_mask is None else int(query_mask.sum()),
        "mass_ref_fp32": [float(x) for x in mass],
        "ref_seconds_cpu": round(t_ref, 2),
    }
    if w.causal and not per_batch:
        t0 = time.time()
        noskip = block_mass_reference(qf, kf, attn_mask=key_mask, causal=w.causal,
                                      block_size=w.block_size, causal_skip=False)
        rec["ref_seconds_cpu_noskip"] = round(time.time() - t0, 2)
        rec["mass_ref_fp32_noskip_identical"] = bool(torch.equal(mass, noskip))
    if fp64:
        m64 = block_mass_reference(q.double(), k.double(), attn_mask=key_mask, causal=w.causal,
                                   block_size=w.block_size)
        rec["mass_ref_fp64"] = [float(x) for x in m64]
    print(f"  {name}: sum={float(mass.sum()):.3f} ref {t_ref:.1f}s", flush=True)
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--big", action="store_true")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    meta = {"generator": "tests/golden/gen_golden.py", "torch": torch.__version__,
            "reference": "kv-block-mass src/kvblockmass/reference.py (block_mass_reference)"}
    if args.only in (None, "small"):
        print("small cases (reference test-suite shapes)")
        (HERE / "small_cases.json").write_text(json.dumps({"meta": meta, "cases": small_cases()}))
    if args.only in (None, "cpu_ref_n2048"):
        (HERE / "cpu_ref_n2048.json").write_text(
            json.dumps({"meta": meta, **workload_case("cpu_ref_n2048")}))
    if args.only in (None, "gqa_n8192_fp32"):
        (HERE / "gqa_n8192_fp32.json").write_text(
            json.dumps({"meta": meta, **workload_case("gqa_n8192_fp32")}))
    if args.big or args.only == "llama3_8b_n32k":
        (HERE / "llama3_8b_n32k.json").write_text(
            json.dumps({"meta": meta, **workload_case("llama3_8b_n32k", fp64=False)}))
    if args.big or args.only == "batched_masked_n16k":
        (HERE / "batched_masked_n16k.json").write_text(
            json.dumps({"meta": meta, **workload_case("batched_masked_n16k", per_batch=True,
                                                      fp64=False)}))


if __name__ == "__main__":
    main()
