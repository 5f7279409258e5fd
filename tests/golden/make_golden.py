#!/usr/bin/env python3
"""Regenerate the golden fixtures in this folder from the reference checkout.

Run in a container where the reference is mounted (read only):

    python tests/golden/make_golden.py --reference <path-to-qcom_htp>

It writes
  mm_reference_cases.json  sha256 digests + qparams of the reference's own arrays, made by importing
                           ``scripts/generate_qnn_matmul_python_cases.py`` and calling its
                           ``make_float_case`` / ``quantize_case`` (all families x 7 cases, 3 shapes)
  mm_small_cases.npz       full arrays of the reference's cases at M=32,K=128,N=32 (its CLI default)
  w16a16_identity.json     digests of the reference's W16A16 byte-split identity vectors
                           (``scripts/verify_w16a16_two_w8a16.py`` draws, default seed 0xB17E)
  gdn_sbr_kat.npz          2 heads of the retained GDN known-answer fixture
                           ``archive/gdn_solve_2026-06/example_gdn_native/solve_op_standalone/sbr``:
                           A (rebuilt from Adiag/Aoff_* blocks, fp32) and Tref = fp64 inv(I-A)
                           stored fp32 (written by archive/.../scripts/gdn_split_br_probe.py:216)

The tests only read these files; nothing at test time touches the reference.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SHAPES = [(256, 256, 256), (32, 128, 32), (64, 192, 96)]


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).reshape(-1).tobytes()).hexdigest()


def load_module(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def make_mm(ref: Path) -> None:
    gen = load_module(ref / "scripts" / "generate_qnn_matmul_python_cases.py", "ref_gen")
    entries = []
    small = {}
    for (m, k, n) in SHAPES:
        for fname, fam in gen.FAMILIES.items():
            if fam.weight_schema == "per_group" and k <= 64:
                continue
            for case in gen.CASES:
                x, w, b = gen.make_float_case(fam, case, m, k, n)
                q = gen.quantize_case(fam, x, w, b)
                e = {
                    "family": fname, "case": case, "shape_mkn": [m, k, n],
                    "seed": gen.seed_for(fam.name, case),
                    "act_scale": float(q["qparams"]["activation"]["scale"]),
                    "out_scale": float(q["qparams"]["output"]["scale"]),
                    "sha256": {
                        "activation_q": sha(q["activation_q"]),
                        "weight_q_nk": sha(q["weight_q_nk"]),
                        "weight_scale": sha(q["weight_scale"]),
                        "bias_q_int32": sha(q["bias_q_int32"]),
                        "output_ref_q": sha(q["output_q"]),
                    },
                    "output_counts": {k2: int(v) for k2, v in gen.output_counts(q["output_q"], fam).items()},
                }
                if q["weight_lpbq_per_block_int_scale"] is not None:
                    e["sha256"]["lpbq_block_scale"] = sha(q["weight_lpbq_per_block_int_scale"])
                    e["sha256"]["lpbq_expanded_q_nk"] = sha(q["weight_lpbq_expanded_q_nk"])
                entries.append(e)
                if (m, k, n) == (32, 128, 32):
                    key = f"{fname}/{case}"
                    small[key + "/activation_q"] = q["activation_q"]
                    small[key + "/weight_q_nk"] = q["weight_q_nk"]
                    small[key + "/weight_scale"] = q["weight_scale"]
                    small[key + "/bias_q_int32"] = q["bias_q_int32"]
                    small[key + "/output_ref_q"] = q["output_q"]
                    small[key + "/scales"] = np.array(
                        [q["qparams"]["activation"]["scale"], q["qparams"]["output"]["scale"]], np.float64)
                    if q["weight_lpbq_per_block_int_scale"] is not None:
                        small[key + "/lpbq_block_scale"] = q["weight_lpbq_per_block_int_scale"]
    payload = {
        "schema": "qhtp_b200.golden.mm.v1",
        "source": "scripts/generate_qnn_matmul_python_cases.py (imported from the reference checkout)",
        "entries": entries,
    }
    (HERE / "mm_reference_cases.json").write_text(json.dumps(payload, indent=1, sort_keys=True) + "\n")
    np.savez_compressed(HERE / "mm_small_cases.npz", **small)
    print(f"mm: {len(entries)} entries, {len(small)} small arrays")


def make_w16(ref: Path) -> None:
    ver = load_module(ref / "scripts" / "verify_w16a16_two_w8a16.py", "ref_w16")
    out = []
    for (m, k, n) in [(64, 64, 64), (256, 256, 256), (128, 256, 96)]:
        rng = np.random.default_rng(0xB17E)
        act = rng.integers(0, 65536, size=(m, k), dtype=np.uint16).astype(np.int64)
        q16 = rng.integers(-32768, 32768, size=(k, n)).astype(np.int64)
        hi, lo = ver.decompose_int16_to_bytes(q16)
        acc_hi = (act - ver.ACT_ZP) @ hi
        acc_lo = (act - ver.ACT_ZP) @ lo
        out.append({"shape_mkn": [m, k, n], "seed": 0xB17E,
                    "sha256": {"act_u16": sha(act.astype(np.uint16)), "q16_kn": sha(q16.astype(np.int16)),
                               "hi_kn": sha(hi.astype(np.int8)), "lo_kn": sha(lo.astype(np.uint8)),
                               "acc_hi": sha(acc_hi), "acc_lo": sha(acc_lo),
                               "acc": sha((act - ver.ACT_ZP) @ q16)}})
    (HERE / "w16a16_identity.json").write_text(json.dumps(
        {"schema": "qhtp_b200.golden.w16a16.v1",
         "source": "scripts/verify_w16a16_two_w8a16.py draws and decompose_int16_to_bytes",
         "entries": out}, indent=1) + "\n")
    print("w16a16: ok")


def make_gdn(ref: Path, heads=(0, 7)) -> None:
    d = ref / "archive/gdn_solve_2026-06/example_gdn_native/solve_op_standalone/sbr"
    H, C, BL, NB = 16, 256, 64, 4
    adiag = np.fromfile(d / "Adiag.raw", np.float32).reshape(H, NB, BL, BL)
    A = np.zeros((H, C, C), np.float32)
    for i in range(NB):
        A[:, i * BL:(i + 1) * BL, i * BL:(i + 1) * BL] = adiag[:, i]
    for (i, k) in [(1, 0), (2, 0), (2, 1), (3, 0), (3, 1), (3, 2)]:
        blk = np.fromfile(d / f"Aoff_{i}{k}.raw", np.float32).reshape(H, BL, BL)
        A[:, i * BL:(i + 1) * BL, k * BL:(k + 1) * BL] = blk
    tref = np.fromfile(d / "Tref.raw", np.float32).reshape(H, C, C)
    hs = list(heads)
    np.savez_compressed(HERE / "gdn_sbr_kat.npz", A=A[hs], Tref=tref[hs], heads=np.array(hs))
    print("gdn: heads", hs)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    a = ap.parse_args()
    make_mm(a.reference)
    make_w16(a.reference)
    make_gdn(a.reference)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
