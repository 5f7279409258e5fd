"""Fixture generator for the fused A-construction + inverse (qhtp_gdn_chunk_inverse).

Runs where the reference tree is readable (path as the first argument).  Calls the reference's own
``gdn_chunk`` (scripts/gdn_ref_kernel.py:60-100, fp64, torch on CPU) on seeded raw inputs at its
native chunk size C = 64, and captures the inverse T = (I - A)^-1 it forms, through its GEMM hook:
the first operand of the 'A_Uv' GEMM (:84) is T.  Writes tests/golden/gdn_kbg_kat.npz with the
inputs (k as bf16-representable f32, beta, per-token log gates) and T.  No bytecode is written into
the reference tree.

    python tests/golden/make_gdn_kbg_golden.py /path/to/reference
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit(f"usage: python {Path(__file__).name} <reference checkout>")
    ref = Path(sys.argv[1])
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(ref / "scripts"))
    sys.path.insert(0, str(ROOT))
    import gdn_ref_kernel as R  # noqa: E402
    from oracle.gdn_oracle import make_kbg  # noqa: E402

    n, C, D = 3, 64, 128
    k, beta, g_tok = make_kbg(n, C, D, seed=0x6B67)
    captured = {}

    def mm(a, b, site=None):
        if site == "A_Uv":
            captured["T"] = a.clone()
        return a @ b

    kt = torch.from_numpy(k).double().reshape(1, n, C, D)       # [B=1, H=n, C, D]
    q = torch.ones_like(kt)
    v = torch.ones_like(kt)
    S = torch.zeros(1, n, D, D, dtype=torch.float64)
    R.gdn_chunk(q, kt, v, torch.from_numpy(g_tok).double().reshape(1, n, C),
                torch.from_numpy(beta).double().reshape(1, n, C), S, mm=mm)
    T = captured["T"].reshape(n, C, C).numpy()
    dst = Path(__file__).resolve().parent / "gdn_kbg_kat.npz"
    np.savez_compressed(dst, k=k, beta=beta, g_tok=g_tok, T=T)
    print(f"{dst}: T {T.shape}, |T| {np.abs(T).max():.3f}")


if __name__ == "__main__":
    main()
