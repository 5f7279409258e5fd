"""Build libqhtp.so (the C-ABI library with the sm_100a kernels) in-tree with nvcc.

    python qcom_htp_b200/build.py [--force] [--ptxas-v]   # -> qcom_htp_b200/libqhtp.so

The library is compiled only for sm_100a (B200): tcgen05 / TMA / TMEM instructions are used
directly, so there is no other target.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libqhtp.so"
SOURCES = ["qhtp_abi.cu", "qgemm.cu", "qdecode.cu", "gdn.cu", "gdn256.cu", "gdn256x2.cu", "noalloc.cu", "wire.cu", "gdn256f.cu", "qgroup.cu", "peak.cu", "qchain.cu", "qdec4.cu"]
HEADERS = ["ptx.cuh", "requant.cuh", "internal.h", "gdn_common.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O2",
]
OBJ_DIR = PKG.parent / "_build"


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the qhtp CUDA library cannot be built")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [PKG.parent / "include" / "qhtp.h"]
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile every source to an object (in parallel, one nvcc per file), then link the shared
    library.  Whole-library rebuild: the sources share headers, so nothing is reused."""
    if not force and not _stale():
        return LIB
    from concurrent.futures import ThreadPoolExecutor
    OBJ_DIR.mkdir(exist_ok=True)
    nv = nvcc()

    def compile_one(src: str):
        obj = OBJ_DIR / (Path(src).stem + ".o")
        cmd = [nv, *NVCC_FLAGS, *(extra or []), "-c", "-o", str(obj), str(CSRC / src)]
        return cmd, obj, subprocess.run(cmd, capture_output=True, text=True)

    with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 4)) as ex:
        results = list(ex.map(compile_one, SOURCES))
    for cmd, _, r in results:
        if verbose:
            print(" ".join(cmd))
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed ({r.returncode}):\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr:
            print(r.stderr)
    link = [nv, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(LIB),
            *[str(o) for _, o, _ in results]]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    force = "--force" in sys.argv
    ptxas_v = "--ptxas-v" in sys.argv
    out = build(force=force or ptxas_v, verbose=True, extra=["-Xptxas", "-v"] if ptxas_v else None)
    print(out)
