"""Fixture generator for the weight wire-format adapters (qhtp_weights_from_wire).

Runs where the reference tree is readable (path as the first argument); the fixture it writes,
tests/golden/wire_formats.npz, travels with the tests.  It packs seeded logical [K, N] weights with
the reference's OWN packing code -- ``_weight_initializer`` and the ``_pack_*`` helpers of
example/qnn_hmx_matmul_common/gen_quant_chain.py:285-742 -- and stores, per wire format, the
logical weights and the exact bytes the reference would put in its ONNX initializer.

gen_quant_chain.py imports onnx (absent here) only to build graphs; the packers are plain numpy.  The
onnx names are stubbed so the module imports, and ``numpy_helper.from_array`` returns the array, which
is precisely the initializer payload.  Nothing is written into the reference tree (no bytecode).

    python tests/golden/make_wire_golden.py /path/to/reference
"""
from __future__ import annotations

import sys
import types
from pathlib import Path

import numpy as np

K, N = 64, 256          # multiples of 32 / 64 / 128, so every packer accepts the shape


def load_reference(ref: Path):
    sys.dont_write_bytecode = True
    onnx = types.ModuleType("onnx")
    helper = types.ModuleType("onnx.helper")
    numpy_helper = types.ModuleType("onnx.numpy_helper")
    numpy_helper.from_array = lambda arr, name=None: np.array(arr, copy=True)
    onnx.TensorProto = types.SimpleNamespace()
    onnx.helper = helper
    onnx.numpy_helper = numpy_helper
    sys.modules.update({"onnx": onnx, "onnx.helper": helper, "onnx.numpy_helper": numpy_helper})
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "example" / "qnn_hmx_matmul_common"))
    import gen_quant_chain as G  # noqa: E402
    return G


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit(f"usage: python {Path(__file__).name} <reference checkout>")
    ref = Path(sys.argv[1])
    G = load_reference(ref)
    rng = np.random.default_rng(0x31E)
    w4 = rng.integers(-8, 8, size=(K, N)).astype(np.int32)        # logical int4 [K, N]
    w8 = rng.integers(-127, 128, size=(K, N)).astype(np.int32)     # logical int8 [K, N]
    fam = G.FAMILIES
    u8i8 = G.Family("u8i8", "HmxU8I8ToU8MatMul", 8, 8, 8)
    out: dict[str, np.ndarray] = {"w4_kn": w4, "w8_kn": w8}

    def init(family, w, order="lohi", enc="twos", w8_order="raw", w8_dtype="uint8"):
        arr = G._weight_initializer(family, w, order, enc, None, w8_order, w8_dtype)
        return np.ascontiguousarray(arr).view(np.uint8).reshape(-1)

    # int4 carriers (the W4A8 HMX tile and every native W4A16 order, both nibble encodings)
    for order in ["lohi", "hilo"]:
        for enc in ["twos", "biased"]:
            out[f"w4a8__{order}__{enc}"] = init(fam["w4a8"], w4, order, enc)
    for order in ["native_kpair_lohi", "native_kpair_hilo", "native_nmajor_kpair_lohi", "native_nmajor_kpair_hilo",
                  "native_nmajor_k4_lohi", "native_nmajor_k4_hilo", "native_kblock32_nmajor_k4_lohi",
                  "native_kblock32_nmajor_k4_hilo", "native_npair_adjacent_nmajor_lohi",
                  "native_npair_adjacent_nmajor_hilo", "native_npair_tile32_nmajor_lohi",
                  "native_npair_tile32_nmajor_hilo", "native_full_codes"]:
        for enc in ["twos", "biased"]:
            out[f"w4a16__{order}__{enc}"] = init(fam["w4a16"], w4, order, enc)
    # LPBQ pre-chain inputs (HmxW4LpbqExpandToI8): K-pair weight bytes + per-block factors
    per_block = G._lpbq_block_scale_pattern("w4a16", K, N, 32)
    lp_w, lp_s = G._lpbq_initializers(w4, per_block, 32)
    out["lpbq__weight"] = np.ascontiguousarray(lp_w).view(np.uint8).reshape(-1)
    out["lpbq__scale"] = np.ascontiguousarray(lp_s).view(np.uint8).reshape(-1)
    out["lpbq__per_block_nb"] = per_block
    # int8 carriers
    for w8_order in ["raw", "kmajor", "kmajor_split128"]:
        for dt in ["uint8", "int8"]:
            out[f"w8a16__{w8_order}__{dt}"] = init(fam["w8a16"], w8, w8_order=w8_order, w8_dtype=dt)
    out["u8i8__raw__uint8"] = init(u8i8, w8)
    dst = Path(__file__).resolve().parent / "wire_formats.npz"
    np.savez_compressed(dst, **out)
    print(f"{dst}: {len(out)} arrays")


if __name__ == "__main__":
    main()
