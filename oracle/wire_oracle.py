"""Test infrastructure (the checker, never the product): CPU restatement of how the reference lays
int4 / int8 MatMul weights out in its QNN initializers (its "wire formats"), as the inverse map
wire bytes -> logical [K, N] weights.

Each layout is restated as the byte address and nibble of logical element (k, n), read off the
reference's packers in example/qnn_hmx_matmul_common/gen_quant_chain.py:
  * W8 K-major 32x32 tiles          ``_pack_w8_kmajor``                 :285-303
  * W8 per-128-channel streams      ``_pack_w8_kmajor_split128``        :306-314
  * W4 K-pairs [K/2, N]             ``_pack_w4_native_kpair_linear``    :369-382
  * W4 N-major K-pairs [N, K/2]     ``_pack_w4_native_nmajor_kpair_linear`` :385-398
  * W4 N32 tiles, k/k+4 pairs       ``_pack_w4_native_nmajor_k4_linear``    :401-422
  * W4 K32 blocks, N32, k/k+4       ``_pack_w4_native_kblock32_nmajor_k4_linear`` :425-452
  * W4 adjacent channel pairs       ``_pack_w4_native_npair_nmajor``        :455-468
  * W4 n / n+32 channel pairs       ``_pack_w4_native_npair_tile32_nmajor`` :471-489
  * W4 full codes [K, N]            ``_weight_initializer`` native_full_codes :619-627
  * W4A8 HMX 32x64 K-major tiles, byte = channels n | n+32   ``_weight_initializer`` :686-712
and the carrier transforms applied there: XOR 0x80 of every byte (:659, :713-717, :736-738), the
"hilo" orders (first element in the high nibble), and the "biased" nibble encoding v + 8 (:622-625).
The LPBQ pre-chain inputs (``_lpbq_initializers`` :350-366, HmxW4LpbqExpandToI8Op.cpp:1-15) are
K-pairs without XOR and factors [N, K/B] flattened: the library's own carriers.

Pinned against tests/golden/wire_formats.npz, bytes produced by the reference's packers
(tests/golden/make_wire_golden.py).
"""
from __future__ import annotations

import numpy as np

# format ids (== QhtpWireFormat in include/qhtp.h) and flags
W8_RAW_KN, W8_KMAJOR_TILE32, W8_KMAJOR_SPLIT128 = 1, 2, 3
W4_TILE32X64_NPAIR32, W4_KPAIR, W4_NMAJOR_KPAIR, W4_NMAJOR_K4, W4_KBLOCK32_NMAJOR_K4 = 4, 5, 6, 7, 8
W4_NPAIR_ADJACENT, W4_NPAIR_TILE32, W4_FULL_CODES = 9, 10, 11
XOR80, HILO, BIASED = 1, 2, 4

W8_FORMATS = {W8_RAW_KN, W8_KMAJOR_TILE32, W8_KMAJOR_SPLIT128}


def _kmajor32(k, n, N):
    kt, r, nt, c = k // 32, k % 32, n // 32, n % 32
    return (kt * (N // 32) + nt) * 1024 + (r // 4) * 128 + c * 4 + r % 4


def byte_and_nibble(fmt: int, k: np.ndarray, n: np.ndarray, K: int, N: int):
    """(byte address, nibble index 0 = low / 1 = high before HILO) of logical element (k, n)."""
    z = np.zeros_like(k)
    if fmt == W8_RAW_KN:
        return k * N + n, z
    if fmt == W8_KMAJOR_TILE32:
        return _kmajor32(k, n, N), z
    if fmt == W8_KMAJOR_SPLIT128:
        return (n // 128) * (K * 128) + _kmajor32(k, n % 128, 128), z
    if fmt == W4_TILE32X64_NPAIR32:
        nb, nc = n // 64, n % 64
        kt, kg, kr = k // 32, (k % 32) // 4, k % 4
        return (kt * (N // 64) + nb) * 1024 + kg * 128 + (nc % 32) * 4 + kr, (nc >= 32).astype(k.dtype)
    if fmt == W4_KPAIR:
        return (k // 2) * N + n, k & 1
    if fmt == W4_NMAJOR_KPAIR:
        return n * (K // 2) + k // 2, k & 1
    if fmt == W4_NMAJOR_K4:
        nb, nc, kg, kr = n // 32, n % 32, k // 8, k % 4
        return ((nb * (K // 8) + kg) * 32 + nc) * 4 + kr, ((k % 8) >= 4).astype(k.dtype)
    if fmt == W4_KBLOCK32_NMAJOR_K4:
        kb, kg, kr, nb, nc = k // 32, (k % 32) // 8, k % 4, n // 32, n % 32
        return (((kb * (N // 32) + nb) * 4 + kg) * 32 + nc) * 4 + kr, ((k % 8) >= 4).astype(k.dtype)
    if fmt == W4_NPAIR_ADJACENT:
        return (n // 2) * K + k, n & 1
    if fmt == W4_NPAIR_TILE32:
        return ((n // 64) * 32 + n % 32) * K + k, ((n % 64) >= 32).astype(k.dtype)
    if fmt == W4_FULL_CODES:
        return k * N + n, z
    raise ValueError(f"unknown wire format {fmt}")


def decode(fmt: int, flags: int, wire: np.ndarray, K: int, N: int) -> np.ndarray:
    """Wire bytes -> logical int32 weights [K, N]."""
    b = np.asarray(wire, np.uint8).reshape(-1)
    if flags & XOR80:
        b = b ^ np.uint8(0x80)
    k, n = np.meshgrid(np.arange(K), np.arange(N), indexing="ij")
    addr, nib = byte_and_nibble(fmt, k, n, K, N)
    v = b[addr].astype(np.int32)
    if fmt in W8_FORMATS:
        return np.where(v >= 128, v - 256, v)
    if fmt != W4_FULL_CODES and flags & HILO:
        nib = 1 - nib
    code = (v >> (4 * nib)) & 15
    if flags & BIASED:
        code ^= 8
    return np.where(code >= 8, code - 16, code)


def wire_bytes(fmt: int, K: int, N: int) -> int:
    return K * N if fmt in W8_FORMATS or fmt == W4_FULL_CODES else K * N // 2


def to_plain(fmt: int, w_kn: np.ndarray) -> np.ndarray:
    """Logical [K, N] -> the library's plain carrier: int8 [N, K] (W8 formats) or the int4 K-pair
    [K/2, N] bytes (low nibble = even k)."""
    if fmt in W8_FORMATS:
        return np.ascontiguousarray(w_kn.T).astype(np.int8)
    nib = (w_kn.astype(np.int32) & 15).astype(np.uint8)
    return (nib[0::2, :] | (nib[1::2, :] << 4)).astype(np.uint8)


def encode(fmt: int, flags: int, w_kn: np.ndarray) -> np.ndarray:
    """Logical [K, N] weights -> wire bytes (the packer direction, for tests on fresh cases)."""
    K, N = w_kn.shape
    k, n = np.meshgrid(np.arange(K), np.arange(N), indexing="ij")
    addr, nib = byte_and_nibble(fmt, k, n, K, N)
    out = np.zeros(wire_bytes(fmt, K, N), np.uint8)
    if fmt in W8_FORMATS:
        out[addr.reshape(-1)] = (w_kn.astype(np.int32) & 255).astype(np.uint8).reshape(-1)
    else:
        code = w_kn.astype(np.int32) & 15
        if flags & BIASED:
            code ^= 8
        if fmt != W4_FULL_CODES and flags & HILO:
            nib = 1 - nib
        np.bitwise_or.at(out, addr.reshape(-1), (code << (4 * nib)).astype(np.uint8).reshape(-1))
    if flags & XOR80:
        out ^= np.uint8(0x80)
    return out


# The reference's carriers in tests/golden/wire_formats.npz: key -> (format, flags)
def golden_cases() -> dict[str, tuple[int, int]]:
    cases = {}
    for hl, fh in (("lohi", 0), ("hilo", HILO)):
        for enc, fb in (("twos", 0), ("biased", BIASED)):
            cases[f"w4a8__{hl}__{enc}"] = (W4_TILE32X64_NPAIR32, XOR80 | fh | fb)
    orders = {"native_kpair": W4_KPAIR, "native_nmajor_kpair": W4_NMAJOR_KPAIR, "native_nmajor_k4": W4_NMAJOR_K4,
              "native_kblock32_nmajor_k4": W4_KBLOCK32_NMAJOR_K4, "native_npair_adjacent_nmajor": W4_NPAIR_ADJACENT,
              "native_npair_tile32_nmajor": W4_NPAIR_TILE32}
    for o, f in orders.items():
        for hl, fh in (("lohi", 0), ("hilo", HILO)):
            for enc, fb in (("twos", 0), ("biased", BIASED)):
                cases[f"w4a16__{o}_{hl}__{enc}"] = (f, XOR80 | fh | fb)
    for enc, fb in (("twos", 0), ("biased", BIASED)):
        cases[f"w4a16__native_full_codes__{enc}"] = (W4_FULL_CODES, fb)
    cases["lpbq__weight"] = (W4_KPAIR, 0)
    for o, f in (("raw", W8_RAW_KN), ("kmajor", W8_KMAJOR_TILE32), ("kmajor_split128", W8_KMAJOR_SPLIT128)):
        for dt in ("uint8", "int8"):
            cases[f"w8a16__{o}__{dt}"] = (f, 0)
    cases["u8i8__raw__uint8"] = (W8_RAW_KN, XOR80)
    return cases
