"""Quantized MatMul oracle (TEST INFRASTRUCTURE ONLY -- the parity checker, never the product).

Two things live here.

1. A restatement of the reference's case generator,
   ``scripts/generate_qnn_matmul_python_cases.py`` (cited per function below).
   It reproduces the reference's seeded float cases and AIMET/QNN affine
   quantization bit for bit.  The RNG call sequence and the scale formulas must
   match the reference exactly, or the generated codes differ.  The golden
   fixtures in ``tests/golden`` pin this: they hold sha256 digests of the
   reference's own arrays, made by importing the reference script.

2. The exact integer/requant model that defines "bit-exact".  The reference
   oracle computes, in float64,

       y = ((x_q + off_A) * s_A) @ w_deq.T + bias_q * (s_A * s_W)
       out = clip(rint(y / s_O - off_O), 0, qmax)          (off = -zero_point)

   with ``w_deq = float32(q * s_W)`` (generate_qnn_matmul_python_cases.py:307,361).
   Write the float32 scale as ``s_W = m_s * 2**e_s`` (integer m_s < 2**24).  Then
   ``w_deq = (q*m_s + e') * 2**e_s``, where ``e'`` is the float32 rounding error
   of ``q*m_s`` in units of 2**e_s.  It is an integer with ``|e'| <= 64`` for
   ``|q| <= 128``.  The whole real value is then

       y* = s_A * 2**e_s * T,   T = m_s * (sum_k (x_q-zp)*q + bias_q) + sum_k (x_q-zp)*e'

   with T an exact int64.  The output is ``clip(round_half_even(y*/s_O + zp_O))``,
   evaluated exactly: a float64 fast path, and an exact rational check for
   anything within 1e-9 of a rounding tie.  This model reproduces the
   reference's ``output_ref_q`` on every generated case (pinned by the golden
   tests).  The GPU kernels compute the same T with int8 tensor-core
   products: the ``q`` plane and the ``e'`` residual plane.

   ``dequant="exact"`` (used for W16A16, which has no f32-dequant reference)
   drops e' and takes the weight dequant ``q*s_W`` exactly:
   ``y* = s_A*s_W*(sum (x_q-zp)*q16 + bias_q)``
   (docs/w16a16_is_two_w8a16.md:14-36, scripts/verify_w16a16_two_w8a16.py:21-48).
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass
from fractions import Fraction

import numpy as np

# ----------------------------------------------------------------------------------------------
# 1. Family table and seeded case generator (restated from the reference)
# ----------------------------------------------------------------------------------------------


@dataclass(frozen=True)
class Family:
    """One quantized MatMul family (generate_qnn_matmul_python_cases.py:27-71).

    act zero-point is 2**(bits-1); u8 outputs have zero-point 0, u16 outputs 32768;
    weights are signed symmetric with qmax = 2**(bits-1)-1.
    """

    name: str
    act_bits: int
    weight_bits: int
    out_bits: int
    schema: str = "per_channel"  # "per_channel" | "lpbq" | "per_group"
    kernel: str = ""
    lpbq_block: int = 32

    @property
    def act_zp(self) -> int:
        return 1 << (self.act_bits - 1)

    @property
    def out_zp(self) -> int:
        return 32768 if self.out_bits == 16 else 0

    @property
    def act_qmax(self) -> int:
        return (1 << self.act_bits) - 1

    @property
    def out_qmax(self) -> int:
        return (1 << self.out_bits) - 1

    @property
    def weight_qmax(self) -> int:
        return (1 << (self.weight_bits - 1)) - 1

    @property
    def act_dtype(self):
        return np.dtype("<u2") if self.act_bits == 16 else np.dtype(np.uint8)

    @property
    def out_dtype(self):
        return np.dtype("<u2") if self.out_bits == 16 else np.dtype(np.uint8)

    def with_block(self, block: int) -> "Family":
        return Family(self.name, self.act_bits, self.weight_bits, self.out_bits, self.schema,
                      self.kernel, block)


# generate_qnn_matmul_python_cases.py:74-125, plus W16A16 (docs/w16a16_is_two_w8a16.md).
FAMILIES = {
    "u8i8": Family("u8i8", 8, 8, 8, "per_channel", "u8i8"),
    "w4a8_per_channel": Family("w4a8_per_channel", 8, 4, 8, "per_channel", "w4a8"),
    "w4a8_per_group": Family("w4a8_per_group", 8, 4, 8, "per_group", "w4a8"),
    "w4a8_lpbq": Family("w4a8_lpbq", 8, 4, 8, "lpbq", "w4a8"),
    "w8a16": Family("w8a16", 16, 8, 16, "per_channel", "w8a16"),
    "w4a16_per_channel": Family("w4a16_per_channel", 16, 4, 16, "per_channel", "w4a16"),
    "w4a16_per_group": Family("w4a16_per_group", 16, 4, 16, "per_group", "w4a16"),
    "w4a16_lpbq": Family("w4a16_lpbq", 16, 4, 16, "lpbq", "w4a16"),
    "w16a16": Family("w16a16", 16, 16, 16, "per_channel", "w16a16"),
}

# Families the reference's python-case generator covers (per_group is generated there but its
# bias is "not modeled" (:460-470); it is outside the promoted gates).
REFERENCE_GENERATED = ("u8i8", "w4a8_per_channel", "w4a8_per_group", "w4a8_lpbq", "w8a16",
                       "w4a16_per_channel", "w4a16_per_group", "w4a16_lpbq")

# generate_qnn_matmul_python_cases.py:128-136
CASES = ("normal_random", "zp_neutral", "positive_boundary", "negative_boundary",
         "single_k_impulse", "bias_only", "scale_only")


def seed_for(family: str, case: str) -> int:
    """Polynomial string hash seeded with 0x5EED (generate_qnn_matmul_python_cases.py:225-229)."""
    h = 0x5EED
    for c in f"{family}:{case}".encode("ascii"):
        h = (h * 131 + c) & 0xFFFFFFFF
    return h


def make_float_case(fam: Family, case: str, m: int, k: int, n: int):
    """Float x[M,K], w[N,K], bias[N] for one case (generate_qnn_matmul_python_cases.py:236-285).

    The order of RNG draws follows the reference exactly; changing it changes every code.
    """
    rng = np.random.default_rng(seed_for(fam.name, case))
    ww = 1.0 if fam.weight_bits == 8 else 0.75
    aw = 1.0 if fam.act_bits == 16 else 0.85
    f32 = np.float32

    def uni(lo, hi, shape):
        return rng.uniform(lo, hi, size=shape).astype(f32)

    if case == "normal_random":
        x = uni(-aw, aw, (m, k)); w = uni(-ww, ww, (n, k)); b = uni(-0.05, 0.05, n)
    elif case == "zp_neutral":
        x = np.zeros((m, k), f32); w = uni(-ww, ww, (n, k)); b = np.zeros(n, f32)
    elif case == "positive_boundary":
        x = uni(0.75 * aw, aw, (m, k)); w = uni(0.75 * ww, ww, (n, k)); b = uni(0.05, 0.15, n)
    elif case == "negative_boundary":
        x = uni(0.75 * aw, aw, (m, k)); w = uni(-ww, -0.75 * ww, (n, k)); b = uni(-0.15, -0.05, n)
    elif case == "single_k_impulse":
        col = 1 % k
        x = np.zeros((m, k), f32); x[:, col] = 0.25 * aw
        w = np.zeros((n, k), f32); w[:, col] = uni(-ww, ww, n)
        b = np.zeros(n, f32)
    elif case == "bias_only":
        x = uni(-0.1 * aw, 0.1 * aw, (m, k)); w = uni(-0.1 * ww, 0.1 * ww, (n, k))
        b = uni(-0.75, 0.75, n)
    elif case == "scale_only":
        x = uni(-3.0 * aw, 3.0 * aw, (m, k)); w = uni(-2.5 * ww, 2.5 * ww, (n, k))
        b = np.zeros(n, f32)
    else:
        raise ValueError(f"unknown case {case!r}")
    return x, w, b


def affine_scale(vmin: float, vmax: float, qmin: int, qmax: int, zp: int) -> float:
    """Fixed-zero-point affine scale (generate_qnn_matmul_python_cases.py:174-182)."""
    s = 1.0e-12
    if vmin < 0 and zp > qmin:
        s = max(s, -vmin / float(zp - qmin))
    if vmax > 0 and qmax > zp:
        s = max(s, vmax / float(qmax - zp))
    return s


def symmetric_scale(vmin: float, vmax: float, qmax: int) -> float:
    """Symmetric scale (generate_qnn_matmul_python_cases.py:185-186)."""
    return max(abs(vmin), abs(vmax), 1.0e-12) / float(qmax)


def lpbq_factorize(group_scales: np.ndarray, max_int: int = 16):
    """Per-channel base scale x integer block factors (generate_qnn_matmul_python_cases.py:189-200)."""
    gmax = max(float(group_scales.max()), 1.0e-12)
    gmin = max(float(group_scales.min()), 1.0e-12)
    base = max(gmin, gmax / float(max_int))
    f = np.ceil(group_scales.astype(np.float64) / base - 1.0e-9)
    return base, np.clip(f, 1, max_int).astype(np.uint8)


def quantize_affine(v: np.ndarray, scale: float, qnn_offset: int, qmax: int, dtype) -> np.ndarray:
    """AIMET/QNN affine quantize: clip(rint(v/scale - offset)) (generate_qnn_matmul_python_cases.py:203-218)."""
    q = np.rint(v.astype(np.float64) / scale - qnn_offset)
    return np.clip(q, 0, qmax).astype(dtype)


def quantize_weight(fam: Family, w: np.ndarray):
    """Quantize w[N,K] (generate_qnn_matmul_python_cases.py:288-423).

    Returns dict with q [N,K] (int8/int16; LPBQ: the compressed int4 codes),
    scale [N] (or [N,G] for per_group) float32, and for LPBQ the block factors
    [N, K/B] uint8 and the expanded codes q*f [N,K] int16.
    """
    n, k = w.shape
    qmax = fam.weight_qmax
    qdt = np.int8 if qmax <= 127 else np.int16
    out = {}
    if fam.schema == "per_channel":
        scales = np.empty(n, np.float32)
        q = np.empty((n, k), qdt)
        for r in range(n):
            row = w[r]
            s = symmetric_scale(float(row.min()), float(row.max()), qmax)
            scales[r] = s
            q[r] = np.clip(np.rint(row.astype(np.float64) / s), -qmax, qmax).astype(qdt)
        out.update(q=q, scale=scales)
        return out
    if fam.schema == "lpbq":
        bs = fam.lpbq_block
        if k <= bs or k % bs:
            raise ValueError(f"{fam.name}: LPBQ K={k} must be > {bs} and a multiple of it")
        nb = k // bs
        gscale = np.empty((n, nb), np.float32)
        scales = np.empty(n, np.float32)
        factors = np.empty((n, nb), np.uint8)
        q = np.empty((n, k), qdt)
        expanded = np.empty((n, k), np.int16)
        for r in range(n):
            row = w[r]
            for b in range(nb):
                blk = row[b * bs:(b + 1) * bs]
                gscale[r, b] = symmetric_scale(float(blk.min()), float(blk.max()), qmax)
            base, f = lpbq_factorize(gscale[r])
            scales[r] = base
            factors[r] = f
            for b in range(nb):
                sl = slice(b * bs, (b + 1) * bs)
                eff = float(base) * float(int(f[b]))
                qb = np.clip(np.rint(row[sl].astype(np.float64) / eff), -qmax, qmax).astype(qdt)
                q[r, sl] = qb
                expanded[r, sl] = qb.astype(np.int16) * np.int16(int(f[b]))
        out.update(q=q, scale=scales, lpbq_factor=factors, expanded=expanded, group_scale=gscale)
        return out
    if fam.schema == "per_group":
        gs = 64
        if k <= gs or k % gs:
            raise ValueError(f"{fam.name}: W4 K={k} must be > {gs} and a multiple of it")
        ng = k // gs
        scales = np.empty((n, ng), np.float32)
        q = np.empty((n, k), qdt)
        for r in range(n):
            for g in range(ng):
                blk = w[r, g * gs:(g + 1) * gs]
                s = symmetric_scale(float(blk.min()), float(blk.max()), qmax)
                scales[r, g] = s
                q[r, g * gs:(g + 1) * gs] = np.clip(np.rint(blk.astype(np.float64) / s),
                                                   -qmax, qmax).astype(qdt)
        out.update(q=q, scale=scales)
        return out
    raise ValueError(fam.schema)


def quantize_weight_fast(fam: Family, w: np.ndarray):
    """Vectorized ``quantize_weight`` for large synthetic cases (per_channel and lpbq only).

    Same float64 formulas in the same order, over whole arrays instead of per-channel loops;
    ``test_quantize_weight_fast_matches_loop`` checks equality with the loop version."""
    n, k = w.shape
    qmax = fam.weight_qmax
    qdt = np.int8 if qmax <= 127 else np.int16
    w64 = w.astype(np.float64)
    if fam.schema == "per_channel":
        mx = np.maximum(np.maximum(np.abs(w.min(axis=1).astype(np.float64)),
                                   np.abs(w.max(axis=1).astype(np.float64))), 1.0e-12)
        s = mx / float(qmax)
        q = np.clip(np.rint(w64 / s[:, None]), -qmax, qmax).astype(qdt)
        return dict(q=q, scale=s.astype(np.float32))
    if fam.schema != "lpbq":
        raise NotImplementedError(fam.schema)
    bs = fam.lpbq_block
    if k <= bs or k % bs:
        raise ValueError(f"{fam.name}: LPBQ K={k} must be > {bs} and a multiple of it")
    nb = k // bs
    wb = w.reshape(n, nb, bs)
    mx = np.maximum(np.maximum(np.abs(wb.min(axis=2).astype(np.float64)),
                               np.abs(wb.max(axis=2).astype(np.float64))), 1.0e-12)
    gscale = (mx / float(qmax)).astype(np.float32)
    g64 = gscale.astype(np.float64)
    gmax = np.maximum(g64.max(axis=1), 1.0e-12)
    gmin = np.maximum(g64.min(axis=1), 1.0e-12)
    base = np.maximum(gmin, gmax / 16.0)
    f = np.clip(np.ceil(g64 / base[:, None] - 1.0e-9), 1, 16).astype(np.uint8)
    eff = base[:, None] * f.astype(np.float64)
    q = np.clip(np.rint(w64.reshape(n, nb, bs) / eff[:, :, None]), -qmax, qmax).astype(qdt).reshape(n, k)
    expanded = (q.astype(np.int16).reshape(n, nb, bs) * f.astype(np.int16)[:, :, None]).reshape(n, k)
    return dict(q=q, scale=base.astype(np.float32), lpbq_factor=f, expanded=expanded, group_scale=gscale)


def weight_deq_f32(fam: Family, wq: dict) -> np.ndarray:
    """float32 dequantized weight exactly as the reference forms it
    (generate_qnn_matmul_python_cases.py:307,361,410): float32(q) * float32(scale)."""
    if fam.schema == "per_channel":
        return wq["q"].astype(np.float32) * wq["scale"][:, None]
    if fam.schema == "lpbq":
        return wq["expanded"].astype(np.float32) * wq["scale"][:, None]
    gs = wq["q"].shape[1] // wq["scale"].shape[1]
    return wq["q"].astype(np.float32) * np.repeat(wq["scale"], gs, axis=1)


@dataclass
class QuantCase:
    """One quantized case: every tensor an op call consumes, plus the reference's own float64 answer."""

    family: Family
    act_q: np.ndarray          # [M,K] u8 / u16
    weight_q: np.ndarray       # [N,K] int8 / int16 (LPBQ: compressed int4 codes)
    weight_scale: np.ndarray   # [N] float32 ([N,G] for per_group)
    bias_q: np.ndarray         # [N] int32
    act_scale: float
    out_scale: float
    lpbq_factor: np.ndarray | None = None     # [N, K/B] uint8
    lpbq_expanded: np.ndarray | None = None   # [N, K] int16
    bias_float: np.ndarray | None = None      # per_group only (bias kept float there)
    ref_output_q: np.ndarray | None = None    # reference float64-formula output
    act_zp_free: int | None = None            # a free (min/max-derived) activation zero point, else the family's
    out_zp_free: int | None = None            # a free output zero point, else the family's

    @property
    def act_zp(self) -> int:
        return self.family.act_zp if self.act_zp_free is None else int(self.act_zp_free)

    @property
    def out_zp(self) -> int:
        return self.family.out_zp if self.out_zp_free is None else int(self.out_zp_free)

    @property
    def act_offset(self) -> int:
        return -self.act_zp

    @property
    def out_offset(self) -> int:
        return -self.out_zp

    def with_act(self, act_q: np.ndarray) -> "QuantCase":
        """The same weights, scales and encodings with another activation (rows, chain steps)."""
        return QuantCase(self.family, act_q, self.weight_q, self.weight_scale, self.bias_q, self.act_scale,
                         self.out_scale, self.lpbq_factor, self.lpbq_expanded, self.bias_float, None,
                         self.act_zp_free, self.out_zp_free)

    @property
    def mma_weight(self) -> np.ndarray:
        """Integer weight codes that multiply the activation: LPBQ uses q*f (int8 range)."""
        return self.lpbq_expanded if self.family.schema == "lpbq" else self.weight_q


def quantize_case(fam: Family, x: np.ndarray, w: np.ndarray, bias: np.ndarray,
                  with_reference_output: bool = True, fast: bool = False,
                  range_rows: int | None = None) -> QuantCase:
    """Quantize a float case (generate_qnn_matmul_python_cases.py:426-481).

    ``fast`` uses the vectorized weight quantizer; ``range_rows`` derives the output scale from the
    float output of the first ``range_rows`` rows only (large synthetic benchmark cases)."""
    xr = x if range_rows is None else x[:range_rows]
    y_float = xr.astype(np.float64) @ w.astype(np.float64).T + bias.astype(np.float64)
    s_a = affine_scale(float(x.min()), float(x.max()), 0, fam.act_qmax, fam.act_zp)
    s_o = affine_scale(float(y_float.min()), float(y_float.max()), 0, fam.out_qmax, fam.out_zp)
    act_q = quantize_affine(x, s_a, -fam.act_zp, fam.act_qmax, fam.act_dtype)
    wq = quantize_weight_fast(fam, w) if fast else quantize_weight(fam, w)
    bias_float = None
    if wq["scale"].ndim == 1:
        bscale = s_a * wq["scale"].astype(np.float64)
        bias_q = np.clip(np.rint(bias.astype(np.float64) / bscale), -(1 << 31), (1 << 31) - 1)
        bias_q = bias_q.astype(np.int32)
        bias_deq = bias_q.astype(np.float64) * bscale
    else:
        bias_q = np.zeros(bias.shape, np.int32)
        bias_deq = bias.astype(np.float64)
        bias_float = bias.astype(np.float32)
    ref = None
    if with_reference_output:
        x_deq = (act_q.astype(np.float64) - fam.act_zp) * s_a
        y = x_deq @ weight_deq_f32(fam, wq).astype(np.float64).T + bias_deq
        ref = quantize_affine(y, s_o, -fam.out_zp, fam.out_qmax, fam.out_dtype)
    return QuantCase(fam, act_q, wq["q"], wq["scale"], bias_q, s_a, s_o,
                     wq.get("lpbq_factor"), wq.get("expanded"), bias_float, ref)


def generate_case(family: str | Family, case: str, m: int, k: int, n: int,
                  lpbq_block: int | None = None, with_reference_output: bool = True) -> QuantCase:
    fam = FAMILIES[family] if isinstance(family, str) else family
    if lpbq_block is not None:
        fam = fam.with_block(lpbq_block)
    x, w, b = make_float_case(fam, case, m, k, n)
    return quantize_case(fam, x, w, b, with_reference_output)


# ----------------------------------------------------------------------------------------------
# 2. BASELINE.json synthetic distributions (normal activations/weights; LPBQ block 64)
# ----------------------------------------------------------------------------------------------


def make_baseline_case(family: str, m: int, k: int, n: int, seed: int = 0x6D6D,
                       lpbq_block: int = 64, w_sigma: float | None = None,
                       with_reference_output: bool = False) -> QuantCase:
    """X~N(0,1) asymmetric-quantized activations, W~N(0,sigma)
    (0.05 for 8-bit, 0.02 for LPBQ int4), bias~N(0,0.1).  Quantization follows the
    same affine/symmetric/LPBQ rules as the reference generator."""
    fam = FAMILIES[family]
    if fam.schema == "lpbq":
        fam = fam.with_block(lpbq_block)
    sigma = w_sigma if w_sigma is not None else (0.02 if fam.weight_bits == 4 else 0.05)
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(sigma)).astype(np.float32)
    b = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    big = m * k * n > (1 << 31)
    if big:
        with_reference_output = False
    return quantize_case(fam, x, w, b, with_reference_output, fast=True, range_rows=256 if big else None)


def qnn_asymmetric_encoding(vmin: float, vmax: float, bits: int = 8) -> tuple[float, int]:
    """QNN/AIMET asymmetric encoding from a float range: the range is widened to hold 0,
    scale = (max - min) / (2^bits - 1), zero point = -round(min / scale) (QNN offset = -zero point,
    dequant (q + offset) * scale, the convention of generate_qnn_matmul_python_cases.py:203-218).
    The zero point is then free in [0, 2^bits - 1] instead of the families' fixed 2^(bits-1)."""
    lo, hi = min(float(vmin), 0.0), max(float(vmax), 0.0)
    qmax = (1 << bits) - 1
    scale = max((hi - lo) / qmax, 1.0e-12)
    zp = int(np.clip(-np.rint(lo / scale), 0, qmax))
    return scale, zp


def make_free_offset_u8i8_case(m: int = 256, k: int = 256, n: int = 256, seed: int = 0x5EED0,
                               x_shift: float = 0.0) -> QuantCase:
    """u8i8 with free asymmetric activation and output encodings.

    X ~ N(0,1) (+ x_shift, which moves the activation zero point), quantized u8 with scale
    (max - min)/255 and zero point -round(min/scale); W ~ N(0, 0.05) quantized symmetric int8 with ONE
    per-tensor scale max|W|/127 (given to the op as N equal per-channel scales); bias ~ N(0, 0.1)
    quantized int32 at s_x * s_w; output Y = X W^T + b requantized u8 with the scale and zero point of
    Y's float min/max, round half to even.  The float64 answer follows the reference oracle's
    quantized path (generate_qnn_matmul_python_cases.py:426-481) with these encodings:
    y = ((x_q - zp_x) s_x) @ float32(q s_w)^T + bias_q s_x s_w, out = clip(rint(y / s_o + zp_o)).
    """
    fam = FAMILIES["u8i8"]
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((m, k), dtype=np.float32) + np.float32(x_shift)).astype(np.float32)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    b = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    y_float = x.astype(np.float64) @ w.astype(np.float64).T + b.astype(np.float64)
    s_x, zp_x = qnn_asymmetric_encoding(float(x.min()), float(x.max()))
    s_o, zp_o = qnn_asymmetric_encoding(float(y_float.min()), float(y_float.max()))
    act_q = quantize_affine(x, s_x, -zp_x, 255, np.uint8)
    s_w = np.float32(symmetric_scale(float(w.min()), float(w.max()), 127))
    q = np.clip(np.rint(w.astype(np.float64) / np.float64(s_w)), -127, 127).astype(np.int8)
    scales = np.full(n, s_w, np.float32)
    bscale = s_x * np.float64(s_w)
    bias_q = np.clip(np.rint(b.astype(np.float64) / bscale), -(1 << 31), (1 << 31) - 1).astype(np.int32)
    x_deq = (act_q.astype(np.float64) - zp_x) * s_x
    w_deq = (q.astype(np.float32) * scales[:, None]).astype(np.float64)
    y = x_deq @ w_deq.T + bias_q.astype(np.float64) * bscale
    ref = quantize_affine(y, s_o, -zp_o, 255, np.uint8)
    return QuantCase(fam, act_q, q, scales, bias_q, s_x, s_o, ref_output_q=ref, act_zp_free=zp_x,
                     out_zp_free=zp_o)


# ----------------------------------------------------------------------------------------------
# 3. Prepared record ("sidecar") and the exact requant model
# ----------------------------------------------------------------------------------------------

RECORD_DTYPE = np.dtype([("beff", "<i8"), ("cmn", "<u8"), ("m_q", "<i4"), ("wbits", "<u4"),
                         ("tn", "<i4"), ("lo_win", "<i4")])   # 32 bytes / output channel


def split_f32(scale: np.ndarray):
    """float32 scale -> (m, e) with scale == m * 2**e exactly, 0 < m < 2**24 integer."""
    s = np.asarray(scale, np.float32).astype(np.float64)
    if np.any(~np.isfinite(s)) or np.any(s <= 0):
        raise ValueError("weight scales must be finite and > 0")
    fr, ex = np.frexp(s)                       # s = fr * 2**ex, fr in [0.5, 1)
    m = np.ldexp(fr, 24).astype(np.int64)      # exact: float32 has a 24-bit significand
    e = ex.astype(np.int64) - 24
    assert np.all(np.ldexp(m.astype(np.float64), e) == s)
    return m, e


def round_to_24_bits(p: np.ndarray) -> np.ndarray:
    """Round integers |p| < 2**53 to 24 significant bits, ties to even (== int -> float32 -> int)."""
    p = np.asarray(p, np.int64)
    a = np.abs(p)
    bl = np.zeros_like(a)
    nz = a > 0
    bl[nz] = np.frexp(a[nz].astype(np.float64))[1]         # bit length (exact for a < 2**53)
    sh = np.maximum(bl - 24, 0)
    unit = np.left_shift(np.int64(1), sh)
    q, r = np.divmod(a, unit)
    half = unit // 2
    up = (r > half) | ((r == half) & (sh > 0) & (q % 2 == 1))
    return np.sign(p) * (q + up) * unit


def residual_plane(q: np.ndarray, m_s: np.ndarray) -> np.ndarray:
    """e'[n,k] = round24(q*m_s) - q*m_s: the float32 rounding error of the weight dequant,
    in units of 2**e_s.  |e'| <= 64 for |q| <= 128, so it is an int8 plane."""
    p = q.astype(np.int64) * m_s.astype(np.int64)[:, None]
    e = round_to_24_bits(p) - p
    assert np.abs(e).max(initial=0) <= 64
    return e.astype(np.int8)


def prepare_record(case: QuantCase, dequant: str = "f32", return_c: bool = False):
    """Per-output-channel prepared record (the B200 "sidecar") and the e' plane.

    beff  : effective bias in T units.  f32 mode: m_s*(bias_q - zp*sum q) - zp*sum e';
            exact mode: bias_q - zp*sum q   (docs/qnn_custom_op_matmul_e2e.md:345-355 folds the
            activation zero-point into the bias the same way: bias_q - zp_act*sum_k w)
    cmn, tn : the float64 requant multiplier c (float64(s_A*2**e_s / s_O) in f32 mode,
            float64(float64(s_A*s_W)/s_O) in exact mode), written c = cm * 2**-cshift with cm its
            53-bit integer mantissa, stored for the fixed-point fast path as (|T| << tn) * cmn *
            2**-96: tn = 96 - cshift, cmn = cm; for c < 2**-44, tn = 0 and cmn = cm * 2**(96 -
            cshift) rounded half up
    m_q   : multiplier of the q-plane accumulator inside T (m_s in f32 mode, 1 in exact mode)
    wbits : the float32 weight scale's bits (its mantissa m_s and exponent e_s feed the exact tie
            check: z* - zp_out = T*mul*mant(s_A)*2**(e_s + exp(s_A)) / s_O, mul = 1 or m_s)
    lo_win: f32 mode with u16 activations: a bound on the lo-byte-plane x e' part of T, in output
            units of 2**-30: |sum_k x_lo*e'| * c <= 255 * sum_k |e'| * c, stored as
            ceil(255 * sum|e'| * c * 2**30) + 1 (capped at 2**30), the products rounded in that order;
            0 otherwise.  A GEMM may leave that product out of its MMAs and compute it exactly only
            for the elements whose value lies within this window of a rounding boundary.
    """
    fam = case.family
    if fam.schema == "per_group":
        raise NotImplementedError("per_group schema has no per-channel record")
    wq = case.mma_weight.astype(np.int64)
    zp = case.act_zp
    m_s, e_s = split_f32(case.weight_scale)
    rec = np.zeros(wq.shape[0], RECORD_DTYPE)
    sum_q = wq.sum(axis=1)
    bias = case.bias_q.astype(np.int64)
    if dequant == "f32":
        ep = residual_plane(wq, m_s)
        sum_e = ep.astype(np.int64).sum(axis=1)
        rec["beff"] = m_s * (bias - zp * sum_q) - zp * sum_e
        c = np.ldexp(np.float64(case.act_scale), e_s) / np.float64(case.out_scale)
        rec["m_q"] = m_s
        mul = np.ones_like(m_s)
        if fam.act_bits == 16:
            sum_abs = np.abs(ep.astype(np.int64)).sum(axis=1)
            x = (255 * sum_abs).astype(np.float64) * c * 1073741824.0
            rec["lo_win"] = np.where(x >= 1073741824.0, 1 << 30, np.ceil(np.minimum(x, 2.0 ** 30)).astype(np.int64) + 1)
    elif dequant == "exact":
        ep = None
        rec["beff"] = bias - zp * sum_q
        c = (np.float64(case.act_scale) * case.weight_scale.astype(np.float64)) / np.float64(case.out_scale)
        rec["m_q"] = 1
        mul = m_s
    else:
        raise ValueError(dequant)
    fc, ec = np.frexp(c)
    cm = np.ldexp(fc, 53).astype(np.uint64)
    cshift = (53 - ec).astype(np.int64)
    if np.any(cshift < 34):
        raise ValueError("requant multiplier c >= 2**18 is outside the supported range")
    small = cshift > 96
    d = np.where(small, cshift - 96, 0)
    cmn = cm.copy()
    with np.errstate(over="ignore"):
        rounded = (cm + (np.uint64(1) << np.maximum(d - 1, 0).astype(np.uint64))) >> d.astype(np.uint64)
    cmn[small] = np.where(d[small] >= 64, 0, rounded[small])
    rec["cmn"] = cmn
    rec["tn"] = np.where(small, 0, 96 - cshift)
    rec["wbits"] = np.asarray(case.weight_scale, np.float32).view(np.uint32)
    if return_c:
        return rec, ep, c, mul
    return rec, ep


def _exact_round(tpre: int, mul: int, e_s: int, s_a: float, s_o: float, zp_out: int) -> int:
    """round_half_even(tpre*mul*s_A*2**e_s/s_O + zp_out) in exact rational arithmetic."""
    z = Fraction(int(tpre) * int(mul)) * Fraction(s_a) * (Fraction(2) ** int(e_s)) / Fraction(s_o)
    z += zp_out
    return round(z)        # Python rounds Fractions half to even


TIE_EPS = 1e-9


def exact_output(case: QuantCase, dequant: str = "f32", return_t: bool = False):
    """Bit-exact output codes of the exact requant model (see module docstring)."""
    fam = case.family
    rec, ep, c, mul = prepare_record(case, dequant, return_c=True)
    xq = case.act_q.astype(np.float64)
    wq = case.mma_weight.astype(np.float64)
    # integer GEMMs in float64: every product and partial sum is an integer < 2**53 -> exact
    p = (xq @ wq.T).astype(np.int64)                       # sum_k x_q*q  (zero-point is in beff)
    tpre = rec["m_q"].astype(np.int64)[None, :] * p + rec["beff"][None, :]
    if ep is not None:
        tpre += (xq @ ep.astype(np.float64).T).astype(np.int64)
    z = tpre.astype(np.float64) * c[None, :] + case.out_zp
    r = np.rint(z)
    frac = z - np.floor(z)
    near = (np.abs(frac - 0.5) <= TIE_EPS) & (z > -1.0) & (z < fam.out_qmax + 1.0)
    if near.any():
        m_s, e_s = split_f32(case.weight_scale)
        for i, j in zip(*np.nonzero(near)):
            r[i, j] = _exact_round(int(tpre[i, j]), int(mul[j]), int(e_s[j]),
                                   case.act_scale, case.out_scale, case.out_zp)
    out = np.clip(r, 0, fam.out_qmax).astype(fam.out_dtype)
    if return_t:
        return out, tpre, int(near.sum())
    return out


def per_group_output(case: QuantCase) -> np.ndarray:
    """Output codes of the per-group W4 schema (generate_qnn_matmul_python_cases.py:392-423 weights,
    :460-470 float bias, :472-481 output), in the operation order the GPU uses.

    The reference computes y = x_deq @ w_deq.T + bias in float64 with w_deq = float32(q*s[n,g]).
    Each group scale is s = m*2**e, so float32(q*s) = (q*m + e')*2**e exactly (e' = residual_plane
    per group), and a group's contribution to a row is the exact integer

        Z[g] = m*sum_g((x-zp)*q) + sum_g((x-zp)*e')          times 2**e[n,g].

    Here acc = sum over g in K order of Z[g]*2**e (each term exact, one float64 rounding per
    addition), y = act_scale*acc + float64(bias), out = clip(rint(y/out_scale + zp_O)).  This
    sequence reproduces the reference's output_ref_q on its per-group golden cases (the reference
    sums inexact float64 products in BLAS order; the two agree except within float64 rounding of a
    tie)."""
    fam = case.family
    if fam.schema != "per_group":
        raise ValueError("per_group_output: per-group families only")
    q = case.weight_q.astype(np.int64)
    n, k = q.shape
    g_count = k // 64
    m_s, e_s = split_f32(case.weight_scale)                   # [N, G]
    p = (q.reshape(n, g_count, 64) * m_s[:, :, None]).reshape(n, k)
    ep = round_to_24_bits(p) - p                              # e' per group, |e'| <= 8
    xz = (case.act_q.astype(np.int64) - case.act_zp).astype(np.float64)
    acc = np.zeros((case.act_q.shape[0], n))
    for g in range(g_count):
        sl = slice(64 * g, 64 * (g + 1))
        sq = (xz[:, sl] @ q[:, sl].astype(np.float64).T).astype(np.int64)   # exact: |.| < 2**53
        se = (xz[:, sl] @ ep[:, sl].astype(np.float64).T).astype(np.int64)
        z = m_s[None, :, g] * sq + se
        acc = acc + np.ldexp(z.astype(np.float64), e_s[None, :, g])
    y = case.act_scale * acc + case.bias_float.astype(np.float64)[None, :]
    r = np.rint(y / case.out_scale + case.out_zp)
    return np.clip(r, 0, fam.out_qmax).astype(fam.out_dtype)


def integer_accumulator(case: QuantCase) -> np.ndarray:
    """sum_k (x_q - zp) * q as int64 -- the W16A16 identity target."""
    xc = case.act_q.astype(np.int64) - case.act_zp
    return (xc.astype(np.float64) @ case.mma_weight.astype(np.float64).T).astype(np.int64)


# ----------------------------------------------------------------------------------------------
# 4. Weight packing formats accepted by the C ABI
# ----------------------------------------------------------------------------------------------


def pack_int4_kpair(q_nk: np.ndarray) -> np.ndarray:
    """int4 codes [N,K] -> K-pair bytes [K/2, N]: byte (k>>1)*N + n, even k in the low nibble
    (the LPBQ carrier of example/qnn_hmx_matmul_common/HmxW4LpbqExpandToI8Op.cpp:5,32-40)."""
    n, k = q_nk.shape
    if k % 2:
        raise ValueError("K must be even for int4 packing")
    nib = (q_nk.astype(np.int16) & 0xF).astype(np.uint8)   # two's complement nibble
    lo = nib[:, 0::2]
    hi = nib[:, 1::2]
    return np.ascontiguousarray((lo | (hi << 4)).T)


def unpack_int4_kpair(packed: np.ndarray, n: int, k: int) -> np.ndarray:
    """Inverse of pack_int4_kpair -> int8 [N,K] (two's-complement nibbles)."""
    p = packed.reshape(k // 2, n).T
    lo = (p & 0xF).astype(np.int16)
    hi = (p >> 4).astype(np.int16)
    q = np.empty((n, k), np.int16)
    q[:, 0::2] = lo
    q[:, 1::2] = hi
    q[q >= 8] -= 16
    return q.astype(np.int8)


def lpbq_expand(q4_nk: np.ndarray, factor: np.ndarray, block: int) -> np.ndarray:
    """int4 x per-block uint8 factor -> saturated int8 (HmxW4LpbqExpandToI8Op.cpp:26-47,94-97)."""
    f = np.repeat(factor.astype(np.int32), block, axis=1)
    return np.clip(q4_nk.astype(np.int32) * f, -128, 127).astype(np.int8)


def split_int16(q16: np.ndarray):
    """Two's-complement byte split q16 == hi*256 + lo, hi int8, lo uint8
    (scripts/verify_w16a16_two_w8a16.py:21-28)."""
    q = q16.astype(np.int64)
    return (q >> 8).astype(np.int8), (q & 0xFF).astype(np.uint8)


def sha256(arr: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(arr).reshape(-1).tobytes()).hexdigest()
