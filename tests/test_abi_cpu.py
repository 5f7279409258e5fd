"""C-ABI checks that need no GPU: the library loads, exports every declared symbol, validates
arguments on the host, and its exact requant decision agrees with rational arithmetic."""
import ctypes as C
import re
from fractions import Fraction
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def L():
    from qcom_htp_b200 import _lib
    return _lib


def test_exports_every_header_symbol(L):
    header = (ROOT / "include" / "qhtp.h").read_text()
    declared = set(re.findall(r"\b(qhtp_[a-z0-9_]+)\s*\(", header))
    assert len(declared) >= 19
    assert declared == set(L.SIGNATURES)
    for name in declared:
        assert hasattr(L.lib, name), name
        assert name in L.SIGNATURES, f"{name} has no ctypes signature"


def test_status_strings(L):
    assert [L.status_string(s) for s in range(4)] == ["ok", "invalid_argument", "unsupported", "runtime_error"]
    assert L.status_string(99) == "unknown"
    assert b"sm_100a" in L.lib.qhtp_version()


def _weights(L, **kw):
    d = dict(family=L.FAMILY["w4a16"], schema=L.SCHEMA["lpbq"], dequant=0, k=4096, n=14336, lpbq_block=64,
             weight=1, weight_scale=1, bias_q=1, lpbq_block_scale=1, act_scale=1e-4, act_offset=-32768,
             out_scale=1e-3, out_offset=-32768)
    d.update(kw)
    return L.QhtpMatmulWeights(**d)


def test_plan_valid_shapes(L):
    p = L.QhtpMatmulPlan()
    assert L.lib.qhtp_matmul_plan(C.byref(_weights(L)), C.byref(p)) == L.OK
    assert p.a_planes == 2 and p.ch_per_tile == 128 and p.n_tiles == 112 and p.k_pad == 4096
    assert p.act_zp == 32768 and p.out_zp == 32768 and p.out_qmax == 65535
    # prepared bytes: planes (256 rows x K per tile) + records + sums + status area
    assert p.prepared_bytes >= 112 * 256 * 4096 + 112 * 128 * 32
    assert L.lib.qhtp_matmul_prepared_bytes(C.byref(p)) == p.prepared_bytes
    assert L.lib.qhtp_matmul_workspace_bytes(C.byref(p), 4096) >= 2 * 4096 * 4096
    # act_scale = act_mant * 2^act_exp2 exactly
    assert Fraction(p.act_mant) * Fraction(2) ** p.act_exp2 == Fraction(1e-4)


def test_plan_int4_code_image_and_decode_workspace(L):
    """int4 families also carry the 4-bit code image (0.5 B per weight, one factor byte per 32
    weights, 16 e' tables of 16 B per channel); runs of M <= 2 rows reserve the partial-sum slots of
    the code-stream kernel (160 CTAs x 2 segments x M x 128 channels x 8 B) before the error word."""
    p = L.QhtpMatmulPlan()
    assert L.lib.qhtp_matmul_plan(C.byref(_weights(L)), C.byref(p)) == L.OK
    image = 112 * 128 * 4096 // 2 + 112 * (4096 // 32) * 128 + 112 * 16 * 128 * 16
    assert p.prepared_bytes >= 112 * 256 * 4096 + 112 * 128 * 32 + image
    ws = [L.lib.qhtp_matmul_workspace_bytes(C.byref(p), m) for m in (1, 2, 3)]
    assert ws[0] >= 2 * 4096 + 160 * 2 * 1 * 128 * 8 + 256
    assert ws[1] >= 4 * 4096 + 160 * 2 * 2 * 128 * 8 + 256
    assert ws[2] == -(-6 * 4096 // 256) * 256 + 256  # M = 3: byte planes and the error word only
    # an 8-bit family has no code image
    q = L.QhtpMatmulPlan()
    assert L.lib.qhtp_matmul_plan(C.byref(_weights(L, family=L.FAMILY["w8a16"], schema=L.SCHEMA["per_channel"],
                                                   lpbq_block=0, lpbq_block_scale=None)), C.byref(q)) == L.OK
    assert L.lib.qhtp_matmul_workspace_bytes(C.byref(q), 1) == 2 * 4096 + 256


@pytest.mark.parametrize("kw,status", [
    (dict(k=4000), 2), (dict(n=100), 2), (dict(k=0), 1), (dict(family=9), 1), (dict(schema=5), 1),
    (dict(lpbq_block=48), 2), (dict(lpbq_block=4096), 2), (dict(act_scale=0.0), 1), (dict(out_scale=-1.0), 1),
    (dict(act_offset=5), 1), (dict(k=65536), 2),
    (dict(family=2, schema=1), 2),              # LPBQ only for int4 weights
    (dict(family=4, schema=0, dequant=0), 2),   # W16A16 has no float32-dequant reference
])
def test_plan_rejects(L, kw, status):
    p = L.QhtpMatmulPlan()
    assert L.lib.qhtp_matmul_plan(C.byref(_weights(L, **kw)), C.byref(p)) == status


def test_plan_per_group(L):
    """Per-group W4 schema (generate_qnn_matmul_python_cases.py:392-423): 128-channel tiles, 256 weight
    rows ([q | e']) per tile, K a multiple of 64 above 64, float32-dequant only, W4 families only."""
    p = L.QhtpMatmulPlan()
    w = _weights(L, schema=L.SCHEMA["per_group"], lpbq_block=0, bias_q=None, bias_float=1, lpbq_block_scale=None,
                 k=4096 + 64, n=14336 + 32)
    assert L.lib.qhtp_matmul_plan(C.byref(w), C.byref(p)) == L.OK
    assert p.mode == 3 and p.ch_per_tile == 128 and p.n_tiles == 113 and p.k_pad == 4224
    # planes (256 rows x k_pad per tile) + group constants (2560 bytes per tile and group) + bias
    assert p.prepared_bytes >= 113 * 256 * 4224 + 113 * 66 * 2560 + 113 * 128 * 8
    for kw, status in [(dict(k=64), 2), (dict(k=96), 2), (dict(family=L.FAMILY["w8a16"]), 2),
                       (dict(family=L.FAMILY["u8i8"]), 2), (dict(dequant=1), 2)]:
        ww = _weights(L, schema=L.SCHEMA["per_group"], lpbq_block=0, bias_float=1, **kw)
        assert L.lib.qhtp_matmul_plan(C.byref(ww), C.byref(L.QhtpMatmulPlan())) == status, kw


def test_prepare_per_group_needs_float_bias(L):
    """The per-group schema takes its bias as float32 (bias_float); a NULL one fails on the host."""
    p = L.QhtpMatmulPlan()
    w = _weights(L, schema=L.SCHEMA["per_group"], lpbq_block=0, bias_q=1, bias_float=None, lpbq_block_scale=None)
    assert L.lib.qhtp_matmul_plan(C.byref(w), C.byref(p)) == L.OK
    fake = C.c_void_p(1 << 20)
    assert L.lib.qhtp_matmul_prepare(C.byref(p), C.byref(w), fake, p.prepared_bytes, None) == L.INVALID_ARGUMENT


def test_null_and_unplanned_calls_are_errors(L):
    p = L.QhtpMatmulPlan()
    assert L.lib.qhtp_matmul_plan(None, C.byref(p)) == L.INVALID_ARGUMENT
    assert L.lib.qhtp_matmul_run(C.byref(p), None, 1, None, None, 0, None) == L.INVALID_ARGUMENT
    assert L.lib.qhtp_matmul_prepare(C.byref(p), None, None, 0, None) == L.INVALID_ARGUMENT
    assert L.lib.qhtp_matmul_run_host(C.byref(p), None, 1, None, None, None, None, 0, 0, None, None) \
        == L.INVALID_ARGUMENT
    assert L.lib.qhtp_u8i8_run_prepared(None) == L.INVALID_ARGUMENT
    assert L.lib.qhtp_gdn_inverse_bf16(None, None, 1, 256, None) == L.INVALID_ARGUMENT
    assert L.lib.qhtp_gdn_inverse_bf16(1024, 1024, 1, 96, None) == L.UNSUPPORTED
    assert L.lib.qhtp_gdn_solve_u16(1024, 1, 256, 32768, C.c_float(0.0), 32768, C.c_float(1.0), 1024, None) \
        == L.INVALID_ARGUMENT


def _split(x: float):
    fr, e = np.frexp(np.float64(x))
    return int(np.ldexp(fr, 53)), int(e) - 53


def test_requant_host_matches_rational_arithmetic(L):
    """The exact tie path (128-bit integer compare) agrees with Fractions, including at exact ties."""
    from qcom_htp_b200.matmul import requant_code_host
    rng = np.random.default_rng(11)
    n_tie = 0
    for i in range(4000):
        s_a = float(rng.uniform(1e-5, 1e-3))
        s_o = float(rng.uniform(1e-3, 1e-1))
        ma, ea = _split(s_a)
        mo, eo = _split(s_o)
        e_s = int(rng.integers(-40, -20))
        mul = int(rng.integers(1, 1 << 24)) if i % 2 else 1
        zp = int(rng.choice([0, 128, 32768]))
        qmax = 255 if zp <= 128 else 65535
        exact_mult = Fraction(mul) * Fraction(s_a) * Fraction(2) ** e_s / Fraction(s_o)
        if i % 4 == 0:
            # place T right at a tie: T = round((r + 0.5 - zp) / mult)
            r = int(rng.integers(0, qmax))
            T = round((Fraction(r) + Fraction(1, 2) - zp) / exact_mult)
        else:
            T = int(rng.integers(-(1 << 40), 1 << 40))
        if abs(T) >= (1 << 62) or abs(T) * mul >= (1 << 75):
            continue   # outside the kernel's documented accumulator range
        c = float(Fraction(s_a) * Fraction(2) ** e_s / Fraction(s_o)) * mul
        cm, ce = _split(c)
        want = min(max(round(T * exact_mult + zp), 0), qmax)
        got = requant_code_host(T, cm, -ce, mul, e_s + ea, ma, mo, eo, zp, qmax)
        frac = T * exact_mult + zp
        if abs(frac - (frac.numerator // frac.denominator) - Fraction(1, 2)) < Fraction(1, 10 ** 9):
            n_tie += 1
        assert got == want, (i, T, mul, e_s, s_a, s_o, zp)
    assert n_tie > 100


def test_exact_tie_half_even(L):
    from qcom_htp_b200.matmul import requant_code_host
    # act_scale = 1 (mant 2^52, exp -52), e_s = -1, out_scale = 1: value = T / 2; c = 0.5 = 2^52 * 2^-53
    # T=5 gives exactly 2.5 -> 2 ; T=7 -> 3.5 -> 4
    c = (1 << 52, 53)
    assert requant_code_host(5, *c, 1, -53, 1 << 52, 1 << 52, -52, 0, 255) == 2
    assert requant_code_host(7, *c, 1, -53, 1 << 52, 1 << 52, -52, 0, 255) == 4
    assert requant_code_host(-1000, *c, 1, -53, 1 << 52, 1 << 52, -52, 0, 255) == 0
    assert requant_code_host(10 ** 6, *c, 1, -53, 1 << 52, 1 << 52, -52, 0, 255) == 255
    assert requant_code_host(-7, *c, 1, -53, 1 << 52, 1 << 52, -52, 128, 255) == 124   # 128 - 3.5 -> 124
    assert requant_code_host(5, 1 << 52, 33, 1, -53, 1 << 52, 1 << 52, -52, 0, 255) == -1   # bad shift


def test_host_run_rejects_small_workspace_before_any_device_work(L):
    """qhtp_matmul_run_host validates sizes on the host: a workspace below
    qhtp_matmul_workspace_bytes(plan, chunk rows) is INVALID_ARGUMENT with a message, before any
    device pointer is touched (the pointers below are never dereferenced)."""
    p = L.QhtpMatmulPlan()
    assert L.lib.qhtp_matmul_plan(C.byref(_weights(L)), C.byref(p)) == L.OK
    p.prepared = 4096                                  # stands in for a prepared buffer
    fake = C.c_void_p(1 << 20)                         # 256-byte aligned, never dereferenced
    used = C.c_uint32(0)
    need = L.lib.qhtp_matmul_workspace_bytes(C.byref(p), 512)
    st = L.lib.qhtp_matmul_run_host(C.byref(p), fake, 4096, fake, fake, fake, fake, need - 1, 512, C.byref(used),
                                    None)
    assert st == L.INVALID_ARGUMENT
    assert b"workspace" in L.lib.qhtp_last_error_string()
    assert L.lib.qhtp_matmul_run_host(C.byref(p), None, 4096, fake, fake, fake, fake, need, 512, None,
                                      None) == L.INVALID_ARGUMENT
