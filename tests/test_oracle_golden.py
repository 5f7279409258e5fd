"""Pin the CPU oracle to the reference's own golden vectors (no GPU).

The fixtures in tests/golden were produced by importing the reference's scripts
(tests/golden/make_golden.py); these tests show that the restated generator reproduces the
reference's inputs bit for bit and that the exact requant model reproduces the reference's
``output_ref_q`` on every case of every promoted family.
"""
import json
from pathlib import Path
from fractions import Fraction

import numpy as np
import pytest

from oracle import gdn_oracle as G
from oracle import mm_oracle as O


def _entries(golden_dir):
    return json.loads((golden_dir / "mm_reference_cases.json").read_text())["entries"]


def test_golden_covers_all_families_and_cases(golden_dir):
    ents = _entries(golden_dir)
    got = {(e["family"], e["case"], tuple(e["shape_mkn"])) for e in ents}
    for fam in O.REFERENCE_GENERATED:
        for case in O.CASES:
            assert (fam, case, (256, 256, 256)) in got


@pytest.mark.parametrize("shape", [(256, 256, 256), (32, 128, 32), (64, 192, 96)])
def test_generator_and_exact_model_match_reference(golden_dir, shape):
    checked = 0
    for e in _entries(golden_dir):
        if tuple(e["shape_mkn"]) != shape:
            continue
        fam = O.FAMILIES[e["family"]]
        assert O.seed_for(fam.name, e["case"]) == e["seed"]
        c = O.generate_case(fam, e["case"], *shape)
        h = e["sha256"]
        assert O.sha256(c.act_q) == h["activation_q"], e["family"] + e["case"]
        assert O.sha256(c.weight_q) == h["weight_q_nk"]
        assert O.sha256(c.weight_scale) == h["weight_scale"]
        assert O.sha256(c.bias_q) == h["bias_q_int32"]
        assert c.act_scale == e["act_scale"] and c.out_scale == e["out_scale"]
        if "lpbq_block_scale" in h:
            assert O.sha256(c.lpbq_factor) == h["lpbq_block_scale"]
            assert O.sha256(c.lpbq_expanded) == h["lpbq_expanded_q_nk"]
        # the restated float64 formula reproduces the reference's output
        assert O.sha256(c.ref_output_q) == h["output_ref_q"]
        # the model the GPU computes reproduces it too: the exact integer/requant model, or for the
        # per-group schema the float64 sum of exact group contributions
        got = O.per_group_output(c) if fam.schema == "per_group" else O.exact_output(c)
        assert O.sha256(got) == h["output_ref_q"], (e["family"], e["case"])
        checked += 1
    assert checked >= 56


def test_small_case_arrays(golden_dir):
    z = np.load(golden_dir / "mm_small_cases.npz")
    for fam in ("u8i8", "w4a8_lpbq", "w8a16", "w4a16_per_channel", "w4a16_lpbq"):
        for case in O.CASES:
            key = f"{fam}/{case}"
            c = O.generate_case(fam, case, 32, 128, 32)
            np.testing.assert_array_equal(c.act_q, z[key + "/activation_q"])
            np.testing.assert_array_equal(c.weight_q, z[key + "/weight_q_nk"])
            np.testing.assert_array_equal(O.exact_output(c), z[key + "/output_ref_q"])


def test_residual_plane_reproduces_f32_dequant():
    rng = np.random.default_rng(5)
    scales = (rng.uniform(1e-6, 1.0, 64) * 10.0 ** rng.integers(-8, 3, 64)).astype(np.float32)
    q = rng.integers(-128, 128, (64, 300)).astype(np.int16)
    m, e = O.split_f32(scales)
    ep = O.residual_plane(q, m)
    assert np.abs(ep).max() <= 64
    deq = q.astype(np.float32) * scales[:, None]                    # numpy float32 product
    rebuilt = np.ldexp((q.astype(np.int64) * m[:, None] + ep).astype(np.float64), e[:, None])
    np.testing.assert_array_equal(deq.astype(np.float64), rebuilt)
    # round_to_24_bits agrees with int -> float32 conversion (round half to even)
    p = rng.integers(-(1 << 31) + 1, 1 << 31, 100000)
    np.testing.assert_array_equal(O.round_to_24_bits(p), p.astype(np.float32).astype(np.int64))


def test_prepare_record_sidecar_fields():
    c = O.generate_case("w4a16_lpbq", "normal_random", 64, 256, 64)
    rec, ep = O.prepare_record(c)
    m, e = O.split_f32(c.weight_scale)
    zp = c.family.act_zp
    w = c.mma_weight.astype(np.int64)
    np.testing.assert_array_equal(rec["beff"], m * (c.bias_q - zp * w.sum(1)) - zp * ep.astype(np.int64).sum(1))
    np.testing.assert_array_equal(rec["m_q"], m)
    assert rec.dtype.itemsize == 32


def test_exact_round_tie_breaking():
    # construct an exact tie: T * sA * 2^e / sO == 2.5
    c = O.generate_case("u8i8", "normal_random", 32, 128, 32)
    assert O._exact_round(5, 1, 0, 1.0, 2.0, 0) == 2          # 2.5 -> 2 (even)
    assert O._exact_round(7, 1, 0, 1.0, 2.0, 0) == 4          # 3.5 -> 4
    assert O._exact_round(-5, 1, 0, 1.0, 2.0, 10) == 8        # 7.5 -> 8
    assert c is not None


def test_w16a16_identity_golden(golden_dir):
    ents = json.loads((golden_dir / "w16a16_identity.json").read_text())["entries"]
    for e in ents:
        m, k, n = e["shape_mkn"]
        rng = np.random.default_rng(e["seed"])
        act = rng.integers(0, 65536, size=(m, k), dtype=np.uint16).astype(np.int64)
        q16 = rng.integers(-32768, 32768, size=(k, n)).astype(np.int64)
        assert O.sha256(act.astype(np.uint16)) == e["sha256"]["act_u16"]
        assert O.sha256(q16.astype(np.int16)) == e["sha256"]["q16_kn"]
        hi, lo = O.split_int16(q16)
        assert O.sha256(hi) == e["sha256"]["hi_kn"] and O.sha256(lo) == e["sha256"]["lo_kn"]
        xc = act - 32768
        acc_hi, acc_lo = xc @ hi.astype(np.int64), xc @ lo.astype(np.int64)
        assert O.sha256(acc_hi) == e["sha256"]["acc_hi"]
        assert O.sha256(acc_lo) == e["sha256"]["acc_lo"]
        np.testing.assert_array_equal(acc_hi * 256 + acc_lo, xc @ q16)
        assert O.sha256(xc @ q16) == e["sha256"]["acc"]


def test_int4_packing_roundtrip():
    rng = np.random.default_rng(1)
    q = rng.integers(-8, 8, (96, 128)).astype(np.int8)
    p = O.pack_int4_kpair(q)
    assert p.shape == (64, 96)
    np.testing.assert_array_equal(O.unpack_int4_kpair(p, 96, 128), q)
    # byte (k>>1)*N + n, even k low nibble
    assert (p[3, 5] & 0xF) == (q[5, 6] & 0xF) and (p[3, 5] >> 4) == (q[5, 7] & 0xF)


def test_lpbq_expand_saturates():
    q4 = np.array([[-8, 7, -1, 3] * 16], np.int8)
    f = np.array([[16]], np.uint8)
    out = O.lpbq_expand(q4, f, 64)
    assert out.min() == -128 and out.max() == 112


def test_gdn_kat_pins_fp64_inverse(golden_dir):
    z = np.load(golden_dir / "gdn_sbr_kat.npz")
    T = G.inverse_fp64(z["A"])
    assert G.oc(T, z["Tref"]) < 1e-7


def test_gdn_block_model_within_gate(golden_dir):
    z = np.load(golden_dir / "gdn_sbr_kat.npz")
    A = z["A"].astype(np.float64)
    sA = np.abs(A).max() / 32767.0
    Aq = np.clip(np.rint(A / sA), -32767, 32767).astype(np.int16)
    T = G.block_model(Aq, sA, 2.0 / 32767.0)
    assert G.oc(T, z["Tref"]) <= G.OC_GATE


def test_gdn_c_restatement_matches_numpy_model():
    import ctypes
    from pathlib import Path
    lib_path = Path(G.__file__).parent / "libgdn_block_ref.so"
    if not lib_path.exists():
        pytest.skip("oracle/libgdn_block_ref.so not built (make -C oracle)")
    lib = ctypes.CDLL(str(lib_path))
    A = G.make_chunk_A(6, C=64, seed=3)
    sA = float(np.abs(A).max() / 32767.0)
    Aq = np.clip(np.rint(A / sA), -32767, 32767).astype(np.int16)
    sT = 2.0 / 32767.0
    T = np.zeros(A.shape, np.float64)
    sAv = np.full(A.shape[0], sA, np.float32)
    rc = lib.gdn_block_ref_solve(Aq.ctypes.data_as(ctypes.c_void_p), sAv.ctypes.data_as(ctypes.c_void_p),
                                 ctypes.c_float(sT), A.shape[0], 64, T.ctypes.data_as(ctypes.c_void_p), 2)
    assert rc == 0
    Tm = G.block_model(Aq, float(np.float32(sA)), float(np.float32(sT)))
    assert np.abs(T - Tm).max() < 1e-6
    assert G.oc(T, G.inverse_fp64(Aq * np.float64(np.float32(sA)))) < 1e-3


def test_gdn_synthetic_A_structure():
    A = G.make_chunk_A(3, C=64, seed=9)
    assert A.shape == (3, 64, 64)
    assert np.all(np.triu(A) == 0)
    # bf16-representable
    assert np.all((A.view(np.uint32) & 0xFFFF) == 0)
    # |beta| < 1, |k_i . k_j| <= 1 for unit keys, decay <= 1
    assert np.abs(A).max() <= 1.0


@pytest.mark.parametrize("family", ["u8i8", "w4a8_lpbq", "w4a16_per_channel", "w4a16_lpbq", "w8a16"])
def test_quantize_weight_fast_matches_loop(family):
    fam = O.FAMILIES[family]
    if fam.schema == "lpbq":
        fam = fam.with_block(64)
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((48, 512)) * 0.02).astype(np.float32)
    w[3] = 0.0                       # all-zero channel -> 1e-12 floor
    a, b = O.quantize_weight(fam, w), O.quantize_weight_fast(fam, w)
    for key in a:
        np.testing.assert_array_equal(a[key], b[key], err_msg=key)


def test_gdn_A_from_kbg_matches_reference_chunk_kernel():
    """chunk_A_from_kbg + inverse_fp64 reproduce the T the reference's own gdn_chunk forms
    (scripts/gdn_ref_kernel.py, fp64; fixture by tests/golden/make_gdn_kbg_golden.py)."""
    z = np.load(Path(__file__).parent / "golden" / "gdn_kbg_kat.npz")
    A = G.chunk_A_from_kbg(z["k"], z["beta"], z["g_tok"])
    T = G.inverse_fp64(A)
    assert np.abs(T - z["T"]).max() < 1e-12


def test_gdn_c_port_matches_reference_solver_binary(tmp_path):
    """The timed CPU baseline (oracle/gdn_block_ref.c) against the reference's own scalar solver
    (example/gdn_native/solve_op/gdn_solve_ref.c:17-84, compiled unmodified into oracle/_ref by
    oracle/Makefile) on shared inputs: the same file formats the reference's main() reads
    (dims.i32, A_codes.i16, sA.f32, sT.f32 -> T_out.f64).  Equal bit for bit."""
    import ctypes
    import subprocess
    odir = Path(G.__file__).parent
    ref_bin = odir / "_ref" / "gdn_solve_ref"
    lib_path = odir / "libgdn_block_ref.so"
    if not ref_bin.exists() or not lib_path.exists():
        pytest.skip("oracle/_ref/gdn_solve_ref or oracle/libgdn_block_ref.so not built (make -C oracle [ref])")
    for C, seed in ((64, 5), (256, 6)):
        A = G.make_chunk_A(3, C=C, seed=seed)
        H = A.shape[0]
        sA = (np.abs(A).reshape(H, -1).max(axis=1) / 32767.0).astype(np.float32)   # one scale per head
        Aq = np.clip(np.rint(A / sA[:, None, None]), -32767, 32767).astype(np.int16)
        sT = np.float32(2.0 / 32767.0)
        np.array([H, C], np.int32).tofile(tmp_path / "dims.i32")
        Aq.tofile(tmp_path / "A_codes.i16")
        sA.tofile(tmp_path / "sA.f32")
        np.array([sT], np.float32).tofile(tmp_path / "sT.f32")
        subprocess.run([str(ref_bin)], cwd=tmp_path, check=True, capture_output=True)
        want = np.fromfile(tmp_path / "T_out.f64", np.float64).reshape(H, C, C)
        lib = ctypes.CDLL(str(lib_path))
        got = np.zeros((H, C, C), np.float64)
        rc = lib.gdn_block_ref_solve(Aq.ctypes.data_as(ctypes.c_void_p), sA.ctypes.data_as(ctypes.c_void_p),
                                     ctypes.c_float(sT), H, C, got.ctypes.data_as(ctypes.c_void_p), 2)
        assert rc == 0
        np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("shift", [0.0, 1.5, -2.0, 3.0])
def test_free_offset_u8i8_exact_model_matches_float64_path(shift):
    """BASELINE configs[0] (u8i8, QNN free-offset asymmetric activation/output encodings, per-tensor
    int8 weights): the exact integer model equals the reference oracle's float64 quantized path on
    every element, at activation zero points far from the families' fixed 128."""
    c = O.make_free_offset_u8i8_case(256, 256, 256, seed=11, x_shift=shift)
    assert 0 <= c.act_zp <= 255 and 0 <= c.out_zp <= 255
    assert len(set(c.weight_scale.tolist())) == 1                   # one per-tensor scale
    np.testing.assert_array_equal(O.exact_output(c), c.ref_output_q)
    if shift != 0.0:
        assert c.act_zp != 128


def test_qnn_asymmetric_encoding_rules():
    s, zp = O.qnn_asymmetric_encoding(-1.0, 3.0)
    assert s == 4.0 / 255 and zp == 64                  # -round(-1 / (4/255)) = round(63.75) = 64
    s, zp = O.qnn_asymmetric_encoding(0.5, 2.0)         # range widened to hold 0: zero point 0
    assert s == 2.0 / 255 and zp == 0
    s, zp = O.qnn_asymmetric_encoding(-2.0, -0.5)
    assert zp == 255
