"""GPU parity of the quantized MatMul family through the C ABI (bit-exact against the oracle)."""
import numpy as np
import pytest
import torch

from oracle import mm_oracle as O
from tests.mm_helpers import build_op, make_w16a16_case, run_case, to_dev

pytestmark = pytest.mark.gpu

PROMOTED = ["u8i8", "w4a8_per_channel", "w4a8_lpbq", "w8a16", "w4a16_per_channel", "w4a16_lpbq"]


@pytest.mark.parametrize("family", PROMOTED)
@pytest.mark.parametrize("case", O.CASES)
def test_reference_cases_256_bit_exact(family, case):
    """The reference's 7 promoted cases at 256^3: every output byte equals the oracle (which equals
    the reference's own output_ref_q, pinned by the golden tests)."""
    c = O.generate_case(family, case, 256, 256, 256)
    got = run_case(c)
    want = O.exact_output(c)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(got, c.ref_output_q)


@pytest.mark.parametrize("family", PROMOTED)
def test_prepared_records_match_oracle_sidecar(family):
    """Sidecar parity: the device-prepared per-channel records equal the oracle's byte for byte."""
    c = O.generate_case(family, "normal_random", 64, 256, 96)
    op = build_op(c)
    rec = op.records()
    want, _ = O.prepare_record(c)
    got = rec[: c.weight_q.shape[0]].view(np.uint8).reshape(-1)
    assert got.tobytes() == want.view(np.uint8).reshape(-1).tobytes()


@pytest.mark.parametrize("family", ["u8i8", "w4a16_lpbq", "w8a16"])
@pytest.mark.parametrize("m", [1, 17, 130, 300])
def test_ragged_m(family, m):
    c = O.generate_case(family, "normal_random", m, 256, 96)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c))


@pytest.mark.parametrize("shape", [(32, 32, 32), (96, 160, 224), (128, 4096, 64)])
def test_odd_shapes_w4a16(shape):
    m, k, n = shape
    fam = O.FAMILIES["w4a16_per_channel"]
    if k <= 64:
        fam = O.FAMILIES["w8a16"]
    c = O.generate_case(fam, "normal_random", m, k, n)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c))


@pytest.mark.parametrize("m", [1, 16, 128])
def test_baseline_lpbq_decode_prefill_shapes(m):
    """BASELINE config: W4A16 LPBQ (block 64), K=4096, N=4096, activations N(0,1)."""
    c = O.make_baseline_case("w4a16_lpbq", m, 4096, 4096, seed=0x6D6D + m)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c))


def test_exact_dequant_mode_matches_oracle():
    for fam in ("u8i8", "w4a16_lpbq"):
        c = O.generate_case(fam, "normal_random", 130, 256, 256)
        np.testing.assert_array_equal(run_case(c, dequant="exact"), O.exact_output(c, dequant="exact"))


@pytest.mark.parametrize("shape", [(64, 64, 64), (256, 256, 256), (128, 256, 96)])
def test_w16a16_two_byte_passes(shape):
    """W16A16 = two byte-weight passes (verify_w16a16_two_w8a16.py shapes), exact integer requant."""
    c = make_w16a16_case(*shape)
    got = run_case(c)
    np.testing.assert_array_equal(got, O.exact_output(c, dequant="exact"))


def test_w16a16_extreme_weights():
    """Full int16 range including -32768 (hi byte -128, lo byte 0) and +32767."""
    m, k, n = 64, 256, 64
    c = make_w16a16_case(m, k, n, seed=4)
    rng = np.random.default_rng(4)
    c.weight_q = rng.choice(np.array([-32768, 32767, -1, 0, 1, -256, 255], np.int16), size=(n, k))
    np.testing.assert_array_equal(run_case(c), O.exact_output(c, dequant="exact"))


def test_lpbq_expand_op():
    from qcom_htp_b200 import lpbq_expand_i8
    rng = np.random.default_rng(2)
    n, k, blk = 96, 256, 64
    q4 = rng.integers(-8, 8, (n, k)).astype(np.int8)
    f = rng.integers(1, 17, (n, k // blk)).astype(np.uint8)
    got = lpbq_expand_i8(to_dev(O.pack_int4_kpair(q4)), to_dev(f), k, n, blk).cpu().numpy()
    np.testing.assert_array_equal(got, O.lpbq_expand(q4, f, blk))


def test_prepared_run_chain():
    """chain > 1: each output feeds the next activation (K == N, equal widths)."""
    c = O.generate_case("w8a16", "normal_random", 64, 256, 256)
    op = build_op(c)
    act = to_dev(c.act_q)
    out = torch.empty((64, 256), dtype=torch.uint16, device="cuda")
    op.run_prepared(act, out, chain=3)
    x = c.act_q
    for _ in range(3):
        c2 = O.QuantCase(c.family, x, c.weight_q, c.weight_scale, c.bias_q, c.act_scale, c.out_scale)
        x = O.exact_output(c2)
    np.testing.assert_array_equal(out.cpu().numpy(), x)


def test_run_prepared_family_mismatch_is_error():
    from qcom_htp_b200 import QhtpError
    c = O.generate_case("u8i8", "normal_random", 32, 128, 32)
    op = build_op(c)
    op.family = "w8a16"   # wrong entry point for this plan
    with pytest.raises(QhtpError):
        op.run_prepared(to_dev(c.act_q), torch.empty((32, 32), dtype=torch.uint8, device="cuda"))


def test_bad_scale_rejected_at_prepare():
    from qcom_htp_b200 import QhtpError
    c = O.generate_case("u8i8", "normal_random", 32, 128, 32)
    c.weight_scale = c.weight_scale.copy()
    c.weight_scale[3] = 0.0
    with pytest.raises(QhtpError):
        build_op(c)


def test_large_shape_properties_w4a16_lpbq():
    """Full BASELINE size (M=4096, K=4096, N=14336): compare a sampled slab against the oracle and
    check determinism across two runs."""
    m, k, n = 4096, 4096, 14336
    c = O.make_baseline_case("w4a16_lpbq", m, k, n, seed=7)
    op = build_op(c)
    act = to_dev(c.act_q)
    out1 = op(act)
    out2 = op(act)
    op.check_device(m)
    assert torch.equal(out1, out2)
    rows = np.r_[0:64, 2000:2064, 4032:4096]
    sub = O.QuantCase(c.family, c.act_q[rows], c.weight_q, c.weight_scale, c.bias_q, c.act_scale, c.out_scale,
                      c.lpbq_factor, c.lpbq_expanded)
    np.testing.assert_array_equal(out1.cpu().numpy()[rows], O.exact_output(sub))


@pytest.mark.parametrize("max_ctas", [1, 16, 147])
def test_run_on_fewer_sms_same_bytes(max_ctas):
    """qhtp_matmul_run_ctas: the row-tiled GEMM on a limited number of SMs gives the same bytes."""
    c = O.make_baseline_case("w4a16_lpbq", 512, 1024, 2048, seed=91)
    op = build_op(c)
    act = to_dev(c.act_q)
    full = op(act)
    part = op(act, max_ctas=max_ctas)
    op.check_device(512)
    assert torch.equal(full, part)
    np.testing.assert_array_equal(part.cpu().numpy(), O.exact_output(c))
