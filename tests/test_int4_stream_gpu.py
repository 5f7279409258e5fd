"""Decode rows (M <= 2) of the int4 families through the 4-bit code stream (qdec4.cu).

The kernel reads the prepared code image (offset-binary nibbles, per-K-step LPBQ factors and
per-(channel, factor) e' tables) instead of the byte planes and must give the oracle's output byte
for byte: every activation width, dequant mode and schema, ragged channel tiles, one- and many-stage
K, tiles shared by several CTAs (partials summed by the combine kernel) and tiles one CTA covers.
QHTP_PLAN_FLAG_FORCE_INT4_STREAM (4) sends small shapes down the path; the production dispatch
takes it by itself only for long weight streams (the N = 14336 case below).
"""
import numpy as np
import pytest
import torch

from oracle import mm_oracle as O
from tests.mm_helpers import build_op, to_dev

pytestmark = pytest.mark.gpu

INT4_STREAM, FORCE = 2, 4
FAMS = ["w4a8_per_channel", "w4a8_lpbq", "w4a16_per_channel", "w4a16_lpbq"]


def run(op, act: np.ndarray) -> np.ndarray:
    out = op(to_dev(act))
    op.check_device(act.shape[0])
    torch.cuda.synchronize()
    return out.cpu().numpy()


def forced(c: O.QuantCase, dequant: str | None = None):
    op = build_op(c, dequant)
    assert op.plan.flags & INT4_STREAM, "the code image was not built"
    op.plan.flags |= FORCE
    return op


@pytest.mark.parametrize("family", FAMS)
@pytest.mark.parametrize("dequant", ["f32", "exact"])
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("kn", [(256, 256), (512, 352), (2048, 96)])
def test_forced_code_stream_bit_exact(family, dequant, m, kn):
    """K = 256 (one stage), 512, 2048 (8 stages); N = 352 and 96 leave a partial last tile."""
    k, n = kn
    c = O.generate_case(family, "normal_random", m, k, n)
    op = forced(c, None if dequant == "f32" else "exact")
    np.testing.assert_array_equal(run(op, c.act_q), O.exact_output(c, dequant=dequant))


@pytest.mark.parametrize("case", O.CASES)
@pytest.mark.parametrize("family", ["w4a16_lpbq", "w4a8_per_channel"])
def test_forced_reference_value_cases(family, case):
    """The reference's seven value cases (boundary codes, impulses, bias-only, scale-only)."""
    c = O.generate_case(family, case, 2, 512, 256)
    np.testing.assert_array_equal(run(forced(c), c.act_q), O.exact_output(c))


@pytest.mark.parametrize("block", [32, 128])
def test_forced_lpbq_block_sizes(block):
    """LPBQ blocks of 32 (a factor per K step) and 128 (one per four steps)."""
    c = O.make_baseline_case("w4a16_lpbq", 2, 1024, 256, seed=0xB10C + block, lpbq_block=block)
    np.testing.assert_array_equal(run(forced(c), c.act_q), O.exact_output(c))


def test_forced_matches_byte_plane_path():
    """The same op and input through both decode kernels: identical bytes."""
    c = O.generate_case("w4a16_lpbq", "normal_random", 2, 1024, 384)
    op = build_op(c)
    planes = run(op, c.act_q)
    op.plan.flags |= FORCE
    codes = run(op, c.act_q)
    np.testing.assert_array_equal(codes, planes)
    np.testing.assert_array_equal(codes, O.exact_output(c))


@pytest.mark.parametrize("m", [1, 2])
def test_dispatch_long_stream_n14336(m):
    """BASELINE decode width (W4A16 LPBQ, K = 4096, N = 14336: 12 stages per SM): the production
    dispatch takes the code stream without the override; tiles are shared between CTAs."""
    c = O.make_baseline_case("w4a16_lpbq", m, 4096, 14336, seed=0xC0DE + m)
    op = build_op(c)
    assert op.plan.flags & INT4_STREAM and not op.plan.flags & FORCE
    np.testing.assert_array_equal(run(op, c.act_q), O.exact_output(c))


def test_factor_outside_range_keeps_byte_planes():
    """An LPBQ factor of 17 (u * f no longer fits a byte): prepare leaves the code stream off and the
    byte-plane kernel runs, still exact (the expanded weight saturates at 127 as in the reference)."""
    c = O.generate_case("w4a16_lpbq", "normal_random", 1, 512, 256)
    c.lpbq_factor[3, 1] = 17
    c.lpbq_expanded[:] = O.lpbq_expand(c.weight_q, c.lpbq_factor, c.family.lpbq_block)
    op = build_op(c)
    assert not op.plan.flags & INT4_STREAM
    op.plan.flags |= FORCE  # no effect without the code image
    np.testing.assert_array_equal(run(op, c.act_q), O.exact_output(c))


def test_repeat_calls_identical_and_no_state():
    """Two calls in a row (the partial slots and combine kernel carry nothing between calls)."""
    c = O.generate_case("w4a8_lpbq", "normal_random", 2, 2048, 512)
    op = forced(c)
    a = run(op, c.act_q)
    b = run(op, c.act_q)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(a, O.exact_output(c))
