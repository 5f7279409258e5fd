"""Decode-shaped GEMM (M <= 128 activation rows): the channel-major kernel with a cluster K split.

Every output byte must equal the oracle's (bit-exact), for each family and dequant mode, at row
counts on both sides of the 16/32/64/128-column instruction shapes and of the row-tiled kernel's
threshold (M = 129), with K split over up to 8 CTAs of a cluster (reduced in rounds of 64 rows)
and ragged channel tiles.
"""
import numpy as np
import pytest

from oracle import mm_oracle as O
from tests.mm_helpers import build_op, make_w16a16_case, run_case

pytestmark = pytest.mark.gpu

FAMS = ["u8i8", "w4a8_per_channel", "w4a8_lpbq", "w8a16", "w4a16_per_channel", "w4a16_lpbq"]


@pytest.mark.parametrize("family", FAMS)
@pytest.mark.parametrize("m", [1, 2, 16, 33, 64, 65, 100, 128, 129])
def test_decode_rows_bit_exact(family, m):
    # K = 2048 -> 16 K blocks: split 4 ways over a cluster; N = 256 -> two channel tiles
    c = O.generate_case(family, "normal_random", m, 2048, 256)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c))


@pytest.mark.parametrize("family", ["w8a16", "w4a16_lpbq", "u8i8"])
def test_decode_eight_way_split_and_ragged_tile(family):
    # K = 4096 -> 32 K blocks over one 96-channel (partial) tile: the split reaches 8 CTAs
    c = O.generate_case(family, "normal_random", 16, 4096, 96)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c))


@pytest.mark.parametrize("case", O.CASES)
def test_decode_reference_value_cases(case):
    """The reference's seven value cases (boundary codes, impulses, bias-only, scale-only) at M=16."""
    c = O.generate_case("w4a16_lpbq", case, 16, 512, 256)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c))


@pytest.mark.parametrize("family", ["w8a16", "w4a16_lpbq", "u8i8"])
def test_decode_exact_dequant_mode(family):
    c = O.generate_case(family, "normal_random", 16, 1024, 256)
    np.testing.assert_array_equal(run_case(c, dequant="exact"), O.exact_output(c, dequant="exact"))


@pytest.mark.parametrize("m", [1, 16, 64, 128])
def test_decode_w16a16(m):
    c = make_w16a16_case(m, 1024, 160, seed=0x16 + m)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c, dequant="exact"))


def test_decode_baseline_width_n14336():
    """BASELINE decode row: W4A16 LPBQ, M = 1, K = 4096, N = 14336 (112 channel tiles, no split)."""
    c = O.make_baseline_case("w4a16_lpbq", 1, 4096, 14336, seed=0xDEC0)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c))


def test_decode_repeat_and_twin_calls_identical():
    """Two calls on the same op and inputs give identical bytes (no state carried between calls)."""
    c = O.generate_case("w4a16_lpbq", "normal_random", 16, 2048, 256)
    op = build_op(c)
    a = run_case(c, op=op)
    b = run_case(c, op=op)
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("m", [64, 65, 128])
def test_dispatch_boundary_wide_n(m):
    """At N = 14336 (112 channel tiles) rows 65..128 go to the row-tiled kernel and up to 64 to the
    channel-major one; both sides of the boundary must give the oracle's bytes."""
    c = O.make_baseline_case("w4a16_lpbq", m, 512, 14336, seed=0xD15 + m)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c))
