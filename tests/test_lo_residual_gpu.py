"""The lo-plane residual bound (plan flag kPlanLoResidualByBound, u16 activations with float32 weight
dequant): the GEMM leaves the product of the activation's lo byte plane with the e' residual plane
out of its MMAs, bounds it per channel (record field lo_win), and adds it exactly only for the
elements whose value lies within that bound of a rounding boundary.  Every output code must still
equal the oracle's (and so the reference's) bit for bit."""
import numpy as np
import pytest
import torch

from oracle import mm_oracle as O
from tests.mm_helpers import build_op, run_case, to_dev

pytestmark = pytest.mark.gpu

FLAG = 1  # kPlanLoResidualByBound


def flagged_count(c: O.QuantCase) -> int:
    """Elements the bound sends to the exact fix-up: the value without the lo x e' term lies within
    lo_win + 2 units of 2^-30 of a rounding boundary (the fast path's window, modelled in float64
    with a margin, so the count is a lower bound of what the kernel sees)."""
    rec, ep, cc, _ = O.prepare_record(c, return_c=True)
    _, T, _ = O.exact_output(c, return_t=True)
    x_lo = (c.act_q.astype(np.int64) & 0xFF).astype(np.float64)
    le = (x_lo @ ep.astype(np.float64).T).astype(np.int64)
    z = (T - le).astype(np.float64) * cc[None, :] + c.out_zp
    dist = np.abs((z - np.floor(z)) - 0.5)
    return int((dist * 2.0 ** 30 < rec["lo_win"][None, :] * 0.9).sum())


@pytest.mark.parametrize("family", ["w8a16", "w4a16_per_channel", "w4a16_lpbq"])
def test_flag_set_for_reference_cases(family):
    c = O.generate_case(family, "normal_random", 256, 256, 256)
    op = build_op(c)
    assert int(op.plan.flags) & FLAG


def test_flag_off_for_u8_activations_and_exact_mode():
    assert not int(build_op(O.generate_case("w4a8_lpbq", "normal_random", 256, 256, 256)).plan.flags) & FLAG
    c = O.generate_case("w8a16", "normal_random", 256, 256, 256)
    assert not int(build_op(c, dequant="exact").plan.flags) & FLAG


@pytest.mark.parametrize("family,seed", [("w8a16", 11), ("w4a16_lpbq", 12), ("w4a16_per_channel", 13)])
def test_fixup_path_runs_and_is_exact(family, seed):
    """K = 4096 widens the bound; enough elements land in the window that the warp-cooperative
    exact fix-up runs many times in one call."""
    c = O.make_baseline_case(family, 512, 4096, 512, seed=seed)
    assert flagged_count(c) >= 5
    op = build_op(c)
    assert int(op.plan.flags) & FLAG
    np.testing.assert_array_equal(run_case(c, op=op), O.exact_output(c))


def test_fixup_rows_past_m_and_ragged_tile():
    """Rows past M in the last row tile take part in the warp's fix-up loop but never store."""
    c = O.make_baseline_case("w8a16", 300, 4096, 256, seed=21)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c))


def test_same_result_as_full_product_mode():
    """The exact-dequant mode is a different rounding model; instead compare the LO3 kernel against
    the oracle on a shape with more row and channel tiles than SMs (persistent tile loop)."""
    c = O.make_baseline_case("w4a16_lpbq", 1024, 1024, 4096, seed=31)
    op = build_op(c)
    act = to_dev(c.act_q)
    out = op(act)
    op.check_device(1024)
    np.testing.assert_array_equal(out.cpu().numpy(), O.exact_output(c))
