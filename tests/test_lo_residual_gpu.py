"""The lo-plane residual bound (plan flag kPlanLoResidualByBound, u16 activations with float32 weight
dequant): the GEMM leaves the product of the activation's lo byte plane with the e' residual plane
out of its MMAs, bounds it per channel (record field lo_win), and adds it exactly only for the
elements whose value lies within that bound of a rounding boundary.  Every output code must still
equal the oracle's (and so the reference's) bit for bit.

The library uses the bound on launches of at least three waves of tiles when prepare found the
expected fix-ups few (flag 8); the fix-up tests below run small shapes, so they force it (flag 16)."""
import numpy as np
import pytest
import torch

from oracle import mm_oracle as O
from tests.mm_helpers import build_op, run_case, to_dev

pytestmark = pytest.mark.gpu

FLAG = 1    # kPlanLoResidualByBound: the bound is valid
PAYS = 8    # kPlanLoResidualPays: prepare expects few fix-ups
FORCE = 16  # kPlanForceLoResidual: every row-tiled launch uses the bound


def forced(op):
    op.plan.flags |= FORCE
    return op


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
    op = forced(build_op(c))
    assert int(op.plan.flags) & FLAG and op.lo_residual_launch(512)
    np.testing.assert_array_equal(run_case(c, op=op), O.exact_output(c))


def test_fixup_rows_past_m_and_ragged_tile():
    """Rows past M in the last row tile take part in the warp's fix-up loop but never store."""
    c = O.make_baseline_case("w8a16", 300, 4096, 256, seed=21)
    np.testing.assert_array_equal(run_case(c, op=forced(build_op(c))), O.exact_output(c))


def test_same_result_as_full_product_mode():
    """The exact-dequant mode is a different rounding model; instead compare the LO3 kernel against
    the oracle on a shape with more row and channel tiles than SMs (persistent tile loop)."""
    c = O.make_baseline_case("w4a16_lpbq", 1024, 1024, 4096, seed=31)
    op = forced(build_op(c))
    act = to_dev(c.act_q)
    out = op(act)
    op.check_device(1024)
    np.testing.assert_array_equal(out.cpu().numpy(), O.exact_output(c))


@pytest.mark.parametrize("family,pays", [("w4a16_lpbq", True), ("w4a16_per_channel", True), ("w8a16", False)])
def test_prepare_decides_by_expected_fixups(family, pays):
    """At K = 4096 the int4 families expect ~3 fix-ups per 128 x 128 tile and W8A16 ~8.5 (its int8
    weights carry wider residuals): prepare marks the bound worth using for the former only.  The
    bound stays valid for all three."""
    c = O.make_baseline_case(family, 64, 4096, 1024, seed=41)
    op = build_op(c)
    assert int(op.plan.flags) & FLAG
    assert bool(int(op.plan.flags) & PAYS) == pays


def test_dispatch_by_waves_same_bytes():
    """Three waves of tiles or more take the bound, fewer keep the full product; forcing it on a
    one-wave launch gives the same bytes as the full product there."""
    m, k, n = 256, 4096, 2048
    c = O.make_baseline_case("w4a16_lpbq", m, k, n, seed=42)
    op = build_op(c)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert int(op.plan.flags) & PAYS
    assert not op.lo_residual_launch(m)                      # 32 tiles
    assert op.lo_residual_launch(3 * sms * 128 // (n // 128))  # three waves of rows
    assert op.lo_residual_launch(m, max_ctas=32 * 128 // (3 * 128))  # ... or of reserved SMs
    act = to_dev(c.act_q)
    full = op(act).cpu().numpy()
    op.check_device(m)
    forced(op)
    assert op.lo_residual_launch(m)
    bound = op(act).cpu().numpy()
    op.check_device(m)
    np.testing.assert_array_equal(full, bound)
    np.testing.assert_array_equal(bound[:32], O.exact_output(c.with_act(c.act_q[:32])))
