"""CPU checks of the lo-plane residual bound that the u16-activation GEMM relies on (record field
lo_win): for every element, the omitted term sum_k x_lo * e' moves the value by at most lo_win units
of 2^-30 of the output scale; and the shapes the GPU test uses do put elements inside the window."""
import numpy as np
import pytest

from oracle import mm_oracle as O
from tests.test_lo_residual_gpu import flagged_count


@pytest.mark.parametrize("family", ["w8a16", "w4a16_per_channel", "w4a16_lpbq"])
@pytest.mark.parametrize("case", O.CASES)
def test_window_bounds_the_lo_residual_term(family, case):
    c = O.generate_case(family, case, 64, 256, 96)
    rec, ep, cc, _ = O.prepare_record(c, return_c=True)
    x_lo = (c.act_q.astype(np.int64) & 0xFF)
    le = np.abs(x_lo @ ep.astype(np.int64).T)
    assert np.all(le.astype(np.float64) * cc[None, :] * 2.0 ** 30 <= rec["lo_win"][None, :])
    assert np.all(rec["lo_win"] >= 1)


def test_window_zero_for_u8_activations_and_exact_mode():
    rec, _ = O.prepare_record(O.generate_case("w4a8_lpbq", "normal_random", 32, 256, 64))
    assert np.all(rec["lo_win"] == 0)
    rec, _ = O.prepare_record(O.generate_case("w8a16", "normal_random", 32, 256, 64), dequant="exact")
    assert np.all(rec["lo_win"] == 0)


@pytest.mark.parametrize("family,seed", [("w8a16", 11), ("w4a16_lpbq", 12), ("w4a16_per_channel", 13)])
def test_gpu_fixup_cases_reach_the_window(family, seed):
    c = O.make_baseline_case(family, 512, 4096, 512, seed=seed)
    assert flagged_count(c) >= 5
