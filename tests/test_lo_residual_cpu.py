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


def test_dispatch_rule_mirror(monkeypatch):
    """QuantMatMul.lo_residual_launch restates the library's choice (qgemm.cu lo_residual_launch)
    with the header's flag values: a valid bound (1) that is forced (16), or that pays (8) on a
    launch of at least three waves of 128 x 128 tiles on the SMs the launch may use."""
    import re
    import types
    from pathlib import Path

    import torch
    from qcom_htp_b200 import _lib as L
    from qcom_htp_b200.matmul import QuantMatMul

    header = (Path(__file__).resolve().parents[1] / "include" / "qhtp.h").read_text()
    flag = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define QHTP_PLAN_FLAG_(\w+) (\d+)u", header)}
    assert flag == {"LO_RESIDUAL_BY_BOUND": 1, "INT4_STREAM": 2, "FORCE_INT4_STREAM": 4, "LO_RESIDUAL_PAYS": 8,
                    "FORCE_LO_RESIDUAL": 16}
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda dev: types.SimpleNamespace(multi_processor_count=148))
    op = object.__new__(QuantMatMul)
    op.device = torch.device("cuda", 0)
    op.plan = L.QhtpMatmulPlan()
    op.plan.n_tiles = 14                      # N = 1792: one 8-GPU shard of N = 14336
    rows3 = 32 * 128                          # 448 tiles >= 3 x 148
    for flags, small, three_waves, reserved in [(0, False, False, False), (1, False, False, False),
                                                (9, False, True, True), (17, True, True, True),
                                                (24, False, False, False), (11, False, True, True)]:
        op.plan.flags = flags
        assert op.lo_residual_launch(128) is small, flags
        assert op.lo_residual_launch(rows3) is three_waves, flags
        assert op.lo_residual_launch(rows3 - 128) is ((flags & 17) == 17), flags  # 434 tiles: only if forced
        assert op.lo_residual_launch(10 * 128, max_ctas=40) is reserved, flags   # 140 tiles on 40 SMs
