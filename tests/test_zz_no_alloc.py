"""qhtp_matmul_run_noalloc: the MatMul entry point for callers that cannot allocate device memory.

Such callers (a runtime plugin whose host runtime owns every device buffer, a latency-critical thread)
cannot hand the op a workspace, so this entry point keeps its scratch in a fixed area inside the
library.  These tests call it through the C ABI and require the same output bytes as
qhtp_matmul_run, on two calls in a row (the scratch area keeps the previous call's contents, so the
second call checks that nothing stale leaks into the result).  The file is named so that pytest
collects it last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import mm_oracle as O
from tests.mm_helpers import build_op, to_dev

pytestmark = pytest.mark.gpu


def _noalloc(op, act: torch.Tensor) -> torch.Tensor:
    from qcom_htp_b200 import _lib as L
    out = torch.empty((act.shape[0], op.n), dtype=torch.uint16 if op.out_bits == 16 else torch.uint8,
                      device=act.device)
    st = L.lib.qhtp_matmul_run_noalloc(C.byref(op.plan), act.data_ptr(), act.shape[0], out.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream)
    L.check("qhtp_matmul_run_noalloc", st)
    return out


@pytest.mark.parametrize("family", ["w4a16_lpbq", "u8i8"])
def test_noalloc_matches_workspace_entry_point_twice(family):
    c = O.generate_case(family, "normal_random", 256, 256, 256)
    c2 = O.generate_case(family, "scale_only", 256, 256, 256)
    op = build_op(c)
    for act_np in (c.act_q, c2.act_q):               # two calls in a row, different activations
        act = to_dev(act_np)
        want = op(act)                                # existing entry point, caller workspace
        got = _noalloc(op, act)
        torch.cuda.synchronize()
        assert torch.equal(got, want)                 # our tolerance for integer outputs: exact
    np.testing.assert_array_equal(got.cpu().numpy(), O.exact_output(
        O.QuantCase(c.family, c2.act_q, c.weight_q, c.weight_scale, c.bias_q, c.act_scale, c.out_scale,
                    c.lpbq_factor, c.lpbq_expanded)))


def test_noalloc_rejects_oversized_workspace():
    from qcom_htp_b200 import _lib as L
    c = O.generate_case("w8a16", "normal_random", 32, 4096, 32)
    op = build_op(c)
    m = 4096                                          # 2*4096*4096 + 256 bytes > 8 MiB
    act = torch.zeros((m, 4096), dtype=torch.uint16, device="cuda")
    out = torch.empty((m, 32), dtype=torch.uint16, device="cuda")
    st = L.lib.qhtp_matmul_run_noalloc(C.byref(op.plan), act.data_ptr(), m, out.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream)
    assert st == L.INVALID_ARGUMENT
    assert b"8 MiB" in L.lib.qhtp_last_error_string()
