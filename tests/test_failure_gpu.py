"""Failure path of the kernels' bounded pipeline waits, exercised without faulting the GPU.

Every mbarrier wait in the kernels gives up after a cycle limit, records a code in the run's device
error word and returns; qhtp_matmul_check reads the word back as QHTP_STATUS_RUNTIME_ERROR.  Here a
self-test kernel waits (with that same wait routine, at a ~1 ms limit) on an mbarrier that no thread
ever arrives on -- a flag nothing sets.  The test checks that every warp gave up, that the status and
device code come back through qhtp_matmul_check, that the check clears the word, and that the context
still runs a GEMM bit-exactly afterwards.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import mm_oracle as O
from tests.mm_helpers import build_op, to_dev

pytestmark = pytest.mark.gpu

TIMEOUT_CODE = 4   # kErrTimeoutOther: the code a timed-out pipeline wait records


@pytest.mark.parametrize("family", ["u8i8", "w4a16_lpbq"])
def test_timed_out_wait_is_reported_and_context_survives(family):
    from qcom_htp_b200 import QhtpError
    from qcom_htp_b200 import _lib as L
    c = O.generate_case(family, "normal_random", 128, 256, 128)
    op = build_op(c)
    m = 128
    ws = op.workspace(m)
    plane_bytes = int(L.lib.qhtp_matmul_workspace_bytes(C.byref(op.plan), m)) - 256
    err_ptr = ws.data_ptr() + plane_bytes          # the run's error word inside the workspace
    gave_up = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    st = L.lib.qhtp_selftest_wait_timeout(err_ptr, gave_up.data_ptr(), 2_000_000, stream)
    assert st == L.OK
    torch.cuda.synchronize()
    assert int(gave_up.item()) == 4                 # all four warps stopped waiting and returned
    code = C.c_int(0)
    st = L.lib.qhtp_matmul_check(C.byref(op.plan), ws.data_ptr(), m, C.byref(code), stream)
    assert st == L.RUNTIME_ERROR and code.value == TIMEOUT_CODE
    # the check cleared the word, and the context is intact: a GEMM runs and is bit-exact
    out = op(to_dev(c.act_q))
    op.check_device(m)
    np.testing.assert_array_equal(out.cpu().numpy(), O.exact_output(c))
    # the Python wrapper raises on a recorded error
    L.lib.qhtp_selftest_wait_timeout(err_ptr, gave_up.data_ptr(), 2_000_000, stream)
    with pytest.raises(QhtpError, match="device code 4"):
        op.check_device(m)


def test_selftest_argument_checks():
    from qcom_htp_b200 import _lib as L
    w = torch.zeros(2, dtype=torch.int32, device="cuda")
    assert L.lib.qhtp_selftest_wait_timeout(None, w.data_ptr(), 1000, None) == L.INVALID_ARGUMENT
    assert L.lib.qhtp_selftest_wait_timeout(w.data_ptr(), None, 1000, None) == L.INVALID_ARGUMENT
    assert L.lib.qhtp_selftest_wait_timeout(w.data_ptr(), w.data_ptr() + 4, 0, None) == L.INVALID_ARGUMENT
    assert L.lib.qhtp_selftest_wait_timeout(w.data_ptr(), w.data_ptr() + 4, (1 << 32) + 1, None) == \
        L.INVALID_ARGUMENT


def test_check_after_normal_run_is_ok():
    from qcom_htp_b200 import _lib as L
    c = O.generate_case("w8a16", "normal_random", 64, 256, 96)
    op = build_op(c)
    op(to_dev(c.act_q))
    code = C.c_int(-1)
    st = L.lib.qhtp_matmul_check(C.byref(op.plan), op.workspace(64).data_ptr(), 64, C.byref(code),
                                 torch.cuda.current_stream().cuda_stream)
    assert st == L.OK and code.value == 0
