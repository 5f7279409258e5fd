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


def _status(op, act_ptr, m, out_ptr, plan=True):
    from qcom_htp_b200 import _lib as L
    return L.lib.qhtp_matmul_run_noalloc(C.byref(op.plan) if plan else None, act_ptr, m, out_ptr,
                                         torch.cuda.current_stream().cuda_stream)


def test_noalloc_host_argument_checks():
    """The host-side checks that stand in for the caller workspace's: null plan, zero rows,
    16-byte-misaligned activation or output, and the 2^24-row limit of qhtp_matmul_run (for u8
    activations the scratch size alone would not bound M).  All rejected before any launch."""
    from qcom_htp_b200 import _lib as L
    c = O.generate_case("u8i8", "normal_random", 64, 128, 64)
    op = build_op(c)
    act = torch.zeros((65, 128), dtype=torch.uint8, device="cuda")
    out = torch.zeros((65, 64), dtype=torch.uint8, device="cuda")
    a, o = act.data_ptr(), out.data_ptr()
    assert _status(op, a, 64, o, plan=False) == L.INVALID_ARGUMENT
    assert _status(op, a, 0, o) == L.INVALID_ARGUMENT
    assert _status(op, a + 8, 64, o) == L.INVALID_ARGUMENT
    assert _status(op, a, 64, o + 8) == L.INVALID_ARGUMENT
    assert _status(op, a, (1 << 24) + 1, o) == L.UNSUPPORTED       # rejected on the host: no big buffers
    torch.cuda.synchronize()
    code = C.c_int(-1)
    assert L.lib.qhtp_matmul_noalloc_check(C.byref(op.plan), 0, C.byref(code), None) == L.INVALID_ARGUMENT


def test_noalloc_u8_rows_beyond_u16_limit_and_error_word():
    """u8 activations need no byte planes, so M may exceed what a u16 activation could use (here
    M = 8192, K = 1024: a u16 activation would need 16 MiB of planes).  Output equals
    qhtp_matmul_run's byte for byte on two calls in a row, and the error word the no-alloc calls keep
    in the library's scratch reads back as clear."""
    from qcom_htp_b200 import _lib as L
    m, k, n = 8192, 1024, 256
    c = O.make_baseline_case("u8i8", m, k, n, seed=0x8A)
    op = build_op(c)
    act = to_dev(c.act_q)
    for _ in range(2):
        want = op(act)
        got = _noalloc(op, act)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    code = C.c_int(-1)
    st = L.lib.qhtp_matmul_noalloc_check(C.byref(op.plan), m, C.byref(code),
                                         torch.cuda.current_stream().cuda_stream)
    assert st == L.OK and code.value == 0
    rows = np.r_[0:32, 8160:8192]
    sub = O.QuantCase(c.family, c.act_q[rows], c.weight_q, c.weight_scale, c.bias_q, c.act_scale, c.out_scale)
    np.testing.assert_array_equal(got.cpu().numpy()[rows], O.exact_output(sub))
