"""GPU parity of the per-group W4 schema (float32 scale per 64 weights of K, float32 bias) through the
C ABI.  The oracle is ``per_group_output``: the float64 sum of exact per-group contributions, which
reproduces the reference's own output_ref_q on its per-group golden cases.  The GPU runs the same
IEEE float64 operations in the same order, so the comparison is exact (every output code)."""
import numpy as np
import pytest

from oracle import mm_oracle as O
from tests.mm_helpers import build_op, run_case, to_dev

pytestmark = pytest.mark.gpu

FAMILIES = ["w4a8_per_group", "w4a16_per_group"]


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("case", O.CASES)
@pytest.mark.parametrize("shape", [(256, 256, 256), (32, 128, 32), (64, 192, 96)])
def test_reference_cases_bit_exact(family, case, shape):
    """The reference's seven cases at its three golden shapes (K=192: a half K block; N=96 and N=32:
    partial 64-channel tiles): every output code equals the oracle and the reference's output."""
    c = O.generate_case(family, case, *shape)
    got = run_case(c)
    np.testing.assert_array_equal(got, O.per_group_output(c))
    np.testing.assert_array_equal(got, c.ref_output_q)


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("m", [1, 17, 130, 300])
def test_ragged_m(family, m):
    c = O.generate_case(family, "normal_random", m, 320, 160)
    np.testing.assert_array_equal(run_case(c), O.per_group_output(c))


@pytest.mark.parametrize("family", FAMILIES)
def test_large_k_many_tiles(family):
    """K=4096 (64 groups, 32 pipeline stages per tile) and more tiles than SMs."""
    c = O.generate_case(family, "normal_random", 512, 4096, 2304, with_reference_output=False)
    np.testing.assert_array_equal(run_case(c), O.per_group_output(c))


def test_same_op_reused_and_stream_order():
    c = O.generate_case("w4a16_per_group", "scale_only", 200, 512, 192)
    op = build_op(c)
    want = O.per_group_output(c)
    for _ in range(3):
        np.testing.assert_array_equal(run_case(c, op=op), want)


def test_bad_group_scale_rejected():
    """A zero group scale fails the prepare with INVALID_ARGUMENT (host sees the device flag)."""
    from qcom_htp_b200 import QhtpError
    c = O.generate_case("w4a8_per_group", "normal_random", 32, 128, 32)
    c.weight_scale = c.weight_scale.copy()
    c.weight_scale[3, 1] = 0.0
    with pytest.raises(QhtpError):
        build_op(c)


def test_chain_per_group():
    """CHAIN mode (each output feeds the next activation, K == N) with per-group weights."""
    import dataclasses

    import torch
    c = O.generate_case("w4a16_per_group", "normal_random", 64, 256, 256)
    op = build_op(c)
    out = torch.empty((64, 256), dtype=torch.uint16, device="cuda")
    op.run_prepared(to_dev(c.act_q), out, chain=3)
    x = c.act_q
    for _ in range(3):
        x = O.per_group_output(dataclasses.replace(c, act_q=x))
    np.testing.assert_array_equal(out.cpu().numpy(), x)


def test_host_buffers_per_group():
    """qhtp_matmul_run_host (pinned host activation and output, row chunks) with per-group weights."""
    import torch
    c = O.generate_case("w4a8_per_group", "scale_only", 300, 256, 192)
    op = build_op(c)
    act_h = torch.from_numpy(np.ascontiguousarray(c.act_q)).pin_memory()
    out_h = op.run_host(act_h, chunk_rows=128)
    torch.cuda.synchronize()
    op.check_host()
    np.testing.assert_array_equal(out_h.numpy(), O.per_group_output(c))
