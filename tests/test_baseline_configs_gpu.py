"""BASELINE.json configurations the reference-style 256^3 cases do not reach, bit-exact on the GPU.

* u8i8 with QNN's free asymmetric encodings -- activation zero point -round(min/scale)
  (not the families' fixed 128), per-tensor symmetric int8 weights, output scale and zero point from
  Y's float min/max.  The C ABI's generic act_offset / out_offset path, at several zero points and on
  both GEMM kernels (row-tiled and decode-shaped).
* W16A16 (two byte-weight passes) at the decode/prefill shapes M in {1, 16, 128},
  K = 4096, N in {4096, 14336}.
* the W4A8 per-channel GEMM at the full 4096 x 4096 x 14336 shape (sampled rows against
  the oracle, every row against a second run for determinism).
"""
import numpy as np
import pytest
import torch

from oracle import mm_oracle as O
from tests.mm_helpers import build_op, make_w16a16_case, run_case, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shift", [0.0, 1.5, -2.0, 3.0])
def test_u8i8_free_offset_encodings_256(shift):
    c = O.make_free_offset_u8i8_case(256, 256, 256, seed=11, x_shift=shift)
    got = run_case(c)
    np.testing.assert_array_equal(got, O.exact_output(c))
    np.testing.assert_array_equal(got, c.ref_output_q)       # the float64 path of the reference oracle


@pytest.mark.parametrize("m", [1, 16, 100, 300])
def test_u8i8_free_offset_ragged_rows_and_decode_kernel(m):
    c = O.make_free_offset_u8i8_case(m, 1024, 384, seed=0xC0 + m, x_shift=-1.0)
    got = run_case(c)
    np.testing.assert_array_equal(got, c.ref_output_q)


@pytest.mark.parametrize("n", [4096, 14336])
@pytest.mark.parametrize("m", [1, 16, 128])
def test_w16a16_baseline_shapes(m, n):
    c = make_w16a16_case(m, 4096, n, seed=0x1616 + m + n)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c, dequant="exact"))


def test_w4a8_per_channel_full_shape():
    m, k, n = 4096, 4096, 14336
    c = O.make_baseline_case("w4a8_per_channel", m, k, n, seed=0x48)
    op = build_op(c)
    act = to_dev(c.act_q)
    out1 = op(act)
    out2 = op(act)
    op.check_device(m)
    assert torch.equal(out1, out2)
    rows = np.r_[0:64, 2048:2112, 4032:4096]
    np.testing.assert_array_equal(out1.cpu().numpy()[rows], O.exact_output(c.with_act(c.act_q[rows])))
