"""CHAIN=N through the prepared-run entry points (qhtp_<family>_run_prepared with chain > 1).

The reference's chain graphs apply one MatMul op `chain` times, each output code tensor feeding the
next op as its activation (gen_quant_chain.py:1346-1362; reference output :1542-1545; CHAIN=8 is the
default of its generator, :1612).  For K == N <= 256 the library runs the whole chain in one kernel
with the intermediate activations kept in shared memory (qchain.cu); every step must still equal the
oracle's step bit for bit, and the fused result must equal the same chain run as separate GEMMs.
"""
import numpy as np
import pytest
import torch

from oracle import mm_oracle as O
from tests.mm_helpers import build_op, make_w16a16_case, to_dev

pytestmark = pytest.mark.gpu

FAMILIES = ["u8i8", "w4a8_per_channel", "w4a8_lpbq", "w8a16", "w4a16_per_channel", "w4a16_lpbq"]


def oracle_chain(c: O.QuantCase, chain: int, dequant: str = "f32") -> np.ndarray:
    x = c.act_q
    for _ in range(chain):
        x = O.exact_output(c.with_act(x), dequant=dequant)
    return x


def run_chain(op, act: np.ndarray, n: int, chain: int) -> np.ndarray:
    out = torch.empty((act.shape[0], n), dtype=torch.uint16 if act.dtype == np.uint16 else torch.uint8,
                      device="cuda")
    op.run_prepared(to_dev(act), out, chain=chain)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def unfused_chain(op, act: np.ndarray, n: int, chain: int) -> np.ndarray:
    x = to_dev(act)
    for _ in range(chain):
        x = op(x)
    op.check_device(act.shape[0])
    return x.cpu().numpy()


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("case", ["normal_random", "positive_boundary", "scale_only"])
def test_chain8_256_bit_exact(family, case):
    """The reference's chain gate shape: CHAIN=8 at M=K=N=256."""
    c = O.generate_case(family, case, 256, 256, 256)
    op = build_op(c)
    got = run_chain(op, c.act_q, 256, 8)
    np.testing.assert_array_equal(got, oracle_chain(c, 8))
    np.testing.assert_array_equal(got, unfused_chain(op, c.act_q, 256, 8))


def test_chain8_w16a16_256():
    c = make_w16a16_case(256, 256, 256, seed=0xC8A1)
    op = build_op(c)
    got = run_chain(op, c.act_q, 256, 8)
    np.testing.assert_array_equal(got, oracle_chain(c, 8, dequant="exact"))


@pytest.mark.parametrize("family", ["u8i8", "w4a16_lpbq", "w8a16"])
@pytest.mark.parametrize("m", [1, 100, 300])
def test_chain_ragged_rows(family, m):
    """Row blocks are independent clusters; rows past M never reach the output."""
    c = O.generate_case(family, "normal_random", m, 256, 256)
    op = build_op(c)
    np.testing.assert_array_equal(run_chain(op, c.act_q, 256, 5), oracle_chain(c, 5))


@pytest.mark.parametrize("family", ["w4a8_per_channel", "w4a16_per_channel"])
@pytest.mark.parametrize("kn", [32, 96, 128, 192])
def test_chain_one_tile_and_partial_tile(family, kn):
    """Clusters of ceil(N / 64) CTAs, 64 channels each: N = 32 (one CTA, half full), 96 (two, the
    second half full), 128 (two), 192 (three)."""
    c = O.generate_case(family, "normal_random", 130, kn, kn)
    op = build_op(c)
    np.testing.assert_array_equal(run_chain(op, c.act_q, kn, 8), oracle_chain(c, 8))


def test_chain_exact_dequant_mode():
    c = O.generate_case("w8a16", "normal_random", 64, 256, 256)
    op = build_op(c, dequant="exact")
    np.testing.assert_array_equal(run_chain(op, c.act_q, 256, 3), oracle_chain(c, 3, dequant="exact"))


def test_chain_two_calls_and_chain_two():
    """Repeated calls are independent (no state carried in the kernel) and chain=2 uses one ping-pong."""
    c = O.generate_case("w4a16_lpbq", "normal_random", 256, 256, 256)
    op = build_op(c)
    a = run_chain(op, c.act_q, 256, 2)
    b = run_chain(op, c.act_q, 256, 2)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(a, oracle_chain(c, 2))


def test_chain_beyond_fused_shape_uses_gemm_loop():
    """K == N = 384 (three channel tiles) is outside the fused kernel: the host loop of GEMMs runs."""
    c = O.generate_case("w8a16", "normal_random", 64, 384, 384)
    op = build_op(c)
    np.testing.assert_array_equal(run_chain(op, c.act_q, 384, 3), oracle_chain(c, 3))
