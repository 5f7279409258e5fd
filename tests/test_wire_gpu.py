"""Weight wire formats on the GPU: qhtp_weights_from_wire turns every reference carrier in
tests/golden/wire_formats.npz (bytes from the reference's own packers) into exactly the plain
carrier the oracle derives, and a MatMul fed through a wire-format weight is bit-exact against the
oracle end to end."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import mm_oracle as O
from oracle import wire_oracle as W
from tests.mm_helpers import KERNEL_FAMILY, to_dev

pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).parent / "golden" / "wire_formats.npz")
CASES = W.golden_cases()


def _decode(fmt, flags, wire: np.ndarray, k: int, n: int) -> np.ndarray:
    from qcom_htp_b200 import weights_from_wire
    out = weights_from_wire(fmt, to_dev(wire), k, n, xor80=bool(flags & W.XOR80), hilo=bool(flags & W.HILO),
                            biased=bool(flags & W.BIASED))
    return out.cpu().numpy()


@pytest.mark.parametrize("key", sorted(CASES))
def test_device_decode_matches_reference_packers(key):
    fmt, flags = CASES[key]
    logical = GOLDEN["w8_kn"] if fmt in W.W8_FORMATS else GOLDEN["w4_kn"]
    k, n = logical.shape
    got = _decode(fmt, flags, GOLDEN[key], k, n)
    np.testing.assert_array_equal(got.view(np.uint8), W.to_plain(fmt, logical).view(np.uint8))


@pytest.mark.parametrize("family,fmt,flags", [
    ("w4a8_per_channel", W.W4_TILE32X64_NPAIR32, W.XOR80),           # the W4A8 HMX op's carrier
    ("w4a16_lpbq", W.W4_KBLOCK32_NMAJOR_K4, W.XOR80 | W.HILO),       # a native W4A16 order
    ("w4a16_per_channel", W.W4_NPAIR_TILE32, W.XOR80 | W.BIASED),
    ("u8i8", W.W8_RAW_KN, W.XOR80),                                  # the u8i8 op's carrier
    ("w8a16", W.W8_KMAJOR_SPLIT128, 0),
])
def test_matmul_from_wire_weights_bit_exact(family, fmt, flags):
    from qcom_htp_b200 import QuantMatMul
    c = O.generate_case(family, "normal_random", 64, 512, 256)
    fam = c.family
    w_kn = c.weight_q.T.astype(np.int32)                     # logical [K, N]
    wire = W.encode(fmt, flags, w_kn)
    plain = torch.from_numpy(_decode(fmt, flags, wire, 512, 256)).cuda()
    kw = {}
    if fam.schema == "lpbq":
        kw = dict(schema="lpbq", lpbq_block_scale=to_dev(c.lpbq_factor), lpbq_block=fam.lpbq_block)
    op = QuantMatMul(KERNEL_FAMILY[fam.name], plain, to_dev(c.weight_scale.astype(np.float32)),
                     to_dev(c.bias_q.astype(np.int32)), act_scale=c.act_scale, out_scale=c.out_scale,
                     act_offset=c.act_offset, out_offset=c.out_offset, **kw)
    out = op(to_dev(c.act_q))
    op.check_device(64)
    np.testing.assert_array_equal(out.cpu().numpy(), O.exact_output(c))
