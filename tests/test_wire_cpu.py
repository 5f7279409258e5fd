"""Weight wire formats (the reference's QNN initializer layouts), no GPU: the oracle's decoder and
encoder reproduce the bytes the reference's own packers wrote (tests/golden/wire_formats.npz, made
by tests/golden/make_wire_golden.py from gen_quant_chain.py), and the C ABI's sizing and argument
checks."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from oracle import wire_oracle as W

GOLDEN = np.load(Path(__file__).parent / "golden" / "wire_formats.npz")
CASES = W.golden_cases()


def test_every_golden_carrier_is_covered():
    assert set(GOLDEN.files) - set(CASES) == {"w4_kn", "w8_kn", "lpbq__scale", "lpbq__per_block_nb"}


@pytest.mark.parametrize("key", sorted(CASES))
def test_oracle_decodes_and_encodes_reference_bytes(key):
    fmt, flags = CASES[key]
    logical = GOLDEN["w8_kn"] if fmt in W.W8_FORMATS else GOLDEN["w4_kn"]
    K, N = logical.shape
    wire = GOLDEN[key]
    assert wire.size == W.wire_bytes(fmt, K, N)
    np.testing.assert_array_equal(W.decode(fmt, flags, wire, K, N), logical)
    np.testing.assert_array_equal(W.encode(fmt, flags, logical), wire)


def test_lpbq_prechain_inputs_are_the_plain_carriers():
    """HmxW4LpbqExpandToI8's inputs: K-pair bytes [K/2, N] and factors [N, K/B] flattened."""
    w4 = GOLDEN["w4_kn"]
    np.testing.assert_array_equal(GOLDEN["lpbq__weight"], W.to_plain(W.W4_KPAIR, w4).reshape(-1))
    np.testing.assert_array_equal(GOLDEN["lpbq__scale"], GOLDEN["lpbq__per_block_nb"].reshape(-1))


def test_abi_sizes_and_argument_checks():
    from qcom_htp_b200 import _lib as L
    for name, f in L.WIRE_FORMAT.items():
        assert L.lib.qhtp_wire_bytes(f, 64, 256) == W.wire_bytes(f, 64, 256), name
    assert L.lib.qhtp_wire_bytes(0, 64, 256) == 0
    fake = C.c_void_p(256)  # never dereferenced: every call below fails validation first
    call = L.lib.qhtp_weights_from_wire
    assert call(99, 0, fake, 1 << 20, 64, 256, fake, 1 << 20, None) == L.INVALID_ARGUMENT
    assert call(W.W4_KPAIR, 8, fake, 1 << 20, 64, 256, fake, 1 << 20, None) == L.INVALID_ARGUMENT   # unknown flag
    assert call(W.W4_KPAIR, 0, None, 1 << 20, 64, 256, fake, 1 << 20, None) == L.INVALID_ARGUMENT
    assert call(W.W4_KPAIR, 0, fake, 100, 64, 256, fake, 1 << 20, None) == L.INVALID_ARGUMENT      # short wire
    assert call(W.W4_TILE32X64_NPAIR32, 0, fake, 1 << 20, 64, 96, fake, 1 << 20, None) == L.UNSUPPORTED
    assert call(W.W8_KMAJOR_SPLIT128, 0, fake, 1 << 20, 64, 64, fake, 1 << 20, None) == L.UNSUPPORTED
    assert call(W.W4_KPAIR, 0, fake, 1 << 20, 63, 256, fake, 1 << 20, None) == L.UNSUPPORTED
