"""qhtp_matmul_run_host: activation and output in pinned host memory, row chunks whose copies
overlap the other chunks' GEMMs.  Every output byte must equal the oracle's, whatever the chunking
(ragged last chunk, chunks on both sides of the decode kernel's 128-row threshold, one chunk)."""
import numpy as np
import pytest
import torch

from oracle import mm_oracle as O
from tests.mm_helpers import build_op

pytestmark = pytest.mark.gpu


def _run_host(case, chunk_rows):
    op = build_op(case)
    act_h = torch.from_numpy(np.ascontiguousarray(case.act_q)).pin_memory()
    out_h = op.run_host(act_h, chunk_rows=chunk_rows)
    torch.cuda.synchronize()
    op.check_host()
    return op, out_h.numpy()


@pytest.mark.parametrize("family,m,chunk_rows", [
    ("w4a16_lpbq", 1000, 0),      # library chunking: 128-row chunks, ragged last one
    ("w4a16_lpbq", 700, 300),     # chunks above the decode threshold and a 100-row tail
    ("u8i8", 300, 64),            # u8 activations, decode-kernel chunks
    ("w8a16", 1, 0),              # one chunk of one row
])
def test_host_run_bit_exact(family, m, chunk_rows):
    c = O.generate_case(family, "normal_random", m, 512, 256)
    op, out = _run_host(c, chunk_rows)
    np.testing.assert_array_equal(out, O.exact_output(c))
    assert op.host_chunk_rows == (chunk_rows or min(m, ((m + 7) // 8 + 127) // 128 * 128))


def test_host_run_twice_and_after_device_run_identical():
    """The library's copy streams and events are reused: back-to-back calls, and a device-buffer call
    in between, give the same bytes."""
    c = O.generate_case("w4a16_lpbq", "normal_random", 640, 512, 256)
    op = build_op(c)
    act_h = torch.from_numpy(np.ascontiguousarray(c.act_q)).pin_memory()
    a = op.run_host(act_h)
    torch.cuda.synchronize()
    a = a.clone()
    dev = op(act_h.cuda())
    b = op.run_host(act_h)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(a.numpy(), b.numpy())
    np.testing.assert_array_equal(a.numpy(), dev.cpu().numpy())
