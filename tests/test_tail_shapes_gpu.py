"""The row-tiled GEMM at shapes whose 128 x 128 tiles leave the persistent CTAs' last wave partly
idle (tiles > SMs, tiles % SMs != 0): every CTA's tile loop, the ragged last wave and the host-buffer
chunking must all give the oracle's output codes."""
import numpy as np
import pytest
import torch

from oracle import mm_oracle as O
from tests.mm_helpers import build_op, make_w16a16_case, run_case, to_dev

pytestmark = pytest.mark.gpu


def sms() -> int:
    return torch.cuda.get_device_properties(0).multi_processor_count


def tiles(m: int, n: int) -> int:
    return ((m + 127) // 128) * ((n + 127) // 128)


@pytest.mark.parametrize("family", ["w4a16_lpbq", "w8a16", "u8i8", "w4a8_per_channel"])
def test_all_tail_shape(family):
    """160 tiles on 148 SMs: one whole wave and 12 tiles in the second (K = 1024)."""
    m, k, n = 1280, 1024, 2048
    assert tiles(m, n) > sms() and tiles(m, n) % sms() != 0
    c = O.make_baseline_case(family, m, k, n, seed=41)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c))


def test_whole_waves_plus_tail_w16a16_and_exact_mode():
    m, k, n = 2560, 1024, 1024          # 160 tiles
    c = make_w16a16_case(m, k, n, seed=42)
    np.testing.assert_array_equal(run_case(c), O.exact_output(c, dequant="exact"))
    c = O.make_baseline_case("w8a16", m, k, n, seed=43)
    np.testing.assert_array_equal(run_case(c, dequant="exact"), O.exact_output(c, dequant="exact"))


@pytest.mark.parametrize("family", ["w4a16_lpbq", "w4a8_per_channel"])
def test_eight_gpu_shard_shape(family):
    """One rank's slab of BASELINE configs[4] at 8 GPUs: M = K = 4096, N = 14336 / 8 = 1792
    (448 tiles: three whole waves and 4 tiles).  Sampled rows against the oracle, and two calls equal."""
    m, k, n = 4096, 4096, 1792
    c = O.make_baseline_case(family, m, k, n, seed=44)
    op = build_op(c)
    act = to_dev(c.act_q)
    out1 = op(act)
    out2 = op(act)
    op.check_device(m)
    assert torch.equal(out1, out2)
    rows = np.r_[0:48, 1000:1040, 2040:2100, 4050:4096]
    np.testing.assert_array_equal(out1.cpu().numpy()[rows], O.exact_output(c.with_act(c.act_q[rows])))


def test_host_buffer_chunks_with_tail():
    """qhtp_matmul_run_host in row chunks of 1280 rows (each chunk 100 tiles, the whole call 200)."""
    m, k, n = 2560, 1024, 1024
    c = O.make_baseline_case("w4a16_per_channel", m, k, n, seed=45)
    op = build_op(c)
    act_h = torch.from_numpy(c.act_q).pin_memory()
    out_h = torch.empty((m, n), dtype=torch.uint16).pin_memory()
    op.run_host(act_h, out_h, chunk_rows=1280)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out_h.numpy(), O.exact_output(c))
