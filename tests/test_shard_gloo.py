"""Multi-GPU host logic on CPU: world_size-2 gloo process groups (no GPU).

The sharded paths run the single-GPU op on each rank's slab with no data-path exchange, so the
checks are: the slabs tile the whole problem, each rank's slab computes exactly the corresponding
part of the full result (the oracle applied to the sliced carriers), and the all-gather reassembles
the full output in order.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import gdn_oracle as G
from oracle import mm_oracle as O
from qcom_htp_b200 import shard as S

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, *args):
    port = _free_port()
    mp.start_processes(_entry, args=(fn, port, args), nprocs=WORLD, start_method="spawn", join=True)


def _entry(rank, fn, port, args):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    try:
        fn(rank, *args)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n,world", [(14336, 8), (4096, 2), (96, 2), (32, 4), (1024, 3)])
def test_shard_range_tiles_channels(n, world):
    ranges = [S.shard_range(n, world, r, S.CHANNEL_ALIGN) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    widths = [b - a for a, b in ranges]
    assert all(w % S.CHANNEL_ALIGN == 0 for w in widths)
    assert max(widths) - min(widths) <= S.CHANNEL_ALIGN


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        S.shard_range(64, 2, 2, 32)
    with pytest.raises(ValueError):
        S.shard_range(40, 2, 0, 32)


def _case_tensors(c):
    fam = c.family
    if fam.weight_bits == 4:
        w = torch.from_numpy(O.pack_int4_kpair(c.weight_q))
    elif fam.weight_bits == 16:
        w = torch.from_numpy(c.weight_q.astype(np.int16))
    else:
        w = torch.from_numpy(c.weight_q.astype(np.int8))
    lp = torch.from_numpy(c.lpbq_factor) if fam.schema == "lpbq" else None
    return w, torch.from_numpy(c.weight_scale.astype(np.float32)), torch.from_numpy(c.bias_q.astype(np.int32)), lp


def _sliced_case(c, shard):
    """The oracle's view of one rank's slab (column slice of every per-channel carrier)."""
    sl = slice(shard.n0, shard.n1)
    return O.QuantCase(c.family, c.act_q, c.weight_q[sl], c.weight_scale[sl], c.bias_q[sl], c.act_scale,
                       c.out_scale, None if c.lpbq_factor is None else c.lpbq_factor[sl],
                       None if c.lpbq_expanded is None else c.lpbq_expanded[sl])


def _matmul_rank(rank, family):
    import torch.distributed as dist
    c = O.generate_case(family, "normal_random", 24, 256, 160)
    w, sc, b, lp = _case_tensors(c)
    sh = S.shard_matmul_weights(w, sc, b, weight_bits=c.family.weight_bits, world=WORLD, rank=rank,
                                lpbq_block_scale=lp)
    # the carriers handed to this rank are exactly the slab of the full ones
    if c.family.weight_bits == 4:
        unpacked = O.unpack_int4_kpair(sh.weight.numpy(), sh.n1 - sh.n0, c.weight_q.shape[1])
        np.testing.assert_array_equal(unpacked, c.weight_q[sh.n0:sh.n1])
    part = _sliced_case(c, sh)
    np.testing.assert_array_equal(sh.weight_scale.numpy(), c.weight_scale[sh.n0:sh.n1].astype(np.float32))
    local = O.exact_output(part)                      # what this rank's op must produce (bit-exact)
    full = O.exact_output(c)
    np.testing.assert_array_equal(local, full[:, sh.n0:sh.n1])
    got = S.gather_channels(torch.from_numpy(local.copy()), WORLD)
    np.testing.assert_array_equal(got.numpy(), full)
    dist.barrier()


@pytest.mark.parametrize("family", ["w4a16_lpbq", "w8a16", "u8i8", "w4a8_per_channel"])
def test_matmul_n_shard_gloo(family):
    _run(_matmul_rank, family)


def _gdn_rank(rank, n_units, C):
    A = G.make_chunk_A(n_units, C=C, seed=0x5EA + C)
    a, b = S.shard_chunks(n_units, WORLD, rank)
    T_local = torch.from_numpy(G.inverse_fp64(A[a:b]).astype(np.float32))
    T = S.gather_chunks(T_local, n_units, WORLD)
    np.testing.assert_array_equal(T.numpy(), G.inverse_fp64(A).astype(np.float32))


@pytest.mark.parametrize("n_units", [5, 8])
def test_gdn_chunk_shard_gloo(n_units):
    _run(_gdn_rank, n_units, 32)


def _failing_rank(rank, marker):
    if rank == 1:
        raise RuntimeError("rank 1 fails before the collective")
    # rank 0 must not hang: the gather ends with an error once rank 1 is gone
    try:
        S.gather_channels(torch.zeros((2, 32), dtype=torch.uint16), WORLD)
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        with open(marker, "w") as f:
            f.write(type(e).__name__)


def test_failed_rank_is_reported(tmp_path):
    """A rank that dies between steps (host-side failure) surfaces as an error on the survivor,
    not a hang, and the launcher reports the failed rank."""
    marker = tmp_path / "rank0_saw_error"
    with pytest.raises(Exception, match="rank 1 fails"):
        _run(_failing_rank, str(marker))
    assert marker.exists()
