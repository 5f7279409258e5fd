"""Multi-GPU sharding of the two hot paths: one process per GPU, no exchange on the data path.

BASELINE's sharded sweep splits the quantized GEMM over output channels (N) and the GDN inverse over
batch x heads.  Output channels are independent in the MatMul family (every channel has its own
weight column, scale, LPBQ factors, bias and requant record), and GDN chunks are independent
matrices, so each rank runs the unchanged single-GPU op on its slab; the only collective is the
optional all-gather of the outputs (``torch.distributed``, NCCL on GPUs, gloo on CPU).

The reference has no distributed backend; this module is the host logic a multi-GPU caller of the
C ABI needs: which slab a rank owns, how to cut each weight carrier for it, and how to reassemble.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

CHANNEL_ALIGN = 32   # the kernels take N in multiples of 32 (reference: M/K/N multiples of 32)


def shard_range(total: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """[start, stop) of rank's share of `total` items split as evenly as possible in units of
    `align` (total must be a multiple of align).  Ranks beyond the number of units get empty ranges."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if total % align:
        raise ValueError(f"{total} items are not a multiple of {align}")
    units = total // align
    base, extra = divmod(units, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start * align, stop * align


@dataclass
class MatmulShard:
    """One rank's slab of a quantized-MatMul weight set, in the carrier formats of QuantMatMul."""
    n0: int
    n1: int
    weight: torch.Tensor            # int8 [N_r, K] | int4 K-pair [K/2, N_r] | int16 [N_r, K]
    weight_scale: torch.Tensor      # f32 [N_r]
    bias_q: torch.Tensor            # int32 [N_r]
    lpbq_block_scale: torch.Tensor | None  # u8 [N_r, K/block]


def shard_matmul_weights(weight: torch.Tensor, weight_scale: torch.Tensor, bias_q: torch.Tensor, *,
                         weight_bits: int, world: int, rank: int,
                         lpbq_block_scale: torch.Tensor | None = None) -> MatmulShard:
    """Cut rank's channel slab out of the full weight set.  The int4 carrier is K-pair packed
    ``[K/2, N]`` (byte (k>>1)*N + n, HmxW4LpbqExpandToI8Op.cpp:94-97), so its slab is a column slice;
    the int8 / int16 carriers are ``[N, K]`` and slice by rows."""
    n = weight_scale.shape[0]
    n0, n1 = shard_range(n, world, rank, CHANNEL_ALIGN)
    if weight_bits == 4:
        if weight.shape[1] != n:
            raise ValueError("int4 weight must be K-pair packed [K/2, N]")
        w = weight[:, n0:n1].contiguous()
    else:
        if weight.shape[0] != n:
            raise ValueError("int8/int16 weight must be [N, K]")
        w = weight[n0:n1].contiguous()
    lp = lpbq_block_scale[n0:n1].contiguous() if lpbq_block_scale is not None else None
    return MatmulShard(n0, n1, w, weight_scale[n0:n1].contiguous(), bias_q[n0:n1].contiguous(), lp)


def gather_channels(out_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather the [M, N_r] output slabs of every rank into [M, N] (rank order = channel order).
    Slabs may differ in width by CHANNEL_ALIGN; they are padded to the widest for the collective."""
    import torch.distributed as dist
    m, nr = out_local.shape
    widths = [torch.zeros(1, dtype=torch.int64, device=out_local.device) for _ in range(world)]
    dist.all_gather(widths, torch.tensor([nr], dtype=torch.int64, device=out_local.device), group=group)
    widths = [int(w.item()) for w in widths]
    wmax = max(widths)
    # transpose to [N_r, M] so each rank's slab is contiguous in the gathered buffer; moved as bytes
    # (NCCL has no 16-bit integer type, and a gather does no arithmetic)
    send = torch.zeros((wmax, m), dtype=out_local.dtype, device=out_local.device)
    send[:nr] = out_local.t()
    recv = torch.empty((world * wmax, m), dtype=out_local.dtype, device=out_local.device)
    dist.all_gather_into_tensor(recv.view(torch.uint8), send.view(torch.uint8), group=group)
    parts = [recv[r * wmax:r * wmax + widths[r]] for r in range(world)]
    return torch.cat(parts, 0).t().contiguous()


def shard_chunks(n_units: int, world: int, rank: int) -> tuple[int, int]:
    """GDN: [start, stop) of the (batch, head, chunk) matrices rank owns (contiguous, balanced)."""
    return shard_range(n_units, world, rank, 1)


def gather_chunks(t_local: torch.Tensor, n_units: int, world: int, group=None) -> torch.Tensor:
    """All-gather GDN outputs [n_r, C, C] into [n_units, C, C] in unit order."""
    import torch.distributed as dist
    c = t_local.shape[-1]
    sizes = [shard_chunks(n_units, world, r) for r in range(world)]
    nmax = max(b - a for a, b in sizes)
    send = torch.zeros((nmax, c, c), dtype=t_local.dtype, device=t_local.device)
    send[:t_local.shape[0]] = t_local
    recv = torch.empty((world * nmax, c, c), dtype=t_local.dtype, device=t_local.device)
    dist.all_gather_into_tensor(recv.view(torch.uint8), send.view(torch.uint8), group=group)
    return torch.cat([recv[r * nmax:r * nmax + (b - a)] for r, (a, b) in enumerate(sizes)], 0)
