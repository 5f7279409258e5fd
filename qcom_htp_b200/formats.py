"""Weight carrier formats accepted by the C ABI (torch tensors, CPU or CUDA).

int4 weights travel as K-pair bytes [K/2, N]: byte (k>>1)*N + n holds k even in the low nibble and
k odd in the high nibble, two's-complement nibbles -- the LPBQ carrier of the reference
(example/qnn_hmx_matmul_common/HmxW4LpbqExpandToI8Op.cpp:5,32-40).  8- and 16-bit weights are
row-major [N, K] (the reference's weight_q_nk).
"""
from __future__ import annotations

import torch


def pack_int4_kpair(q_nk: torch.Tensor) -> torch.Tensor:
    """int4 codes [N, K] (int8 in [-8, 7]) -> uint8 K-pair bytes [K/2, N]."""
    if q_nk.dim() != 2 or q_nk.shape[1] % 2:
        raise ValueError("expected [N, K] with even K")
    if int(q_nk.min()) < -8 or int(q_nk.max()) > 7:
        raise ValueError("int4 codes must lie in [-8, 7]")
    nib = (q_nk.to(torch.int16) & 0xF).to(torch.uint8)
    packed = nib[:, 0::2] | (nib[:, 1::2] << 4)
    return packed.t().contiguous()


def unpack_int4_kpair(packed: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """uint8 K-pair bytes [K/2, N] -> int8 codes [N, K]."""
    p = packed.reshape(k // 2, n).t().to(torch.int16)
    q = torch.empty((n, k), dtype=torch.int16, device=packed.device)
    q[:, 0::2] = p & 0xF
    q[:, 1::2] = p >> 4
    q = torch.where(q >= 8, q - 16, q)
    return q.to(torch.int8)


def lpbq_expand_reference_layout(q4_nk: torch.Tensor, block_scale: torch.Tensor, block: int) -> torch.Tensor:
    """Host-side statement of the LPBQ expand rule: sat_int8(q4 * factor[n, k // block]) -> int8 [N, K]."""
    f = block_scale.to(torch.int32).repeat_interleave(block, dim=1)
    return (q4_nk.to(torch.int32) * f).clamp(-128, 127).to(torch.int8)
