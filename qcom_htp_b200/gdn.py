"""GDN / KDA chunk triangular inverse T = (I - A)^-1: host side of the B200 replacement for

  gdnbm_solve (example/gdn_native/baremetal/inc/gdnbm.idl:10-12, src/gdnbm_imp.cpp:1207)
  GdnSolve    (example/gdn_native/solve_op/src/GdnSolveOp.cpp:195-281, u16 codes in/out)

A is strictly lower triangular per (batch, head, chunk); chunks are independent.
"""
from __future__ import annotations

import struct
import time

import torch

from . import _lib as L

SUPPORTED_C = (32, 64, 128, 256)


def _stream(stream) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def gdn_inverse(A: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """A bf16 [..., C, C] (CUDA, contiguous) -> T = (I - A)^-1 float32 [..., C, C]."""
    if A.dtype != torch.bfloat16 or not A.is_cuda or not A.is_contiguous():
        raise TypeError("A must be a contiguous CUDA bfloat16 tensor")
    C = A.shape[-1]
    if A.dim() < 2 or A.shape[-2] != C or C not in SUPPORTED_C:
        raise ValueError(f"A must be [..., C, C] with C in {SUPPORTED_C}")
    n = A.numel() // (C * C)
    if out is None:
        out = torch.empty(A.shape, dtype=torch.float32, device=A.device)
    elif out.shape != A.shape or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("bad output tensor")
    L.check("qhtp_gdn_inverse_bf16", L.lib.qhtp_gdn_inverse_bf16(A.data_ptr(), out.data_ptr(), n, C, _stream(stream)))
    return out


def gdn_solve_u16(A: torch.Tensor, *, zpA: int, sA: float, zpT: int, sT: float, out: torch.Tensor | None = None,
                  stream=None) -> torch.Tensor:
    """GdnSolve on u16 codes: value = (code - zp) * scale for A and T (gdn_solve_oc_check.py:28-29)."""
    if A.dtype != torch.uint16 or not A.is_cuda or not A.is_contiguous():
        raise TypeError("A must be a contiguous CUDA uint16 tensor")
    C = A.shape[-1]
    if A.shape[-2] != C or C not in SUPPORTED_C:
        raise ValueError(f"A must be [..., C, C] with C in {SUPPORTED_C}")
    n = A.numel() // (C * C)
    if out is None:
        out = torch.empty(A.shape, dtype=torch.uint16, device=A.device)
    L.check("qhtp_gdn_solve_u16", L.lib.qhtp_gdn_solve_u16(A.data_ptr(), n, C, zpA, float(sA), zpT, float(sT),
                                                           out.data_ptr(), _stream(stream)))
    return out


def _bits_to_float(bits: int) -> float:
    return struct.unpack("<f", struct.pack("<i", bits))[0]


def gdnbm_solve(A: bytes | torch.Tensor, H: int, C: int, zpA: int, zpT: int, sA_bits: int, sT_bits: int,
                nthreads: int = 0):
    """Signature mirror of the reference FastRPC entry ``solve`` (gdnbm.idl:10-12):
    A / T are u16 codes [H, C, C] (bytes), scales passed as float bits.  Returns (rc, T, stats) with
    rc = -1 when C != 256 (the reference's contract, gdnbm_imp.cpp:1210) and stats =
    [elapsed_ns, sms, H].  ``nthreads`` is accepted for signature compatibility; the GPU schedules
    heads itself."""
    del nthreads
    if C != 256:
        return -1, None, [0, 0, H]
    if isinstance(A, (bytes, bytearray)):
        a = torch.frombuffer(bytearray(A), dtype=torch.uint16).reshape(H, C, C).cuda()
    else:
        a = A.reshape(H, C, C).contiguous()
    t0 = time.perf_counter_ns()
    T = gdn_solve_u16(a, zpA=zpA, sA=_bits_to_float(sA_bits), zpT=zpT, sT=_bits_to_float(sT_bits))
    torch.cuda.synchronize()
    el = time.perf_counter_ns() - t0
    sms = torch.cuda.get_device_properties(a.device).multi_processor_count
    return 0, T.cpu().numpy().tobytes(), [el, sms, H]
