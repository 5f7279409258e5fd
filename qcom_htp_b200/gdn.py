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


def gdn_chunk_inverse(k: torch.Tensor, beta: torch.Tensor, g: torch.Tensor, out: torch.Tensor | None = None,
                      stream=None) -> torch.Tensor:
    """The chunk's A built from the gated-delta-rule inputs and inverted in one kernel
    (qhtp_gdn_chunk_inverse; Stage A of gdn_chunk, scripts/gdn_ref_kernel.py:66-82): raw keys k bf16
    [..., 256, 128], beta and per-token log gates g float32 [..., 256] -> T = (I - A)^-1 float32
    [..., 256, 256]."""
    if k.dtype != torch.bfloat16 or not k.is_cuda or not k.is_contiguous():
        raise TypeError("k must be a contiguous CUDA bfloat16 tensor")
    if k.dim() < 2 or k.shape[-2] != 256 or k.shape[-1] != 128:
        raise ValueError("k must be [..., 256, 128]")
    lead = k.shape[:-1]
    for name, t in (("beta", beta), ("g", g)):
        if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous() or t.shape != lead:
            raise TypeError(f"{name} must be a contiguous CUDA float32 tensor of shape {tuple(lead)}")
    n = k.numel() // (256 * 128)
    shape = (*k.shape[:-2], 256, 256)
    if out is None:
        out = torch.empty(shape, dtype=torch.float32, device=k.device)
    elif out.shape != shape or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("bad output tensor")
    L.check("qhtp_gdn_chunk_inverse", L.lib.qhtp_gdn_chunk_inverse(
        k.data_ptr(), beta.data_ptr(), g.data_ptr(), out.data_ptr(), n, 256, 128, _stream(stream)))
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
