"""qcom_htp_b200: B200-native (sm_100a) quantized MatMul family and GDN chunk inverse.

A drop-in for two hot paths of zzh-www/qcom_htp: the QNN custom MatMul ops (u8i8, W4A8, W8A16,
W4A16 per-channel / LPBQ, W16A16) and the GDN/KDA triangular inverse.  Compute runs in
``libqhtp.so`` (hand-written CUDA, C ABI in ``include/qhtp.h``); importing this package fails if
that library is missing -- there is no CPU fallback.
"""
from . import _lib  # noqa: F401  (loads libqhtp.so or raises)
from ._lib import QhtpError
from . import ops  # noqa: F401  (registers torch.ops.qhtp.*)
from .gdn import gdn_chunk_inverse, gdn_inverse, gdn_solve_u16, gdnbm_solve
from .matmul import (QuantMatMul, hmx_u8i4_to_u8_matmul, hmx_u8i8_to_u8_matmul, hmx_u16i4_to_u16_matmul,
                     hmx_u16i8_to_u16_matmul, hmx_u16i16_to_u16_matmul, lpbq_expand_i8, weights_from_wire)

__all__ = ["QhtpError", "QuantMatMul", "gdn_chunk_inverse", "gdn_inverse", "gdn_solve_u16", "gdnbm_solve", "hmx_u8i8_to_u8_matmul",
           "hmx_u8i4_to_u8_matmul", "hmx_u16i8_to_u16_matmul", "hmx_u16i4_to_u16_matmul",
           "hmx_u16i16_to_u16_matmul", "lpbq_expand_i8", "weights_from_wire"]
