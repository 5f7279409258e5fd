"""torch.library custom ops over the C ABI: ``torch.ops.qhtp.*``.

The callers of the library inside a PyTorch model: each op checks its tensors (device, dtype,
contiguity, shape), passes ``data_ptr()`` and the current CUDA stream to the C ABI, allocates its
output, and turns a non-OK status into ``QhtpError`` (a ``RuntimeError``) carrying
``qhtp_status_string``.  Each has a fake (meta) implementation, so shapes propagate through tracing.

    torch.ops.qhtp.matmul_<family>(act, weight, weight_scale, bias_q, lpbq_block_scale, lpbq_block,
                                   act_scale, act_offset, out_scale, out_offset) -> out
        family in u8i8, w4a8, w8a16, w4a16, w16a16: the QNN HmxU8I8ToU8MatMul / HmxU8I4ToU8MatMul /
        HmxU16I8ToU16MatMul / HmxU16I4ToU16MatMul / HmxU16I16ToU16MatMul ops.  Weights in the
        carriers of ``QuantMatMul``; ``lpbq_block_scale`` None (per-channel) or uint8 [N, K/block].
        The prepared weights (qhtp_matmul_prepare) are cached per weight tensors and parameters,
        and rebuilt when a weight tensor is modified in place.
    torch.ops.qhtp.matmul_per_group_<family>(act, weight, weight_scale, bias_float, act_scale, act_offset,
                                             out_scale, out_offset) -> out
        family in w4a8, w4a16: the per-group W4 schema (generate_qnn_matmul_python_cases.py:392-423):
        weight_scale float32 [N, K/64], bias_float float32 [N]; prepared weights cached like the above.
    torch.ops.qhtp.gdn_inverse(A bf16 [..., C, C]) -> T float32
    torch.ops.qhtp.gdn_chunk_inverse(k bf16 [..., 256, 128], beta, g float32 [..., 256]) -> T float32
    torch.ops.qhtp.gdn_solve_u16(A uint16 [..., C, C], zpA, sA, zpT, sT) -> T uint16
"""
from __future__ import annotations

from collections import OrderedDict

import torch

from . import gdn as _gdn
from .matmul import FAMILY_BITS, QuantMatMul

_CACHE: OrderedDict = OrderedDict()
_CACHE_SIZE = 32


def _key(t: torch.Tensor | None):
    return None if t is None else (t.data_ptr(), t._version, tuple(t.shape), t.dtype, t.device)


def _prepared(family, weight, weight_scale, bias_q, lpbq_block_scale, lpbq_block, act_scale, act_offset,
              out_scale, out_offset) -> QuantMatMul:
    key = (family, _key(weight), _key(weight_scale), _key(bias_q), _key(lpbq_block_scale), lpbq_block,
           act_scale, act_offset, out_scale, out_offset)
    op = _CACHE.get(key)
    if op is None:
        kw = {}
        if lpbq_block_scale is not None:
            kw = dict(schema="lpbq", lpbq_block_scale=lpbq_block_scale, lpbq_block=lpbq_block)
        op = QuantMatMul(family, weight, weight_scale, bias_q, act_scale=act_scale, out_scale=out_scale,
                         act_offset=act_offset, out_offset=out_offset, **kw)
        _CACHE[key] = op
        while len(_CACHE) > _CACHE_SIZE:
            _CACHE.popitem(last=False)
    else:
        _CACHE.move_to_end(key)
    return op


def _out_n(family: str, weight: torch.Tensor) -> int:
    return weight.shape[1] if FAMILY_BITS[family][1] == 4 else weight.shape[0]


def _register_matmul(family: str) -> None:
    out_dtype = torch.uint16 if FAMILY_BITS[family][2] == 16 else torch.uint8

    @torch.library.custom_op(f"qhtp::matmul_{family}", mutates_args=(), device_types="cuda")
    def _op(act: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor, bias_q: torch.Tensor,
            lpbq_block_scale: torch.Tensor | None, lpbq_block: int, act_scale: float, act_offset: int,
            out_scale: float, out_offset: int) -> torch.Tensor:
        op = _prepared(family, weight, weight_scale, bias_q, lpbq_block_scale, lpbq_block, act_scale, act_offset,
                       out_scale, out_offset)
        return op(act.contiguous())

    @_op.register_fake
    def _(act, weight, weight_scale, bias_q, lpbq_block_scale, lpbq_block, act_scale, act_offset, out_scale,
          out_offset):
        return act.new_empty((act.shape[0], _out_n(family, weight)), dtype=out_dtype)


for _family in FAMILY_BITS:
    _register_matmul(_family)


def _register_matmul_per_group(family: str) -> None:
    out_dtype = torch.uint16 if FAMILY_BITS[family][2] == 16 else torch.uint8

    @torch.library.custom_op(f"qhtp::matmul_per_group_{family}", mutates_args=(), device_types="cuda")
    def _op(act: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor, bias_float: torch.Tensor,
            act_scale: float, act_offset: int, out_scale: float, out_offset: int) -> torch.Tensor:
        key = ("per_group", family, _key(weight), _key(weight_scale), _key(bias_float), act_scale, act_offset,
               out_scale, out_offset)
        op = _CACHE.get(key)
        if op is None:
            op = QuantMatMul(family, weight, weight_scale, None, schema="per_group", bias_float=bias_float,
                             act_scale=act_scale, out_scale=out_scale, act_offset=act_offset, out_offset=out_offset)
            _CACHE[key] = op
            while len(_CACHE) > _CACHE_SIZE:
                _CACHE.popitem(last=False)
        else:
            _CACHE.move_to_end(key)
        return op(act.contiguous())

    @_op.register_fake
    def _(act, weight, weight_scale, bias_float, act_scale, act_offset, out_scale, out_offset):
        return act.new_empty((act.shape[0], weight.shape[1]), dtype=out_dtype)


for _family in ("w4a8", "w4a16"):
    _register_matmul_per_group(_family)


@torch.library.custom_op("qhtp::gdn_inverse", mutates_args=(), device_types="cuda")
def gdn_inverse_op(A: torch.Tensor) -> torch.Tensor:
    return _gdn.gdn_inverse(A.contiguous())


@gdn_inverse_op.register_fake
def _(A):
    return A.new_empty(A.shape, dtype=torch.float32)


@torch.library.custom_op("qhtp::gdn_chunk_inverse", mutates_args=(), device_types="cuda")
def gdn_chunk_inverse_op(k: torch.Tensor, beta: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    return _gdn.gdn_chunk_inverse(k.contiguous(), beta.contiguous(), g.contiguous())


@gdn_chunk_inverse_op.register_fake
def _(k, beta, g):
    return k.new_empty((*k.shape[:-1], k.shape[-2]), dtype=torch.float32)


@torch.library.custom_op("qhtp::gdn_solve_u16", mutates_args=(), device_types="cuda")
def gdn_solve_u16_op(A: torch.Tensor, zpA: int, sA: float, zpT: int, sT: float) -> torch.Tensor:
    return _gdn.gdn_solve_u16(A.contiguous(), zpA=zpA, sA=sA, zpT=zpT, sT=sT)


@gdn_solve_u16_op.register_fake
def _(A, zpA, sA, zpT, sT):
    return A.new_empty(A.shape, dtype=torch.uint16)
