"""Quantized MatMul family: host side of the B200 replacement for the reference's custom ops.

Reference ops and their counterparts here (all with QNN affine semantics, offset = -zero_point):

  HmxU8I8ToU8MatMul   (example/qnn_hmx_matmul_u8i8/src/HmxU8I8ToU8MatMulOp.cpp:481-792)   family "u8i8"
  HmxU8I4ToU8MatMul   (example/qnn_hmx_matmul_w4a8/src/HmxU8I4ToU8MatMulOp.cpp:1113-1122) family "w4a8"
  HmxU16I8ToU16MatMul (example/qnn_hmx_matmul_w8a16/src/HmxU16I8ToU16MatMulOp.cpp)        family "w8a16"
  HmxU16I4ToU16MatMul (example/qnn_hmx_matmul_w4a16/src/HmxU16I4ToU16MatMulOp.cpp)        family "w4a16"
  HmxU16I16ToU16MatMul(example/qnn_hmx_matmul_w16a16/src/HmxU16I16ToU16MatMulOp.cpp:1214) family "w16a16"
  HmxW4LpbqExpandToI8 (example/qnn_hmx_matmul_common/HmxW4LpbqExpandToI8Op.cpp:49-157)    lpbq_expand_i8

Like the reference's QHPI precompute + hot callback split (HmxU8I8ToU8MatMulOp.cpp:218-286 and
:289), a ``QuantMatMul`` prepares once (weight byte planes, effective bias, requant constants) and
then each call runs one GEMM kernel.  Unlike the QHPI kernels, which return success on bad inputs,
every error raises ``QhtpError``.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib as L

FAMILY_BITS = {"u8i8": (8, 8, 8), "w4a8": (8, 4, 8), "w8a16": (16, 8, 16), "w4a16": (16, 4, 16),
               "w16a16": (16, 16, 16)}

RECORD_DTYPE = np.dtype([("beff", "<i8"), ("cmn", "<u8"), ("m_q", "<i4"), ("wbits", "<u4"), ("tn", "<i4"),
                         ("lo_win", "<i4")])


def _stream_handle(stream) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else int(t.data_ptr())


def _dt(bits: int) -> torch.dtype:
    return torch.uint16 if bits == 16 else torch.uint8


class QuantMatMul:
    """A prepared quantized MatMul: out[M,N] = requant(act[M,K] x weight[N,K]^T + bias).

    Parameters (tensors on the CUDA device the op runs on)
    ----------
    family        "u8i8" | "w4a8" | "w8a16" | "w4a16" | "w16a16"
    weight        int8 [N,K] (8-bit), uint8 K-pair [K/2,N] (int4), int16 [N,K] (W16A16)
    weight_scale  float32 [N] per-output-channel scale (LPBQ: the per-channel base scale;
                  per_group: float32 [N, K/64], one scale per 64 weights along K)
    bias_q        int32 [N], quantized at act_scale * weight_scale (None for per_group)
    bias_float    float32 [N], per_group only: the float bias the reference keeps unquantized
                  (generate_qnn_matmul_python_cases.py:460-470)
    act_scale/out_scale, act_offset/out_offset  QNN affine parameters (offset = -zero_point);
                  offsets default to the family's fixed zero points (A8: 128, A16/out16: 32768, out8: 0)
    schema        "per_channel" | "lpbq" | "per_group"; LPBQ needs lpbq_block_scale uint8 [N, K/lpbq_block];
                  per_group (W4 families) needs K a multiple of 64 above 64
    dequant       "f32" (float32 weight dequant, the reference oracle's rule; default for 4/8-bit)
                  or "exact" (w*s exactly; the only mode for W16A16)
    """

    def __init__(self, family: str, weight: torch.Tensor, weight_scale: torch.Tensor, bias_q: torch.Tensor | None,
                 *, act_scale: float, out_scale: float, act_offset: int | None = None, out_offset: int | None = None,
                 schema: str = "per_channel", lpbq_block_scale: torch.Tensor | None = None, lpbq_block: int = 0,
                 dequant: str | None = None, bias_float: torch.Tensor | None = None, stream=None):
        if family not in FAMILY_BITS:
            raise ValueError(f"unknown family {family!r}")
        a_bits, w_bits, o_bits = FAMILY_BITS[family]
        if dequant is None:
            dequant = "exact" if w_bits == 16 else "f32"
        self.family, self.schema, self.dequant = family, schema, dequant
        self.act_bits, self.weight_bits, self.out_bits = a_bits, w_bits, o_bits
        if act_offset is None:
            act_offset = -(1 << (a_bits - 1))
        if out_offset is None:
            out_offset = -32768 if o_bits == 16 else 0
        if w_bits == 4:
            k2, n = weight.shape
            k = 2 * k2
            want = torch.uint8
        else:
            n, k = weight.shape
            want = torch.int16 if w_bits == 16 else torch.int8
        if weight.dtype != want:
            raise TypeError(f"{family}: weight must be {want}, got {weight.dtype}")
        if schema not in L.SCHEMA:
            raise ValueError(f"unknown schema {schema!r}")
        per_group = schema == "per_group"
        bias_t = bias_float if per_group else bias_q
        if bias_t is None:
            raise ValueError("per_group needs bias_float" if per_group else "bias_q is required")
        for name, t in (("weight", weight), ("weight_scale", weight_scale), ("bias", bias_t)):
            if not t.is_cuda or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous CUDA tensor")
        if weight_scale.dtype != torch.float32 or bias_t.dtype != (torch.float32 if per_group else torch.int32):
            raise TypeError("weight_scale must be float32 and the bias " + ("float32" if per_group else "int32"))
        want_scales = n * (k // 64) if per_group else n
        if weight_scale.numel() != want_scales or bias_t.numel() != n:
            raise ValueError(f"weight_scale must have {want_scales} elements and the bias N")
        if schema == "lpbq":
            if lpbq_block_scale is None or lpbq_block_scale.dtype != torch.uint8:
                raise ValueError("LPBQ needs lpbq_block_scale uint8 [N, K/block]")
            if lpbq_block <= 0 or k % lpbq_block or lpbq_block_scale.numel() != n * (k // lpbq_block):
                raise ValueError("bad LPBQ block / block-scale shape")
            lpbq_block_scale = lpbq_block_scale.contiguous()
        self.k, self.n = k, n
        self.device = weight.device
        self._keep = [weight, weight_scale, bias_t, lpbq_block_scale]
        self._w = L.QhtpMatmulWeights(
            family=L.FAMILY[family], schema=L.SCHEMA[schema], dequant=L.DEQUANT[dequant], k=k, n=n,
            lpbq_block=lpbq_block if schema == "lpbq" else 0,
            weight=_ptr(weight), weight_scale=_ptr(weight_scale), bias_q=None if per_group else _ptr(bias_q),
            lpbq_block_scale=_ptr(lpbq_block_scale),
            act_scale=float(act_scale), act_offset=int(act_offset), out_scale=float(out_scale),
            out_offset=int(out_offset), bias_float=_ptr(bias_float) if per_group else None)
        self.plan = L.QhtpMatmulPlan()
        L.check("qhtp_matmul_plan", L.lib.qhtp_matmul_plan(C.byref(self._w), C.byref(self.plan)))
        with torch.cuda.device(self.device):
            self.prepared = torch.empty(int(self.plan.prepared_bytes), dtype=torch.uint8, device=self.device)
            L.check("qhtp_matmul_prepare", L.lib.qhtp_matmul_prepare(
                C.byref(self.plan), C.byref(self._w), _ptr(self.prepared), self.prepared.numel(),
                _stream_handle(stream)))
        self._ws: dict[int, torch.Tensor] = {}

    # ------------------------------------------------------------------ run
    def workspace(self, m: int) -> torch.Tensor:
        ws = self._ws.get(m)
        if ws is None:
            nbytes = int(L.lib.qhtp_matmul_workspace_bytes(C.byref(self.plan), m))
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._ws[m] = ws
        return ws

    def __call__(self, act: torch.Tensor, out: torch.Tensor | None = None, stream=None, max_ctas: int = 0) -> torch.Tensor:
        """out[M, N] = the quantized MatMul of act[M, K].  max_ctas > 0 limits the row-tiled GEMM to that
        many SMs (qhtp_matmul_run_ctas), leaving the rest to concurrent work on other streams."""
        if act.dim() != 2 or act.shape[1] != self.k:
            raise ValueError(f"act must be [M, {self.k}]")
        if act.dtype != _dt(self.act_bits) or not act.is_cuda or not act.is_contiguous():
            raise TypeError(f"act must be a contiguous CUDA {_dt(self.act_bits)} tensor")
        m = act.shape[0]
        if out is None:
            out = torch.empty((m, self.n), dtype=_dt(self.out_bits), device=act.device)
        elif out.shape != (m, self.n) or out.dtype != _dt(self.out_bits) or not out.is_contiguous():
            raise ValueError("bad output tensor")
        ws = self.workspace(m)
        L.check("qhtp_matmul_run", L.lib.qhtp_matmul_run_ctas(
            C.byref(self.plan), _ptr(act), m, _ptr(out), _ptr(ws), ws.numel(), max_ctas, _stream_handle(stream)))
        return out

    def run_host(self, act_host: torch.Tensor, out_host: torch.Tensor | None = None, chunk_rows: int = 0,
                 stream=None) -> torch.Tensor:
        """qhtp_matmul_run_host: activation and output in (pinned) host memory; row chunks whose
        copies in both directions overlap the GEMMs of the other chunks.  The device staging buffers
        and the workspace are kept per M.  Returns when the work is enqueued: the output is complete
        once `stream` is (synchronize before reading it)."""
        if act_host.dim() != 2 or act_host.shape[1] != self.k or act_host.is_cuda:
            raise ValueError(f"act_host must be a host [M, {self.k}] tensor")
        if act_host.dtype != _dt(self.act_bits) or not act_host.is_contiguous():
            raise TypeError(f"act_host must be a contiguous {_dt(self.act_bits)} tensor")
        m = act_host.shape[0]
        if out_host is None:
            out_host = torch.empty((m, self.n), dtype=_dt(self.out_bits)).pin_memory()
        elif (out_host.shape != (m, self.n) or out_host.dtype != _dt(self.out_bits) or out_host.is_cuda
              or not out_host.is_contiguous()):
            raise ValueError("bad host output tensor")
        key = ("host", m, chunk_rows)
        st = self._ws.get(key)
        if st is None:
            nbytes = int(L.lib.qhtp_matmul_workspace_bytes(C.byref(self.plan), m))  # >= any chunk's
            st = (torch.empty((m, self.k), dtype=_dt(self.act_bits), device=self.device),
                  torch.empty((m, self.n), dtype=_dt(self.out_bits), device=self.device),
                  torch.zeros(nbytes, dtype=torch.uint8, device=self.device))
            self._ws[key] = st
        act_d, out_d, ws = st
        used = C.c_uint32(0)
        L.check("qhtp_matmul_run_host", L.lib.qhtp_matmul_run_host(
            C.byref(self.plan), act_host.data_ptr(), m, out_host.data_ptr(), _ptr(act_d), _ptr(out_d), _ptr(ws),
            ws.numel(), chunk_rows, C.byref(used), _stream_handle(stream)))
        self.host_chunk_rows = used.value
        self._host_ws = ws
        return out_host

    def check_host(self, stream=None) -> None:
        """check_device for the last run_host call (its workspace, its chunk size)."""
        self.check_device(self.host_chunk_rows, stream, workspace=self._host_ws)

    def check_device(self, m: int, stream=None, workspace: torch.Tensor | None = None) -> None:
        """Synchronize and raise if a kernel recorded a device-side error for workspace(m)."""
        code = C.c_int(0)
        ws = self.workspace(m) if workspace is None else workspace
        st = L.lib.qhtp_matmul_check(C.byref(self.plan), _ptr(ws), m, C.byref(code), _stream_handle(stream))
        if st != L.OK:
            raise L.QhtpError(f"qhtp_matmul_check (device code {code.value})", st)

    def lo_residual_launch(self, m: int, max_ctas: int = 0) -> bool:
        """Whether a row-tiled launch over M rows leaves the lo-plane x e' product out of its MMAs (the
        library's rule, qgemm.cu lo_residual_launch): the bound is valid (plan flag 1) and either the
        caller forces it (flag 16) or prepare found it worth it (flag 8) and the launch has at least
        three waves of 128 x 128 tiles on the SMs it may use.  Descriptive only: outputs are the same."""
        f = int(self.plan.flags)
        if not f & 1:
            return False
        if f & 16:
            return True
        slots = torch.cuda.get_device_properties(self.device).multi_processor_count
        if 0 < max_ctas < slots:
            slots = max_ctas
        tiles = ((m + 127) // 128) * int(self.plan.n_tiles)
        return bool(f & 8) and tiles >= 3 * slots

    def scratch_bytes(self, m: int, chain: int = 1) -> int:
        """Device scratch bytes run_prepared needs for M rows (qhtp_prepared_run_scratch_bytes)."""
        return int(L.lib.qhtp_prepared_run_scratch_bytes(C.byref(self.plan), m, chain))

    def records(self, stream=None) -> np.ndarray:
        """The prepared per-channel records (the B200 "sidecar"), padded to the channel tile."""
        npad = int(self.plan.n_tiles) * int(self.plan.ch_per_tile)
        buf = np.zeros(npad, RECORD_DTYPE)
        L.check("qhtp_matmul_read_records", L.lib.qhtp_matmul_read_records(
            C.byref(self.plan), buf.ctypes.data, buf.nbytes, _stream_handle(stream)))
        return buf

    def run_prepared(self, act: torch.Tensor, out: torch.Tensor, chain: int = 1, stream=None,
                     scratch: torch.Tensor | None = None) -> torch.Tensor:
        """The qhtp_<family>_run_prepared entry point (handwritten_hmx_matmul.h:46-50 counterpart).
        chain > 1 applies the op `chain` times, each output feeding the next activation.  `scratch`:
        a caller-owned uint8 device buffer of at least scratch_bytes(M, chain) bytes (else one is
        allocated for the call)."""
        m = act.shape[0]
        nbytes = self.scratch_bytes(m, chain)
        if scratch is None:
            scratch = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        elif scratch.numel() * scratch.element_size() < nbytes or not scratch.is_contiguous():
            raise ValueError(f"scratch must be a contiguous device buffer of at least {nbytes} bytes")
        run = L.QhtpPreparedRun(
            m=m, k=self.k, n=self.n, chain=chain,
            activation=L.QhtpConstBuffer(_ptr(act), act.numel() * act.element_size()),
            plan=C.pointer(self.plan),
            scratch=L.QhtpBuffer(_ptr(scratch), nbytes),
            output=L.QhtpBuffer(_ptr(out), out.numel() * out.element_size()),
            stream=_stream_handle(stream))
        fn = getattr(L.lib, f"qhtp_{self.family}_run_prepared")
        L.check(f"qhtp_{self.family}_run_prepared", fn(C.byref(run)))
        self._last_scratch = scratch   # keep alive until the stream is done with it
        return out


def lpbq_expand_i8(w4_kpair: torch.Tensor, block_scale: torch.Tensor, k: int, n: int, block: int,
                   stream=None) -> torch.Tensor:
    """HmxW4LpbqExpandToI8: int4 K-pair [K/2,N] x uint8 [N,K/block] -> int8 [N,K] (row-major)."""
    out = torch.empty((n, k), dtype=torch.int8, device=w4_kpair.device)
    L.check("qhtp_lpbq_expand_i8", L.lib.qhtp_lpbq_expand_i8(
        _ptr(w4_kpair), _ptr(block_scale.contiguous()), k, n, block, _ptr(out), _stream_handle(stream)))
    return out


def _one_shot(family, act, weight, weight_scale, bias_q, act_scale, out_scale, **kw):
    return QuantMatMul(family, weight, weight_scale, bias_q, act_scale=act_scale, out_scale=out_scale, **kw)(act)


def hmx_u8i8_to_u8_matmul(act, weight, weight_scale, bias_q, *, act_scale, out_scale, **kw):
    """One-shot HmxU8I8ToU8MatMul (prepare + run)."""
    return _one_shot("u8i8", act, weight, weight_scale, bias_q, act_scale, out_scale, **kw)


def hmx_u8i4_to_u8_matmul(act, weight, weight_scale, bias_q, *, act_scale, out_scale, **kw):
    """One-shot HmxU8I4ToU8MatMul (W4A8, per-channel or LPBQ)."""
    return _one_shot("w4a8", act, weight, weight_scale, bias_q, act_scale, out_scale, **kw)


def hmx_u16i8_to_u16_matmul(act, weight, weight_scale, bias_q, *, act_scale, out_scale, **kw):
    """One-shot HmxU16I8ToU16MatMul (W8A16)."""
    return _one_shot("w8a16", act, weight, weight_scale, bias_q, act_scale, out_scale, **kw)


def hmx_u16i4_to_u16_matmul(act, weight, weight_scale, bias_q, *, act_scale, out_scale, **kw):
    """One-shot HmxU16I4ToU16MatMul (W4A16, per-channel or LPBQ)."""
    return _one_shot("w4a16", act, weight, weight_scale, bias_q, act_scale, out_scale, **kw)


def hmx_u16i16_to_u16_matmul(act, weight, weight_scale, bias_q, *, act_scale, out_scale, **kw):
    """One-shot HmxU16I16ToU16MatMul (W16A16 as two byte-weight passes)."""
    return _one_shot("w16a16", act, weight, weight_scale, bias_q, act_scale, out_scale, **kw)


def requant_code_host(T: int, cm: int, cshift: int, mul: int, e2: int, act_mant: int, out_mant: int,
                      out_exp2: int, zp_out: int, qmax: int) -> int:
    """The kernels' exact requant decision, evaluated on the host (testing aid)."""
    return int(L.lib.qhtp_requant_code_host(T, cm, cshift, mul, e2, act_mant, out_mant, out_exp2, zp_out, qmax))


def weights_from_wire(fmt: str | int, wire: torch.Tensor, k: int, n: int, *, xor80: bool = False, hilo: bool = False,
                      biased: bool = False, stream=None) -> torch.Tensor:
    """Decode a weight in one of the reference's wire layouts (its QNN initializer bytes, on the
    device) into this library's plain carrier: int8 [N, K] for the W8 layouts, the int4 K-pair bytes
    [K/2, N] (uint8) for the W4 layouts.  ``fmt``: a key of ``_lib.WIRE_FORMAT`` or its id."""
    f = L.WIRE_FORMAT[fmt] if isinstance(fmt, str) else int(fmt)
    flags = (L.WIRE_XOR80 if xor80 else 0) | (L.WIRE_HILO if hilo else 0) | (L.WIRE_BIASED if biased else 0)
    if not wire.is_cuda or not wire.is_contiguous():
        raise TypeError("wire must be a contiguous CUDA tensor")
    w8 = f <= L.WIRE_FORMAT["w8_kmajor_split128"]
    out = torch.empty((n, k) if w8 else (k // 2, n), dtype=torch.int8 if w8 else torch.uint8, device=wire.device)
    L.check("qhtp_weights_from_wire", L.lib.qhtp_weights_from_wire(
        f, flags, _ptr(wire), wire.numel() * wire.element_size(), k, n, _ptr(out), out.numel(),
        _stream_handle(stream)))
    return out
