"""ctypes binding of libqhtp.so (the C ABI declared in include/qhtp.h).

The library is the only compute path: if it is missing or fails to load, importing this module
raises, and nothing falls back to a CPU implementation.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqhtp.so"

OK, INVALID_ARGUMENT, UNSUPPORTED, RUNTIME_ERROR = 0, 1, 2, 3

FAMILY = {"u8i8": 0, "w4a8": 1, "w8a16": 2, "w4a16": 3, "w16a16": 4}
SCHEMA = {"per_channel": 0, "lpbq": 1, "per_group": 2}
DEQUANT = {"f32": 0, "exact": 1}


class QhtpMatmulWeights(C.Structure):
    _fields_ = [
        ("family", C.c_uint32), ("schema", C.c_uint32), ("dequant", C.c_uint32),
        ("k", C.c_uint32), ("n", C.c_uint32), ("lpbq_block", C.c_uint32),
        ("weight", C.c_void_p), ("weight_scale", C.c_void_p), ("bias_q", C.c_void_p),
        ("lpbq_block_scale", C.c_void_p),
        ("act_scale", C.c_double), ("act_offset", C.c_int32),
        ("out_scale", C.c_double), ("out_offset", C.c_int32),
        ("bias_float", C.c_void_p),
    ]


class QhtpMatmulPlan(C.Structure):
    _fields_ = [
        ("magic", C.c_uint32),
        ("family", C.c_uint32), ("schema", C.c_uint32), ("dequant", C.c_uint32),
        ("k", C.c_uint32), ("n", C.c_uint32), ("lpbq_block", C.c_uint32),
        ("act_bits", C.c_uint32), ("weight_bits", C.c_uint32), ("out_bits", C.c_uint32),
        ("mode", C.c_uint32), ("a_planes", C.c_uint32), ("ch_per_tile", C.c_uint32),
        ("n_tiles", C.c_uint32), ("k_pad", C.c_uint32),
        ("act_zp", C.c_int32), ("out_zp", C.c_int32), ("out_qmax", C.c_int32),
        ("act_scale", C.c_double), ("out_scale", C.c_double),
        ("act_mant", C.c_uint64), ("act_exp2", C.c_int32), ("flags", C.c_uint32),
        ("out_mant", C.c_uint64), ("out_exp2", C.c_int32),
        ("plane_bytes", C.c_uint64), ("record_bytes", C.c_uint64), ("prepared_bytes", C.c_uint64),
        ("prepared", C.c_void_p),
    ]


class QhtpBuffer(C.Structure):
    _fields_ = [("data", C.c_void_p), ("bytes", C.c_size_t)]


class QhtpConstBuffer(C.Structure):
    _fields_ = [("data", C.c_void_p), ("bytes", C.c_size_t)]


class QhtpPreparedRun(C.Structure):
    _fields_ = [
        ("m", C.c_uint32), ("k", C.c_uint32), ("n", C.c_uint32), ("chain", C.c_uint32),
        ("activation", QhtpConstBuffer), ("plan", C.POINTER(QhtpMatmulPlan)),
        ("scratch", QhtpBuffer), ("output", QhtpBuffer), ("stream", C.c_void_p),
    ]


# every symbol include/qhtp.h declares: name -> (restype, argtypes)
SIGNATURES = {
    "qhtp_status_string": (C.c_char_p, [C.c_int]),
    "qhtp_version": (C.c_char_p, []),
    "qhtp_last_error_string": (C.c_char_p, []),
    "qhtp_matmul_plan": (C.c_int, [C.POINTER(QhtpMatmulWeights), C.POINTER(QhtpMatmulPlan)]),
    "qhtp_matmul_prepared_bytes": (C.c_size_t, [C.POINTER(QhtpMatmulPlan)]),
    "qhtp_matmul_prepare": (C.c_int, [C.POINTER(QhtpMatmulPlan), C.POINTER(QhtpMatmulWeights), C.c_void_p,
                                      C.c_size_t, C.c_void_p]),
    "qhtp_matmul_workspace_bytes": (C.c_size_t, [C.POINTER(QhtpMatmulPlan), C.c_uint32]),
    "qhtp_matmul_run": (C.c_int, [C.POINTER(QhtpMatmulPlan), C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p,
                                  C.c_size_t, C.c_void_p]),
    "qhtp_matmul_run_ctas": (C.c_int, [C.POINTER(QhtpMatmulPlan), C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p,
                                       C.c_size_t, C.c_uint32, C.c_void_p]),
    "qhtp_matmul_run_noalloc": (C.c_int, [C.POINTER(QhtpMatmulPlan), C.c_void_p, C.c_uint32, C.c_void_p,
                                          C.c_void_p]),
    "qhtp_matmul_noalloc_check": (C.c_int, [C.POINTER(QhtpMatmulPlan), C.c_uint32, C.POINTER(C.c_int),
                                            C.c_void_p]),
    "qhtp_matmul_run_host": (C.c_int, [C.POINTER(QhtpMatmulPlan), C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_void_p, C.c_size_t, C.c_uint32, C.POINTER(C.c_uint32),
                                       C.c_void_p]),
    "qhtp_wire_bytes": (C.c_size_t, [C.c_uint32, C.c_uint32, C.c_uint32]),
    "qhtp_weights_from_wire": (C.c_int, [C.c_uint32, C.c_uint32, C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint32,
                                         C.c_void_p, C.c_size_t, C.c_void_p]),
    "qhtp_matmul_check": (C.c_int, [C.POINTER(QhtpMatmulPlan), C.c_void_p, C.c_uint32, C.POINTER(C.c_int),
                                    C.c_void_p]),
    "qhtp_selftest_wait_timeout": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p]),
    "qhtp_selftest_mma_rate": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p]),
    "qhtp_matmul_read_records": (C.c_int, [C.POINTER(QhtpMatmulPlan), C.c_void_p, C.c_size_t, C.c_void_p]),
    "qhtp_lpbq_expand_i8": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p,
                                      C.c_void_p]),
    "qhtp_prepared_run_scratch_bytes": (C.c_size_t, [C.POINTER(QhtpMatmulPlan), C.c_uint32, C.c_uint32]),
    "qhtp_u8i8_run_prepared": (C.c_int, [C.POINTER(QhtpPreparedRun)]),
    "qhtp_w4a8_run_prepared": (C.c_int, [C.POINTER(QhtpPreparedRun)]),
    "qhtp_w8a16_run_prepared": (C.c_int, [C.POINTER(QhtpPreparedRun)]),
    "qhtp_w4a16_run_prepared": (C.c_int, [C.POINTER(QhtpPreparedRun)]),
    "qhtp_w16a16_run_prepared": (C.c_int, [C.POINTER(QhtpPreparedRun)]),
    "qhtp_gdn_inverse_bf16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p]),
    "qhtp_gdn_chunk_inverse": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32,
                                         C.c_int32, C.c_void_p]),
    "qhtp_gdn_solve_u16": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_float, C.c_int32,
                                     C.c_float, C.c_void_p, C.c_void_p]),
    "qhtp_requant_code_host": (C.c_int32, [C.c_int64, C.c_uint64, C.c_int32, C.c_uint32, C.c_int32, C.c_uint64,
                                           C.c_uint64, C.c_int32, C.c_int32, C.c_int32]),
}


class QhtpError(RuntimeError):
    """A qhtp C-ABI call returned a non-OK status."""

    def __init__(self, fn: str, status: int):
        self.status = status
        detail = ""
        if status == RUNTIME_ERROR:
            detail = f": {lib.qhtp_last_error_string().decode()}"
        super().__init__(f"{fn} failed: {status_string(status)} ({status}){detail}")


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `python qcom_htp_b200/build.py` "
                          "(there is no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def status_string(status: int) -> str:
    return lib.qhtp_status_string(status).decode()


def check(fn: str, status: int) -> None:
    if status != OK:
        raise QhtpError(fn, status)


# qhtp_weights_from_wire layouts and flags (QhtpWireFormat, QHTP_WIRE_* in include/qhtp.h)
WIRE_FORMAT = {"w8_raw_kn": 1, "w8_kmajor_tile32": 2, "w8_kmajor_split128": 3, "w4_tile32x64_npair32": 4,
               "w4_kpair": 5, "w4_nmajor_kpair": 6, "w4_nmajor_k4": 7, "w4_kblock32_nmajor_k4": 8,
               "w4_npair_adjacent": 9, "w4_npair_tile32": 10, "w4_full_codes": 11}
WIRE_XOR80, WIRE_HILO, WIRE_BIASED = 1, 2, 4
