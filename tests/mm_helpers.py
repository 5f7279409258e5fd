"""Test helpers: move an oracle case onto the GPU in the C-ABI carrier formats and run it."""
from __future__ import annotations

import numpy as np
import torch

from oracle import mm_oracle as O

KERNEL_FAMILY = {"u8i8": "u8i8", "w4a8_per_channel": "w4a8", "w4a8_lpbq": "w4a8", "w8a16": "w8a16",
                 "w4a16_per_channel": "w4a16", "w4a16_lpbq": "w4a16", "w16a16": "w16a16",
                 "w4a8_per_group": "w4a8", "w4a16_per_group": "w4a16"}


def to_dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def build_op(case: O.QuantCase, dequant: str | None = None):
    from qcom_htp_b200 import QuantMatMul
    fam = case.family
    kf = fam.kernel if fam.name not in KERNEL_FAMILY else KERNEL_FAMILY[fam.name]
    if fam.weight_bits == 4:
        w = to_dev(O.pack_int4_kpair(case.weight_q))
    elif fam.weight_bits == 16:
        w = to_dev(case.weight_q.astype(np.int16))
    else:
        w = to_dev(case.weight_q.astype(np.int8))
    kw = {}
    if fam.schema == "lpbq":
        kw = dict(schema="lpbq", lpbq_block_scale=to_dev(case.lpbq_factor), lpbq_block=fam.lpbq_block)
    if fam.schema == "per_group":
        return QuantMatMul(kf, w, to_dev(case.weight_scale.astype(np.float32)), None, schema="per_group",
                           bias_float=to_dev(case.bias_float.astype(np.float32)), act_scale=case.act_scale,
                           out_scale=case.out_scale, act_offset=case.act_offset, out_offset=case.out_offset)
    return QuantMatMul(kf, w, to_dev(case.weight_scale.astype(np.float32)), to_dev(case.bias_q.astype(np.int32)),
                       act_scale=case.act_scale, out_scale=case.out_scale, act_offset=case.act_offset,
                       out_offset=case.out_offset, dequant=dequant, **kw)


def run_case(case: O.QuantCase, dequant: str | None = None, op=None) -> np.ndarray:
    op = op or build_op(case, dequant)
    out = op(to_dev(case.act_q))
    op.check_device(case.act_q.shape[0])
    return out.cpu().numpy()


def make_w16a16_case(m: int, k: int, n: int, seed: int = 0xB17E) -> O.QuantCase:
    """W16A16 case: u16 activations, int16 per-channel weights (full int16 range), int32 bias."""
    rng = np.random.default_rng(seed)
    fam = O.FAMILIES["w16a16"]
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(n) * 0.1).astype(np.float32)
    return O.quantize_case(fam, x, w, b, with_reference_output=False)
