"""torch.ops.qhtp.* on the GPU: the matmul ops give the oracle's bytes (per-channel, LPBQ, per-group), reuse
their prepared weights across calls and re-prepare when a weight tensor changes in place, and the
GDN ops match the direct wrappers; a bad argument surfaces as QhtpError (a RuntimeError)."""
import numpy as np
import pytest
import torch

from oracle import gdn_oracle as G
from oracle import mm_oracle as O
from tests.mm_helpers import to_dev

pytestmark = pytest.mark.gpu


def _args(c):
    fam = c.family
    w = to_dev(O.pack_int4_kpair(c.weight_q)) if fam.weight_bits == 4 else to_dev(c.weight_q.astype(np.int8))
    lp = to_dev(c.lpbq_factor) if fam.schema == "lpbq" else None
    return (w, to_dev(c.weight_scale.astype(np.float32)), to_dev(c.bias_q.astype(np.int32)), lp,
            fam.lpbq_block if fam.schema == "lpbq" else 0, float(c.act_scale), int(c.act_offset),
            float(c.out_scale), int(c.out_offset))


@pytest.mark.parametrize("family,op", [("w4a16_lpbq", "matmul_w4a16"), ("u8i8", "matmul_u8i8"),
                                       ("w4a8_per_channel", "matmul_w4a8")])
def test_matmul_op_bit_exact_and_cached(family, op):
    import qcom_htp_b200.ops as ops
    c = O.generate_case(family, "normal_random", 96, 512, 256)
    args = _args(c)
    fn = getattr(torch.ops.qhtp, op)
    out1 = fn(to_dev(c.act_q), *args)
    n_cached = len(ops._CACHE)
    out2 = fn(to_dev(c.act_q), *args)
    torch.cuda.synchronize()
    assert len(ops._CACHE) == n_cached                     # the second call reused the prepared weights
    np.testing.assert_array_equal(out1.cpu().numpy(), O.exact_output(c))
    assert torch.equal(out1, out2)


@pytest.mark.parametrize("family", ["w4a8_per_group", "w4a16_per_group"])
def test_per_group_op_bit_exact_and_cached(family):
    """torch.ops.qhtp.matmul_per_group_<family>: the oracle's codes, prepared weights reused."""
    import qcom_htp_b200.ops as ops
    c = O.generate_case(family, "normal_random", 80, 320, 192)
    args = (to_dev(O.pack_int4_kpair(c.weight_q)), to_dev(c.weight_scale.astype(np.float32)),
            to_dev(c.bias_float.astype(np.float32)), float(c.act_scale), int(c.act_offset), float(c.out_scale),
            int(c.out_offset))
    fn = getattr(torch.ops.qhtp, "matmul_per_group_" + family.split("_")[0])
    out1 = fn(to_dev(c.act_q), *args)
    n_cached = len(ops._CACHE)
    out2 = fn(to_dev(c.act_q), *args)
    torch.cuda.synchronize()
    assert len(ops._CACHE) == n_cached
    np.testing.assert_array_equal(out1.cpu().numpy(), O.per_group_output(c))
    assert torch.equal(out1, out2)


def test_matmul_op_reprepares_after_inplace_weight_change():
    c = O.generate_case("u8i8", "normal_random", 64, 256, 128)
    args = list(_args(c))
    act = to_dev(c.act_q)
    torch.ops.qhtp.matmul_u8i8(act, *args)
    args[1].mul_(2.0)                                      # weight_scale modified in place
    out = torch.ops.qhtp.matmul_u8i8(act, *args)
    c2 = O.QuantCase(c.family, c.act_q, c.weight_q, (c.weight_scale.astype(np.float32) * 2).astype(c.weight_scale.dtype),
                     c.bias_q, c.act_scale, c.out_scale, c.lpbq_factor, c.lpbq_expanded)
    np.testing.assert_array_equal(out.cpu().numpy(), O.exact_output(c2))


def test_gdn_ops_match_wrappers():
    from qcom_htp_b200 import gdn_chunk_inverse, gdn_inverse
    A = torch.from_numpy(G.make_chunk_A(4, 256, 128, seed=0x51)).to(torch.bfloat16).cuda()
    assert torch.equal(torch.ops.qhtp.gdn_inverse(A), gdn_inverse(A))
    k, beta, g = G.make_kbg(3, 256, 128, seed=0x52)
    kt, bt, gt = torch.from_numpy(k).to(torch.bfloat16).cuda(), torch.from_numpy(beta).cuda(), torch.from_numpy(g).cuda()
    assert torch.equal(torch.ops.qhtp.gdn_chunk_inverse(kt, bt, gt), gdn_chunk_inverse(kt, bt, gt))


def test_op_error_is_runtime_error():
    A = torch.zeros((2, 96, 96), dtype=torch.bfloat16, device="cuda")   # C = 96 is not supported
    with pytest.raises((RuntimeError, ValueError)):
        torch.ops.qhtp.gdn_inverse(A)
