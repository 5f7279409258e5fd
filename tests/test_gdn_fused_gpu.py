"""Fused A construction + inverse (qhtp_gdn_chunk_inverse): from raw keys, beta and per-token log
gates to T = (I - A)^-1, within the reference's oc gate (gdn_solve_oc_check.py:27-31, 1.05e-2) of
the fp64 oracle built the way the reference's chunk kernel builds A, and close to the unfused path
(A formed by the oracle, rounded to bf16, inverted by gdn_inverse)."""
import numpy as np
import pytest
import torch

from oracle import gdn_oracle as G

pytestmark = pytest.mark.gpu


def _run(n, seed):
    from qcom_htp_b200 import gdn_chunk_inverse
    k, beta, g = G.make_kbg(n, 256, 128, seed=seed)
    kt = torch.from_numpy(k).to(torch.bfloat16).cuda()
    T = gdn_chunk_inverse(kt, torch.from_numpy(beta).cuda(), torch.from_numpy(g).cuda())
    torch.cuda.synchronize()
    return k, beta, g, T.cpu().numpy()


@pytest.mark.parametrize("n", [1, 7, 149, 300])
def test_fused_within_oc_gate(n):
    k, beta, g, T = _run(n, 0x6B00 + n)
    A = G.chunk_A_from_kbg(k, beta, g)
    Tref = G.inverse_fp64(A)
    oc = G.oc(T, Tref)
    assert oc < 1e-2 * G.OC_GATE, oc          # bf16 A: ~1e-4; the gate is 1.05e-2
    assert np.all(np.triu(T, 1) == 0.0)       # strict upper triangle written as zeros
    assert np.allclose(np.diagonal(T, axis1=1, axis2=2), 1.0)


def test_fused_matches_unfused_path():
    from qcom_htp_b200 import gdn_inverse
    k, beta, g, T = _run(16, 0x6BAA)
    A = G.chunk_A_from_kbg(k, beta, g).astype(np.float32)
    T2 = gdn_inverse(torch.from_numpy(A).to(torch.bfloat16).cuda()).cpu().numpy()
    assert G.oc(T, T2) < 2e-3


def test_fused_repeat_identical_and_batched_shape():
    from qcom_htp_b200 import gdn_chunk_inverse
    k, beta, g = G.make_kbg(6, 256, 128, seed=0x6BBB)
    kt = torch.from_numpy(k).to(torch.bfloat16).cuda().reshape(2, 3, 256, 128)
    b = torch.from_numpy(beta).cuda().reshape(2, 3, 256)
    gg = torch.from_numpy(g).cuda().reshape(2, 3, 256)
    T1 = gdn_chunk_inverse(kt, b, gg)
    T2 = gdn_chunk_inverse(kt, b, gg)
    torch.cuda.synchronize()
    assert T1.shape == (2, 3, 256, 256)
    assert torch.equal(T1, T2)
