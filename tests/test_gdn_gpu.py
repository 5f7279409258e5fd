"""GPU parity of the GDN chunk inverse through the C ABI (oc gate against the fp64 inverse)."""
import numpy as np
import pytest
import torch

from oracle import gdn_oracle as G

pytestmark = pytest.mark.gpu


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda().to(torch.bfloat16)


def test_kat_fixture(golden_dir):
    """Reference known-answer fixture (H=16 -> 2 heads kept, C=256, dense lower A)."""
    from qcom_htp_b200 import gdn_inverse
    z = np.load(golden_dir / "gdn_sbr_kat.npz")
    A = z["A"]
    Ab = _bf16(A)
    T = gdn_inverse(Ab).cpu().numpy()
    Tref = G.inverse_fp64(Ab.float().cpu().numpy())          # exact inverse of the bf16 input
    oc = G.oc(T, Tref)
    print(f"KAT oc vs fp64(bf16 A) = {oc:.3e}; vs fixture Tref = {G.oc(T, z['Tref']):.3e}")
    assert oc <= G.OC_GATE
    assert oc < 2e-3
    assert np.all(np.triu(T, 1) == 0)


@pytest.mark.parametrize("C", [32, 64, 128, 256])
def test_synthetic_chunks(C):
    from qcom_htp_b200 import gdn_inverse
    A = G.make_chunk_A(24, C=C, seed=C)
    T = gdn_inverse(_bf16(A)).cpu().numpy()
    Tref = G.inverse_fp64(A)
    oc = G.oc(T, Tref)
    print(f"C={C} oc={oc:.3e}")
    assert oc <= G.OC_GATE
    assert oc < 1e-4
    assert np.all(np.triu(T, 1) == 0)
    assert np.all(np.diagonal(T, axis1=1, axis2=2) == 1.0)


@pytest.mark.parametrize("C", [64, 256])
def test_dense_random_lower(C):
    """Dense strictly-lower A (no decay): every off-diagonal block matters."""
    from qcom_htp_b200 import gdn_inverse
    rng = np.random.default_rng(C)
    A = np.tril(rng.uniform(-1.0, 1.0, (8, C, C)) / np.sqrt(C), -1).astype(np.float32)
    Ab = _bf16(A)
    T = gdn_inverse(Ab).cpu().numpy()
    oc = G.oc(T, G.inverse_fp64(Ab.float().cpu().numpy()))
    print(f"dense C={C} oc={oc:.3e}")
    assert oc <= G.OC_GATE


def test_upper_triangle_input_ignored():
    from qcom_htp_b200 import gdn_inverse
    A = G.make_chunk_A(4, C=256, seed=1)
    noisy = A + np.triu(np.full_like(A, 7.0))
    T1 = gdn_inverse(_bf16(A)).cpu().numpy()
    T2 = gdn_inverse(_bf16(noisy)).cpu().numpy()
    np.testing.assert_array_equal(T1, T2)


def test_batched_shape_and_determinism():
    from qcom_htp_b200 import gdn_inverse
    A = G.make_chunk_A(2 * 3 * 5, C=256, seed=5).reshape(2, 3, 5, 256, 256)
    Ab = _bf16(A)
    T1 = gdn_inverse(Ab)
    T2 = gdn_inverse(Ab)
    assert T1.shape == (2, 3, 5, 256, 256)
    assert torch.equal(T1, T2)


def test_u16_codes_carrier():
    """gdnbm_solve / GdnSolve carrier: u16 codes with zero-point 32768 and the gate's default scales
    (gdn_solve_oc_check.py:20-23)."""
    from qcom_htp_b200 import gdn_solve_u16
    sA, sT, zp = 2.770166930875267e-05, 6.103701895199438e-05, 32768
    A = G.make_chunk_A(8, C=256, seed=3, as_bf16=False)
    Ac = G.to_codes(A, sA, zp)
    Tc = gdn_solve_u16(torch.from_numpy(Ac).cuda(), zpA=zp, sA=sA, zpT=zp, sT=sT).cpu().numpy()
    T = G.from_codes(Tc, sT, zp)
    Tref = G.inverse_fp64(G.from_codes(Ac, sA, zp))
    oc = G.oc(T, Tref)
    print(f"u16 codes oc={oc:.3e}")
    assert oc <= G.OC_GATE


def test_gdnbm_signature_mirror():
    import struct
    from qcom_htp_b200 import gdnbm_solve
    sA, sT, zp = 2.770166930875267e-05, 6.103701895199438e-05, 32768
    bits = lambda f: struct.unpack("<i", struct.pack("<f", f))[0]
    A = G.make_chunk_A(4, C=256, seed=8, as_bf16=False)
    Ac = G.to_codes(A, sA, zp)
    rc, Tb, stats = gdnbm_solve(Ac.tobytes(), 4, 256, zp, zp, bits(sA), bits(sT), 4)
    assert rc == 0 and stats[2] == 4
    T = G.from_codes(np.frombuffer(Tb, np.uint16).reshape(4, 256, 256), np.float32(sT), zp)
    assert G.oc(T, G.inverse_fp64(G.from_codes(Ac, np.float32(sA), zp))) <= G.OC_GATE
    rc, _, _ = gdnbm_solve(Ac.tobytes(), 4, 128, zp, zp, bits(sA), bits(sT), 4)
    assert rc == -1      # the reference's C != 256 contract


@pytest.mark.parametrize("n_chunks", [1, 64, 149])
def test_u16_codes_c256_structure_and_gate(n_chunks):
    """u16 carrier at C=256 (the tensor-core kernel): upper triangle exactly the zero code, diagonal
    exactly the code of 1.0, oc against the fp64 inverse of the decoded input within the gate.
    149 chunks = one more than the 148 persistent CTAs (a second pass for one CTA)."""
    from qcom_htp_b200 import gdn_solve_u16
    sA, sT, zp = 2.770166930875267e-05, 6.103701895199438e-05, 32768
    A = G.make_chunk_A(n_chunks, C=256, seed=0xC0DE + n_chunks, as_bf16=False)
    Ac = G.to_codes(A, sA, zp)
    Tc = gdn_solve_u16(torch.from_numpy(Ac).cuda(), zpA=zp, sA=sA, zpT=zp, sT=sT).cpu().numpy()
    iu = np.triu_indices(256, 1)
    assert np.all(Tc[:, iu[0], iu[1]] == zp)
    one = int(np.rint(np.float32(1.0) * np.float32(1.0 / np.float32(sT)))) + zp
    assert np.all(np.diagonal(Tc, axis1=1, axis2=2) == min(one, 65535))
    T = G.from_codes(Tc, np.float32(sT), zp)
    oc = G.oc(T, G.inverse_fp64(G.from_codes(Ac, np.float32(sA), zp)))
    print(f"u16 C=256 n={n_chunks} oc={oc:.3e}")
    assert oc <= G.OC_GATE


def test_u16_codes_c128_small_kernel():
    """C=128 u16 (served by the first kernel): same contract."""
    from qcom_htp_b200 import gdn_solve_u16
    sA, sT, zp = 2.770166930875267e-05, 6.103701895199438e-05, 32768
    A = G.make_chunk_A(16, C=128, seed=0x128, as_bf16=False)
    Ac = G.to_codes(A, sA, zp)
    Tc = gdn_solve_u16(torch.from_numpy(Ac).cuda(), zpA=zp, sA=sA, zpT=zp, sT=sT).cpu().numpy()
    T = G.from_codes(Tc, np.float32(sT), zp)
    assert G.oc(T, G.inverse_fp64(G.from_codes(Ac, np.float32(sA), zp))) <= G.OC_GATE


@pytest.mark.parametrize("n_chunks", [1, 149])
def test_bf16_c256_chunk_counts(n_chunks):
    from qcom_htp_b200 import gdn_inverse
    A = G.make_chunk_A(n_chunks, C=256, seed=0xB16 + n_chunks)
    T = gdn_inverse(_bf16(A)).cpu().numpy()
    assert G.oc(T, G.inverse_fp64(A)) < 1e-4
    assert np.all(np.triu(T, 1) == 0)
