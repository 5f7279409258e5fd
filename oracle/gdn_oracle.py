"""GDN/KDA chunk triangular-inverse oracle (TEST INFRASTRUCTURE ONLY -- the checker, never the product).

* ``make_chunk_A``   : the synthetic A of BASELINE.json config "GDN chunk triangular inverse":
                       A = -strict_tril(beta_i * (k_i . k_j) * exp(g_i - g_j)), k L2-normalised,
                       beta = sigmoid(N(0,1)), g = cumsum(logsigmoid(0.5*N(0,1) - 2)) within the chunk.
                       This is the chunk-local A of ``scripts/gdn_ref_kernel.py:71-87`` (its l2norm at
                       :31-32, the decay at :79-83; the sign there is folded into A so that
                       T = (I - A)^-1, as in ``solve_op/gdn_solve_ref.c:1``).
* ``chunk_A_from_kbg``: the same A from the raw gated-delta-rule inputs (k, beta, per-token log
                       gates), as the reference's fused chunk kernel builds it (Stage A of
                       ``gdn_chunk``, ``scripts/gdn_ref_kernel.py:66-82``); ``make_kbg`` draws them.
* ``inverse_fp64``   : the precision oracle, fp64 ``inv(I - A)`` per chunk
                       (``scripts/gdn_solve_oc_check.py:30``), computed by triangular solve.
* ``oc``             : ``||T - Tref||_F / (||Tref||_F + 1e-12)`` over all chunks jointly
                       (``scripts/gdn_solve_oc_check.py:31``), gate 1.05e-2.
* ``block_model``    : the reference's BL=16 int16-code forward substitution + fp64 block merge,
                       restated from ``example/gdn_native/solve_op/gdn_solve_ref.c:16-69``; the C
                       restatement ``gdn_block_ref.c`` in this folder is the timed CPU baseline.
* ``codes`` helpers  : the u16 code carrier of ``gdnbm_solve`` / ``GdnSolve``
                       (``scripts/gdn_solve_oc_check.py:28-29``: value = (code - zp) * scale).
"""
from __future__ import annotations

import numpy as np

OC_GATE = 1.05e-2
BL = 16


def _bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 -> bfloat16 (nearest-even), returned as float32 holding bf16 values."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def make_chunk_A(n_chunks: int, C: int = 256, dk: int = 128, seed: int = 0x6D6E,
                 as_bf16: bool = True) -> np.ndarray:
    """[n_chunks, C, C] strictly-lower A for independent (batch, head, chunk) units (float32 array
    holding bf16-representable values when ``as_bf16``)."""
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((n_chunks, C, dk)).astype(np.float32)
    k /= np.sqrt((k.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6).astype(np.float32)
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal((n_chunks, C))))
    z = 0.5 * rng.standard_normal((n_chunks, C)) - 2.0
    logsig = -np.logaddexp(0.0, -z)
    g = np.cumsum(logsig, axis=-1)
    kk = np.einsum("ncd,nkd->nck", k.astype(np.float64), k.astype(np.float64))
    diff = g[:, :, None] - g[:, None, :]
    tril = np.tril(np.ones((C, C), bool), -1)
    decay = np.exp(np.where(tril, diff, -np.inf))
    A = -(beta[:, :, None] * kk * decay)
    A = np.where(tril, A, 0.0).astype(np.float32)
    return _bf16_round(A) if as_bf16 else A


def chunk_A_from_kbg(k: np.ndarray, beta: np.ndarray, g_tok: np.ndarray) -> np.ndarray:
    """fp64 strictly-lower A of each chunk from the gated-delta-rule inputs, restating the Stage-A
    prefix of ``gdn_chunk`` (``scripts/gdn_ref_kernel.py:66-82``): k L2-normalised over Dk (eps 1e-6,
    :31-32), k_beta = k * beta, g = cumsum of the per-token log gates over the chunk (:72), decay =
    exp(g_i - g_j) on and below the diagonal, attn = -(k_beta k^T) * decay with the diagonal and the
    upper triangle zeroed (:75-77).  A = attn, so that T = (I - A)^-1 (the reference's forward
    substitution and ``+ eye`` at :78-81).  k [n, C, Dk]; beta, g_tok [n, C]."""
    k = np.asarray(k, np.float64)
    k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    kb = k * np.asarray(beta, np.float64)[..., None]
    g = np.cumsum(np.asarray(g_tok, np.float64), axis=-1)
    C = k.shape[-2]
    strict = np.tril(np.ones((C, C), bool), -1)
    diff = np.where(strict, g[..., :, None] - g[..., None, :], -np.inf)
    return np.where(strict, -np.einsum("ncd,nkd->nck", kb, k) * np.exp(diff), 0.0)


def make_kbg(n_chunks: int, C: int = 256, dk: int = 128, seed: int = 0x6D6F):
    """Synthetic gated-delta-rule chunk inputs of the BASELINE GDN config: raw k ~ N(0,1) rounded to
    bf16 [n, C, Dk], beta = sigmoid(N(0,1)) [n, C], per-token log gates logsigmoid(0.5 N(0,1) - 2)
    [n, C] (f32)."""
    rng = np.random.default_rng(seed)
    k = _bf16_round(rng.standard_normal((n_chunks, C, dk)).astype(np.float32))
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((n_chunks, C))))).astype(np.float32)
    z = 0.5 * rng.standard_normal((n_chunks, C)) - 2.0
    g_tok = (-np.logaddexp(0.0, -z)).astype(np.float32)
    return k, beta, g_tok


def inverse_fp64(A: np.ndarray) -> np.ndarray:
    """fp64 (I - A)^-1 per chunk by forward substitution on a unit lower-triangular system."""
    A = np.asarray(A, np.float64)
    n, C, _ = A.shape
    T = np.zeros_like(A)
    eye = np.eye(C)
    # row i: T[i,:] = e_i + A[i,:i] @ T[:i,:]
    for i in range(C):
        T[:, i, :] = eye[i] + np.einsum("nk,nkc->nc", A[:, i, :i], T[:, :i, :])
    return T


def oc(T: np.ndarray, Tref: np.ndarray) -> float:
    """Frobenius relative error over all chunks jointly (gdn_solve_oc_check.py:31)."""
    T = np.asarray(T, np.float64)
    Tref = np.asarray(Tref, np.float64)
    return float(np.linalg.norm(T - Tref) / (np.linalg.norm(Tref) + 1e-12))


def _clip16(v: np.ndarray) -> np.ndarray:
    return np.clip(np.round(v), -32767, 32767).astype(np.int16)   # llround: half away from zero


def block_model(Aq: np.ndarray, sA: float, sT: float) -> np.ndarray:
    """Reference BL=16 algorithm on int16 codes of A (gdn_solve_ref.c:19-69): per-block forward
    substitution with int32 accumulation and int16 requant at sT, then the fp64 block merge
    T_ij = T_ii @ sum_{k=j}^{i-1} A_ik T_kj.  Returns fp64 T [n, C, C]."""
    Aq = np.asarray(Aq, np.int16)
    n, C, _ = Aq.shape
    nb = C // BL
    Af = Aq.astype(np.float64) * sA
    Tblk = {}
    for b in range(nb):
        s = slice(b * BL, (b + 1) * BL)
        Ab = Aq[:, s, s].astype(np.int64)
        Tb = np.zeros((n, BL, BL), np.int64)
        for i in range(BL):
            acc = np.einsum("nk,nkj->nj", Ab[:, i, :i], Tb[:, :i, :]) if i else np.zeros((n, BL), np.int64)
            acc = acc.astype(np.int32).astype(np.float64)
            ei = np.where(np.arange(BL) == i, 1.0 / sT, 0.0)
            # llround(ei + acc*sA): round half away from zero
            v = ei[None, :] + acc * sA
            Tb[:, i, :] = np.clip(np.sign(v) * np.floor(np.abs(v) + 0.5), -32767, 32767).astype(np.int64)
        Tblk[(b, b)] = Tb.astype(np.float64) * sT
    for i in range(nb):
        for j in range(i - 1, -1, -1):
            acc = np.zeros((n, BL, BL))
            for k in range(j, i):
                acc += Af[:, i * BL:(i + 1) * BL, k * BL:(k + 1) * BL] @ Tblk[(k, j)]
            Tblk[(i, j)] = Tblk[(i, i)] @ acc
    T = np.zeros((n, C, C))
    for (i, j), blk in Tblk.items():
        T[:, i * BL:(i + 1) * BL, j * BL:(j + 1) * BL] = blk
    return T


def to_codes(v: np.ndarray, scale: float, zp: int) -> np.ndarray:
    """float -> u16 code = clip(rint(v/scale) + zp, 0, 65535)."""
    return np.clip(np.rint(np.asarray(v, np.float64) / scale) + zp, 0, 65535).astype(np.uint16)


def from_codes(c: np.ndarray, scale: float, zp: int) -> np.ndarray:
    return (np.asarray(c).astype(np.int64) - zp) * scale
