"""CPU oracle for the screened density-fitted Coulomb (RI-J) path and the screened nuclear
attraction on the same pair list — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it. The product path
(``gs_dft_b200``) runs the CUDA kernels and fails loudly when they are missing.

It is a NumPy FP64 restatement of the reference (andresguzco/gs-dft) algorithm. Each function cites
the reference file:line it follows. Parity pin: the restatement is checked against golden vectors
produced by executing the reference's own source files under a NumPy stand-in for the JAX API
(``tests/golden/make_golden.py``); the gradient, which the reference obtains by JAX autodiff, is
checked against central finite differences of that executed reference energy and, for the node
reverse pass, against the reference's hand-written ``nodes_bwd`` (gs_dft/coulomb/ri.py:190-222).

Third-party arithmetic: the reference takes Boys F0 from ``dftax.energy.boys`` (dftax 0.8.0, not
in the reference tree; used only in the aux metric, gs_dft/coulomb/ri.py:35,72-74). Here
F0(T) = 1/2 sqrt(pi/T) erf(sqrt(T)) with its Taylor series at small T, the closed form the
reference's own tests use (tests/unit/test_coulomb_stream.py:115-134). The metric V is therefore
pinned to that closed form, not to dftax's table.

One deliberate, documented deviation: the pair overlap used for screening is evaluated once per
unordered pair, in the orientation (min(i,j), max(i,j)), and shared by (i,j) and (j,i). The
reference evaluates both orientations; they agree to the last bit or two. This keeps the ordered
list exactly symmetric and makes the overflow ranking's tie order well defined.
"""
from __future__ import annotations

import math

import numpy as np
from scipy.special import erf

PI = math.pi

# ----------------------------------------------------------------------------------------------
#  Laplace half-line node table  (gs_dft/integrals/dense.py:46-53, 77-82)
# ----------------------------------------------------------------------------------------------


def gauss_legendre_halfline(n_quad: int = 20):
    """t = s/(1-s) map of Gauss-Legendre on [0,1) (gs_dft/integrals/dense.py:46-53)."""
    x, w = np.polynomial.legendre.leggauss(n_quad)
    s = (x + 1.0) / 2.0
    w_s = w / 2.0
    t = s / (1.0 - s)
    jac = 1.0 / (1.0 - s) ** 2
    return np.asarray(t, np.float64), np.asarray(w_s * jac, np.float64)


QUAD_T, QUAD_W = gauss_legendre_halfline(20)


def gauss_legendre_segment(upper: float, n_quad: int = 12):
    """Gauss-Legendre on [0, upper]: the node table of the erf(omega r)/r kernel, the same node
    integral taken to omega instead of infinity (gs_dft/integrals/dense.py:56-76)."""
    x, w = np.polynomial.legendre.leggauss(n_quad)
    return 0.5 * float(upper) * (x + 1.0), 0.5 * float(upper) * w


def _node_table(omega):
    """(t, w) of the 3-centre kernel: the half-line rule, or the 12-node segment rule on
    [0, omega] for the long-range kernel (gs_dft/coulomb/ri.py:149,232-235)."""
    return (QUAD_T, QUAD_W) if not omega else gauss_legendre_segment(omega, 12)

# ----------------------------------------------------------------------------------------------
#  Splat chart  (gs_dft/basis/spectral.py:33-40, 71-82)
# ----------------------------------------------------------------------------------------------


def quat_to_rotation(q):
    """gs_dft/basis/spectral.py:33-40 — normalise with +1e-12, then the Hamilton matrix."""
    n = np.sqrt(np.sum(q * q, axis=-1, keepdims=True))
    q = q / (n + 1e-12)
    w, x, y, z = q[..., 0], q[..., 1], q[..., 2], q[..., 3]
    r0 = np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1)
    r1 = np.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1)
    r2 = np.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1)
    return np.stack([r0, r1, r2], -2)


def splat_A(quat, log_scale):
    """A = R diag(exp l) R^T (gs_dft/basis/spectral.py:71-76); entry (i,k) summed j = 0,1,2."""
    R = quat_to_rotation(quat)
    a = np.exp(log_scale)
    A = np.empty(R.shape)
    for i in range(3):
        for k in range(3):
            A[:, i, k] = ((R[:, i, 0] * a[:, 0]) * R[:, k, 0] + (R[:, i, 1] * a[:, 1]) * R[:, k, 1]
                          + (R[:, i, 2] * a[:, 2]) * R[:, k, 2])
    return A


def splat_norm(log_scale):
    """N = (8 det A / pi^3)^(1/4), det A = exp(sum l) (gs_dft/basis/spectral.py:78-82)."""
    detA = np.exp(np.sum(log_scale, axis=-1))
    return (8.0 * detA / PI ** 3) ** 0.25


def full_quantities(quat, log_scale, centers):
    """(A, mu, N) once per call (gs_dft/coulomb/stream.py:79-81)."""
    return splat_A(quat, log_scale), np.asarray(centers, np.float64), splat_norm(log_scale)

# ----------------------------------------------------------------------------------------------
#  Closed-form 3x3 algebra  (gs_dft/integrals/linalg3.py:17-51)
# ----------------------------------------------------------------------------------------------


def det3(A):
    """Cofactor expansion along the first row (gs_dft/integrals/linalg3.py:17-23)."""
    return (A[..., 0, 0] * (A[..., 1, 1] * A[..., 2, 2] - A[..., 1, 2] * A[..., 2, 1])
            - A[..., 0, 1] * (A[..., 1, 0] * A[..., 2, 2] - A[..., 1, 2] * A[..., 2, 0])
            + A[..., 0, 2] * (A[..., 1, 0] * A[..., 2, 1] - A[..., 1, 1] * A[..., 2, 0]))


def adj3(A):
    """Adjugate (gs_dft/integrals/linalg3.py:26-41)."""
    c00 = A[..., 1, 1] * A[..., 2, 2] - A[..., 1, 2] * A[..., 2, 1]
    c01 = A[..., 0, 2] * A[..., 2, 1] - A[..., 0, 1] * A[..., 2, 2]
    c02 = A[..., 0, 1] * A[..., 1, 2] - A[..., 0, 2] * A[..., 1, 1]
    c10 = A[..., 1, 2] * A[..., 2, 0] - A[..., 1, 0] * A[..., 2, 2]
    c11 = A[..., 0, 0] * A[..., 2, 2] - A[..., 0, 2] * A[..., 2, 0]
    c12 = A[..., 0, 2] * A[..., 1, 0] - A[..., 0, 0] * A[..., 1, 2]
    c20 = A[..., 1, 0] * A[..., 2, 1] - A[..., 1, 1] * A[..., 2, 0]
    c21 = A[..., 0, 1] * A[..., 2, 0] - A[..., 0, 0] * A[..., 2, 1]
    c22 = A[..., 0, 0] * A[..., 1, 1] - A[..., 0, 1] * A[..., 1, 0]
    return np.stack([np.stack([c00, c01, c02], -1), np.stack([c10, c11, c12], -1),
                     np.stack([c20, c21, c22], -1)], -2)


def matvec3(A, b):
    """sum_l A[k,l] b[l], l summed left to right."""
    return np.stack([A[..., k, 0] * b[..., 0] + A[..., k, 1] * b[..., 1] + A[..., k, 2] * b[..., 2]
                     for k in range(3)], -1)


def solve3(A, b):
    """adj(A) b / det(A) (gs_dft/integrals/linalg3.py:49-51)."""
    return matvec3(adj3(A), b) / det3(A)[..., None]

# ----------------------------------------------------------------------------------------------
#  Pair quantities and overlap  (gs_dft/coulomb/stream.py:203-215; gs_dft/screening/pairs.py:342-345)
# ----------------------------------------------------------------------------------------------


def full_pair_quantities(q, pi, pj):
    """A_hat = A_i + A_j, P = A_hat^-1 (A_i mu_i + A_j mu_j), KN = N_i N_j exp(-d.A_i A_hat^-1 A_j d)
    (gs_dft/coulomb/stream.py:203-215)."""
    A, mu, N = q
    Ai, Aj = A[pi], A[pj]
    mui, muj = mu[pi], mu[pj]
    Aij = Ai + Aj
    rhs = matvec3(Ai, mui) + matvec3(Aj, muj)
    Pa = solve3(Aij, rhs)
    d = mui - muj
    Ajd = matvec3(Aj, d)
    AiAinvAjd = matvec3(Ai, solve3(Aij, Ajd))
    K = np.exp(-(d[..., 0] * AiAinvAjd[..., 0] + d[..., 1] * AiAinvAjd[..., 1]
                 + d[..., 2] * AiAinvAjd[..., 2]))
    return Aij, Pa, N[pi] * N[pj] * K


def overlap_pairs(q, pi, pj):
    """S_ij = KN pi^1.5 / sqrt(det A_hat) (gs_dft/screening/pairs.py:342-345)."""
    Aij, _, NK = full_pair_quantities(q, pi, pj)
    return NK * PI ** 1.5 / np.sqrt(det3(Aij))


def canonical_abs_overlap(q, pi, pj):
    """|S| evaluated in the (min, max) orientation, shared by (i,j) and (j,i)."""
    lo = np.minimum(pi, pj)
    hi = np.maximum(pi, pj)
    return np.abs(overlap_pairs(q, lo, hi))

# ----------------------------------------------------------------------------------------------
#  Significant-pair list  (gs_dft/screening/pairs.py:50-164, 225-322)
# ----------------------------------------------------------------------------------------------


def pair_weights(pi, pj, unique):
    """bool mask, or (2 - delta_ij) weights when unique (gs_dft/screening/pairs.py:318-322)."""
    if not unique:
        return np.ones(pi.shape[0], bool)
    return np.where(pi == pj, 1.0, 2.0)


def _significant_flat(q, M, eps, unique, row_chunk=256):
    """Ascending flat indices i*M+j with |S_ij| > eps, plus their |S| (pairs.py:50-87,103-118)."""
    flats, vals = [], []
    for a in range(0, M, row_chunk):
        rows = np.arange(a, min(a + row_chunk, M))
        pi = np.repeat(rows, M)
        pj = np.tile(np.arange(M), rows.size)
        s = canonical_abs_overlap(q, pi, pj)
        sig = s > eps
        if unique:
            sig &= pj >= pi
        flats.append(pi[sig].astype(np.int64) * M + pj[sig])
        vals.append(s[sig])
    return np.concatenate(flats), np.concatenate(vals)


def count_significant(q, M, eps, unique):
    """_count_significant (gs_dft/screening/pairs.py:103-118)."""
    return int(_significant_flat(q, M, eps, unique)[0].size)


def _decode(flat, M, pad_to, unique):
    """_decode_flat (gs_dft/screening/pairs.py:90-100): tail-padded with (0,0), weight 0."""
    pi = (flat // M).astype(np.int32)
    pj = (flat % M).astype(np.int32)
    valid = pair_weights(pi, pj, unique)
    k = pi.size
    if pad_to is not None and pad_to > k:
        z = np.zeros(pad_to - k, np.int32)
        pi = np.concatenate([pi, z])
        pj = np.concatenate([pj, z])
        valid = np.concatenate([valid, np.zeros(pad_to - k, valid.dtype)])
    return pi, pj, valid


def neighbor_pairs(q, eps=1e-5, pad_to=None, unique=False, headroom=2):
    """Significant ordered pairs, lexsorted, tail-padded; overflow keeps the ``pad_to`` largest |S|
    (ties by ascending flat index), re-lexsorted (gs_dft/screening/pairs.py:225-315, 155-164).
    Returns (pi, pj, valid, n_sig)."""
    M = int(q[1].shape[0])
    n_all = M * (M + 1) // 2 if unique else M * M
    if eps < 0.0 and (pad_to is None or pad_to >= n_all):
        if unique:
            pi, pj = np.triu_indices(M)
        else:
            pi = np.repeat(np.arange(M), M)
            pj = np.tile(np.arange(M), M)
        flat = pi.astype(np.int64) * M + pj
        out = _decode(flat, M, pad_to, unique)
        return (*out, n_all)
    flat, vals = _significant_flat(q, M, eps, unique)
    n_sig = int(flat.size)
    if pad_to is None:
        return (*_decode(flat, M, None, unique), n_sig)
    if n_sig <= pad_to:
        return (*_decode(flat, M, pad_to, unique), n_sig)
    if n_sig > headroom * pad_to:
        raise ValueError(f"neighbor_pairs: {n_sig} significant pairs exceed {headroom}x the pad")
    order = np.argsort(-vals, kind="stable")[:pad_to]
    keep = np.sort(flat[order])
    return (*_decode(keep, M, pad_to, unique), n_sig)


def pad_rule(n0, pad, G):
    """pad_to = ceil(pad * n0 / G) * G  (gs_dft/ks/train.py:356-359)."""
    return -(-int(pad * n0) // G) * G


def stripe_pairs(pi, pj, valid, G):
    """Round-robin deal so every device block has the same valid:dummy ratio
    (gs_dft/ks/shard.py:146-166)."""
    n = pi.shape[0]
    if G <= 1 or n % G:
        return pi, pj, valid
    f = lambda a: a.reshape(-1, G).T.reshape(-1)
    return f(pi), f(pj), f(valid)

# ----------------------------------------------------------------------------------------------
#  Product auxiliary basis  (gs_dft/basis/isotropic.py:22-39, 81-116; gs_dft/coulomb/ri.py:238-240)
# ----------------------------------------------------------------------------------------------


def init_product_aux(q, scales=(1.0,), diagonal_only=True, pi=None, pj=None, valid=None):
    """Frozen product aux: per kept pair, alpha0 = det(A_hat)^(1/3), centre = product centre;
    log_alpha = log(alpha0*s) per scale (gs_dft/basis/isotropic.py:81-116). Returns (log_alpha, R)."""
    M = q[1].shape[0]
    if diagonal_only or pi is None:
        pi = pj = np.arange(M)
        valid = None
    Aij, Pa, _ = full_pair_quantities(q, pi, pj)
    alpha0 = det3(Aij) ** (1.0 / 3.0)
    if valid is not None:
        alpha0 = np.where(valid, alpha0, 1.0)
    log_alpha = np.concatenate([np.log(alpha0 * float(s)) for s in scales])
    R = np.concatenate([Pa for _ in scales], axis=0)
    return log_alpha, R


def aux_quantities(log_alpha, R):
    """(beta, R, norm): alpha = exp(log_alpha), norm = (2 alpha/pi)^(3/4)
    (gs_dft/basis/isotropic.py:30-39; gs_dft/coulomb/ri.py:238-240)."""
    alpha = np.exp(log_alpha)
    return alpha, R, (2.0 * alpha / PI) ** 0.75

# ----------------------------------------------------------------------------------------------
#  Aux metric, factor, solve  (gs_dft/coulomb/ri.py:63-123, 243-275, 472-482)
# ----------------------------------------------------------------------------------------------


def boys0(T):
    """F0(T) = 1/2 sqrt(pi/T) erf(sqrt T); Taylor 1 - T/3 + T^2/10 - T^3/42 below 1e-8."""
    T = np.asarray(T, np.float64)
    small = T < 1e-8
    Ts = np.where(small, 1.0, T)
    big = 0.5 * np.sqrt(PI / Ts) * erf(np.sqrt(Ts))
    ser = 1.0 - T / 3.0 + T * T / 10.0 - T * T * T / 42.0
    return np.where(small, ser, big)


def coulomb_block(g1, P1, KN1, g2, P2, KN2, omega=None):
    """(1|2) = KN1 KN2 2 pi^2.5/(g1 g2 sqrt(g1+g2)) F0(g1g2/(g1+g2) |P1-P2|^2); with ``omega`` the
    long-range erf(omega r)/r kernel, F0(T) -> sqrt(z) F0(z T), z = omega^2/(omega^2 + rho)
    (gs_dft/coulomb/ri.py:63-76)."""
    gab = g1[:, None] * g2[None, :]
    gsum = g1[:, None] + g2[None, :]
    dx = P1[:, None, :] - P2[None, :, :]
    PQ2 = dx[..., 0] ** 2 + dx[..., 1] ** 2 + dx[..., 2] ** 2
    rho = gab / gsum
    T = rho * PQ2
    if omega:
        z = omega ** 2 / (omega ** 2 + rho)
        F0 = np.sqrt(z) * boys0(z * T)
    else:
        F0 = boys0(T)
    coul = 2.0 * PI ** 2.5 / (gab * np.sqrt(gsum)) * F0
    return (KN1[:, None] * KN2[None, :]) * coul


def aux_metric(beta, R, KN, omega=None):
    """V_PQ = (P|Q), or the long-range (P|erf(omega r)/r|Q) (gs_dft/coulomb/ri.py:267-275)."""
    return coulomb_block(beta, R, KN, beta, R, KN, omega)


def aux_cholesky(V, lam):
    """Lower Cholesky of V + lam I (gs_dft/coulomb/ri.py:243-264)."""
    Vs = V.copy()
    Vs[np.diag_indices_from(Vs)] += lam
    return np.linalg.cholesky(Vs)


def df_coulomb_solve(gamma, L):
    """d = cho_solve((L, lower), gamma); E_J = 1/2 gamma.d (gs_dft/coulomb/ri.py:472-482)."""
    from scipy.linalg import cho_solve
    d = cho_solve((L, True), gamma)
    return 0.5 * float(np.dot(gamma, d)), d

# ----------------------------------------------------------------------------------------------
#  3-centre (aux | pair) block  (gs_dft/coulomb/ri.py:126-185)
# ----------------------------------------------------------------------------------------------

PREF = 2.0 * PI ** 3 / math.sqrt(PI)


def isobra_nodes(beta, dp2, Lam, nodes=None):
    """sum_t w_t (G0G1G2)^-1/2 exp(-t^2 sum_k W_k/G_k) in the division-lean form
    (gs_dft/coulomb/ri.py:167-185). beta (A,), dp2 (A,B,3), Lam (B,3) -> (A,B). ``nodes`` = (t, w)
    (default the half-line rule)."""
    b = beta[:, None]
    L0, L1, L2 = Lam[None, :, 0], Lam[None, :, 1], Lam[None, :, 2]
    coul = np.zeros((beta.shape[0], Lam.shape[0]))
    for t, w in zip(*(nodes or (QUAD_T, QUAD_W))):
        t2 = t * t
        G0 = b * L0 + t2 * (b + L0)
        G1 = b * L1 + t2 * (b + L1)
        G2 = b * L2 + t2 * (b + L2)
        invp = 1.0 / (G0 * G1 * G2)
        num = b * (L0 * dp2[..., 0] * G1 * G2 + L1 * dp2[..., 1] * G0 * G2
                   + L2 * dp2[..., 2] * G0 * G1)
        coul = coul + w * np.sqrt(invp) * np.exp(-t2 * num * invp)
    return coul


def isobra_nodes_bwd(beta, dp2, Lam, gI):
    """The reference's analytic reverse of the node sum (gs_dft/coulomb/ri.py:190-222):
    returns (d_beta, d_dp2 (A,B,3), d_Lam (B,3))."""
    b = beta[:, None]
    Ls = (Lam[None, :, 0], Lam[None, :, 1], Lam[None, :, 2])
    d_beta = np.zeros_like(b)
    d_Lam = [np.zeros((1, Lam.shape[0])) for _ in range(3)]
    d_dp2 = [np.zeros((beta.shape[0], Lam.shape[0])) for _ in range(3)]
    for t, w in zip(QUAD_T, QUAD_W):
        t2 = t * t
        G = [b * L + t2 * (b + L) for L in Ls]
        invG = [1.0 / Gk for Gk in G]
        W = [b * L * dp2[..., k] for k, L in enumerate(Ls)]
        S = W[0] * invG[0] + W[1] * invG[1] + W[2] * invG[2]
        I = w * np.sqrt(invG[0] * invG[1] * invG[2]) * np.exp(-t2 * S)
        gIt = gI * I
        db = np.zeros_like(gIt)
        for k, L in enumerate(Ls):
            dIdG = gIt * (t2 * W[k] * invG[k] - 0.5) * invG[k]
            dIdW = -gIt * t2 * invG[k]
            db = db + dIdG * (L + t2) + dIdW * L * dp2[..., k]
            d_Lam[k] = d_Lam[k] + np.sum(dIdG * (b + t2) + dIdW * b * dp2[..., k], axis=0,
                                         keepdims=True)
            d_dp2[k] = d_dp2[k] + dIdW * b * L
        d_beta = d_beta + np.sum(db, axis=1, keepdims=True)
    return d_beta[:, 0], np.stack(d_dp2, -1), np.stack([dL[0] for dL in d_Lam], -1)


def full_isobra_block(beta, R, KN_aux, A_pair, P_pair, KN_pair, omega=None):
    """(P|a): eigh of A_hat, dp2 = (U^T (R - P))^2, node sum, prefactor
    (gs_dft/coulomb/ri.py:126-151); ``omega``: the long-range kernel's segment rule. Returns
    (N_aux, n_pair)."""
    Lam, U = np.linalg.eigh(A_pair)
    d = R[:, None, :] - P_pair[None, :, :]
    dp2 = np.einsum("bki,abk->abi", U, d) ** 2
    coul = isobra_nodes(beta, dp2, Lam, _node_table(omega))
    return (KN_aux[:, None] * KN_pair[None, :]) * PREF * coul

# ----------------------------------------------------------------------------------------------
#  Screened gamma stream and energy  (gs_dft/coulomb/ri.py:436-494)
# ----------------------------------------------------------------------------------------------


def pair_density(C_occ, occ, pi, pj, valid):
    """q_a = valid_a * sum_o occ_o C_io C_jo (gs_dft/coulomb/ri.py:456)."""
    return np.asarray(valid, np.float64) * np.sum(occ[None, :] * C_occ[pi] * C_occ[pj], axis=1)


def df_coulomb_gamma_screened(q_splat, C_occ, occ, aux_q, pi, pj, valid, chunk=2048):
    """gamma_P = sum_a (P|a) q_a over the pair list, chunked (gs_dft/coulomb/ri.py:436-469)."""
    beta, R, KN = aux_q
    gamma = np.zeros(beta.shape[0])
    for a in range(0, pi.shape[0], chunk):
        ci, cj, cv = pi[a:a + chunk], pj[a:a + chunk], valid[a:a + chunk]
        qa = pair_density(C_occ, occ, ci, cj, cv)
        blk = full_isobra_block(beta, R, KN, *full_pair_quantities(q_splat, ci, cj))
        gamma = gamma + blk @ qa
    return gamma


def energy(sys_arrays, aux_q, L, pi, pj, valid, chunk=2048):
    """E_J^DF = 1/2 gamma^T (V + lam I)^-1 gamma (gs_dft/coulomb/ri.py:485-494).
    ``sys_arrays`` = (quat, log_scale, centers, C_occ, occ). Returns (E, gamma, d)."""
    quat, log_scale, centers, C_occ, occ = sys_arrays
    q = full_quantities(quat, log_scale, centers)
    gamma = df_coulomb_gamma_screened(q, C_occ, occ, aux_q, pi, pj, valid, chunk)
    E, d = df_coulomb_solve(gamma, L)
    return E, gamma, d

# ----------------------------------------------------------------------------------------------
#  Analytic gradient (the reference obtains it by JAX autodiff through ri.py:126-185,
#  stream.py:203-215 and spectral.py:33-82, with the node reverse of ri.py:190-222).
# ----------------------------------------------------------------------------------------------


def _pair_vjp_integral(beta, R, KN_aux, dvec, A_pair, P_pair, KN_pair, qa, W=None, omega=None):
    """For each pair: J_a = sum_P (P|a) d_P and the cotangents of (A_hat, P_a, KN_a) of
    E = sum_P d_P sum_a (P|a) q_a, without the 1/(lambda_i - lambda_j) terms of an eigh VJP.
    With ``W`` (N_aux, B) the cotangents are those of E = sum_{P,a} W[P,a] (P|a) instead
    (dvec and qa unused; J returned as zeros).

    Per node, f = w det(G)^-1/2 exp(-t^2 beta d^T A_hat G^-1 d) with G = (beta+t^2) A_hat + t^2 beta I:
      df/dA_hat = f (-1/2 (beta+t^2) G^-1 - t^4 beta^2 z z^T),  z = G^-1 d
      df/dP     = f 2 t^2 beta A_hat z.
    Evaluated in the eigenframe of A_hat (G and A_hat commute)."""
    Lam, U = np.linalg.eigh(A_pair)                           # (B,3), (B,3,3)
    dd = R[:, None, :] - P_pair[None, :, :]                   # (A,B,3)
    y = np.einsum("bki,abk->abi", U, dd)                      # eigenframe displacement
    b = beta[:, None]
    coul = np.zeros(y.shape[:2])
    Dk = np.zeros(y.shape)                                    # sum_t f s / G_k
    Zkl = np.zeros(y.shape + (3,))                            # sum_t f t^4 beta^2 z_k z_l
    Vk = np.zeros(y.shape)                                    # sum_t f t^2 beta lam_k z_k
    for t, w in zip(*_node_table(omega)):
        t2 = t * t
        s = b + t2
        G = b[..., None] * Lam[None] + t2 * (b[..., None] + Lam[None])   # (A,B,3)
        invG = 1.0 / G
        S = np.sum(b[..., None] * Lam[None] * y * y * invG, axis=-1)
        f = w * np.sqrt(invG[..., 0] * invG[..., 1] * invG[..., 2]) * np.exp(-t2 * S)
        coul += f
        z = y * invG
        Dk += (f * s)[..., None] * invG
        Zkl += (f * t2 * t2 * b * b)[..., None, None] * z[..., :, None] * z[..., None, :]
        Vk += (f * t2 * b)[..., None] * Lam[None] * z
    if W is not None:
        cq = W * KN_aux[:, None] * (KN_pair * PREF)[None, :]          # W_Pa KN_P KN_a pref
        J = np.zeros(KN_pair.shape[0])
        KNbar = np.sum(W * KN_aux[:, None] * PREF * coul, axis=0)
    else:
        c = dvec[:, None] * KN_aux[:, None] * (KN_pair * PREF)[None, :]   # d_P KN_P KN_a pref
        J = np.sum(c * coul, axis=0)
        cq = c * qa[None, :]
        KNbar = qa * np.sum(dvec[:, None] * KN_aux[:, None] * PREF * coul, axis=0)
    Mk = -0.5 * np.sum(cq[..., None] * Dk, axis=0)                     # (B,3) diagonal part
    Mkl = -np.sum(cq[..., None, None] * Zkl, axis=0)                   # (B,3,3)
    Mkl[:, [0, 1, 2], [0, 1, 2]] += Mk
    Abar = np.einsum("bik,bkl,bjl->bij", U, Mkl, U)
    Pbar_eig = 2.0 * np.sum(cq[..., None] * Vk, axis=0)                # (B,3) eigenframe
    Pbar = np.einsum("bik,bk->bi", U, Pbar_eig)
    return J, Abar, Pbar, KNbar


def _pair_chain(q_splat, pi, pj, Abar_h, Pbar, KNbar):
    """Cotangents of (A_hat, P, KN) -> (A_i, A_j, mu_i, mu_j, N_i, N_j)
    (the reverse of gs_dft/coulomb/stream.py:203-215)."""
    A, mu, N = q_splat
    Ai, Aj, mui, muj = A[pi], A[pj], mu[pi], mu[pj]
    Ah = Ai + Aj
    Ahinv = np.linalg.inv(Ah)
    b = np.einsum("pkl,pl->pk", Ai, mui) + np.einsum("pkl,pl->pk", Aj, muj)
    P = np.einsum("pkl,pl->pk", Ahinv, b)
    v = np.einsum("pkl,pl->pk", Ahinv, Pbar)
    Ah_bar = Abar_h - v[:, :, None] * P[:, None, :]
    gAi = Ah_bar + v[:, :, None] * mui[:, None, :]
    gAj = Ah_bar + v[:, :, None] * muj[:, None, :]
    gmui = np.einsum("plk,pl->pk", Ai, v)
    gmuj = np.einsum("plk,pl->pk", Aj, v)
    d = mui - muj
    e = np.einsum("pkl,pl->pk", Ahinv, np.einsum("pkl,pl->pk", Aj, d))
    f = d - e
    Hd = np.einsum("pkl,pl->pk", Ai, e)                       # A_i A_hat^-1 A_j d
    K = np.exp(-np.sum(d * Hd, axis=-1))
    KN = N[pi] * N[pj] * K
    gNi = KNbar * N[pj] * K
    gNj = KNbar * N[pi] * K
    Qbar = -KNbar * KN
    gd = (2.0 * Qbar)[:, None] * Hd
    gmui = gmui + gd
    gmuj = gmuj - gd
    gAi = gAi + Qbar[:, None, None] * e[:, :, None] * e[:, None, :]
    gAj = gAj + Qbar[:, None, None] * f[:, :, None] * f[:, None, :]
    return gAi, gAj, gmui, gmuj, gNi, gNj


def chart_vjp(quat, log_scale, gA, gN):
    """Reverse of the chart A = R(q) diag(e^l) R^T, N = (8 e^(sum l)/pi^3)^(1/4)
    (gs_dft/basis/spectral.py:33-40, 71-82). gA may be non-symmetric; only its symmetric part acts."""
    gS = 0.5 * (gA + np.swapaxes(gA, -1, -2))
    R = quat_to_rotation(quat)
    a = np.exp(log_scale)
    N = splat_norm(log_scale)
    RtgR = np.einsum("mik,mij,mjl->mkl", R, gS, R)
    g_log = a * np.stack([RtgR[:, k, k] for k in range(3)], -1) + (gN * N / 4.0)[:, None]
    gR = 2.0 * np.einsum("mij,mjk->mik", gS, R) * a[:, None, :]
    n = np.sqrt(np.sum(quat * quat, axis=-1))
    qh = quat / (n + 1e-12)[:, None]
    w, x, y, z = qh[:, 0], qh[:, 1], qh[:, 2], qh[:, 3]
    g = gR
    gw = 2 * (-z * g[:, 0, 1] + y * g[:, 0, 2] + z * g[:, 1, 0] - x * g[:, 1, 2]
              - y * g[:, 2, 0] + x * g[:, 2, 1])
    gx = 2 * (y * g[:, 0, 1] + z * g[:, 0, 2] + y * g[:, 1, 0] - 2 * x * g[:, 1, 1]
              - w * g[:, 1, 2] + z * g[:, 2, 0] + w * g[:, 2, 1] - 2 * x * g[:, 2, 2])
    gy = 2 * (-2 * y * g[:, 0, 0] + x * g[:, 0, 1] + w * g[:, 0, 2] + x * g[:, 1, 0]
              + z * g[:, 1, 2] - w * g[:, 2, 0] + z * g[:, 2, 1] - 2 * y * g[:, 2, 2])
    gz = 2 * (-2 * z * g[:, 0, 0] - w * g[:, 0, 1] + x * g[:, 0, 2] + w * g[:, 1, 0]
              - 2 * z * g[:, 1, 1] + y * g[:, 1, 2] + x * g[:, 2, 0] + y * g[:, 2, 1])
    gqh = np.stack([gw, gx, gy, gz], -1)
    dot = np.sum(quat * gqh, axis=-1)
    g_quat = gqh / (n + 1e-12)[:, None] - quat * (dot / (np.maximum(n, 1e-300) * (n + 1e-12) ** 2))[:, None]
    return g_quat, g_log


def energy_and_grad(sys_arrays, aux_q, L, pi, pj, valid, chunk=1024):
    """E_J, gamma, d, J (per listed pair; 0 on zero-weight entries) and the gradient of E_J with
    respect to (quat, log_scale, centers, C_occ), aux and pair list frozen."""
    quat, log_scale, centers, C_occ, occ = sys_arrays
    qs = full_quantities(quat, log_scale, centers)
    E, gamma, dvec = energy(sys_arrays, aux_q, L, pi, pj, valid, chunk)
    beta, R, KN_aux = aux_q
    M = centers.shape[0]
    n = pi.shape[0]
    J = np.zeros(n)
    gA = np.zeros((M, 3, 3))
    gmu = np.zeros((M, 3))
    gN = np.zeros(M)
    gC = np.zeros_like(C_occ)
    w = np.asarray(valid, np.float64)
    for a in range(0, n, chunk):
        sl = slice(a, a + chunk)
        ci, cj, cw = pi[sl], pj[sl], w[sl]
        live = cw != 0
        if not np.any(live):
            continue
        ci, cj, cw = ci[live], cj[live], cw[live]
        qa = pair_density(C_occ, occ, ci, cj, cw)
        Ah, Pa, KNa = full_pair_quantities(qs, ci, cj)
        Jc, Abar, Pbar, KNbar = _pair_vjp_integral(beta, R, KN_aux, dvec, Ah, Pa, KNa, qa)
        J[np.arange(a, min(a + chunk, n))[live]] = Jc
        _scatter_pair_grads(qs, ci, cj, cw, Jc, Abar, Pbar, KNbar, C_occ, occ, gA, gmu, gN, gC)
    g_quat, g_log = chart_vjp(quat, log_scale, gA, gN)
    return dict(E=E, gamma=gamma, d=dvec, J=J, g_quat=g_quat, g_log_scale=g_log,
                g_centers=gmu, g_C=gC, gA=gA, gmu=gmu, gN=gN)


def _scatter_pair_grads(qs, ci, cj, cw, Jc, Abar, Pbar, KNbar, C_occ, occ, gA, gmu, gN, gC):
    """Chain one chunk's pair cotangents to the splats (in place): (A_hat, P, KN) -> (A, mu, N) of
    both members, and dE/dq_a = Jc -> C_occ through q_a = w_a sum_o occ_o C_io C_jo."""
    gAi, gAj, gmui, gmuj, gNi, gNj = _pair_chain(qs, ci, cj, Abar, Pbar, KNbar)
    np.add.at(gA, ci, gAi)
    np.add.at(gA, cj, gAj)
    np.add.at(gmu, ci, gmui)
    np.add.at(gmu, cj, gmuj)
    np.add.at(gN, ci, gNi)
    np.add.at(gN, cj, gNj)
    s = (Jc * cw)[:, None] * occ[None, :]
    np.add.at(gC, ci, s * C_occ[cj])
    np.add.at(gC, cj, s * C_occ[ci])

# ----------------------------------------------------------------------------------------------
#  Screened exact (pair|pair) Coulomb  (gs_dft/coulomb/stream.py:249-320)
# ----------------------------------------------------------------------------------------------


def eri_block_schur(q_splat, bi, bj, ki, kj):
    """(a|b) for bra pairs (bi, bj) x ket pairs (ki, kj) through the Schur complement of the 6x6
    precision G = [[X, -t^2 I], [-t^2 I, Y]], X = A_a + t^2 I, Y = A_b + t^2 I, S = Y - t^4 X^-1:
    det G = det X det S, v^T G^-1 v = v_a.u + w.S^-1 w, u = X^-1 v_a, w = t^2 u + v_b
    (gs_dft/coulomb/stream.py:249-283)."""
    Aa, Pa, KNa = full_pair_quantities(q_splat, bi, bj)
    Ab, Pb, KNb = full_pair_quantities(q_splat, ki, kj)
    va = matvec3(Aa, Pa)
    vb = matvec3(Ab, Pb)
    cv = np.sum(Pa * va, -1)[:, None] + np.sum(Pb * vb, -1)[None, :]
    eye = np.eye(3)
    coul = np.zeros((Aa.shape[0], Ab.shape[0]))
    for t, wq in zip(QUAD_T, QUAD_W):
        t2 = t * t
        X = Aa + t2 * eye
        Xinv = adj3(X) / det3(X)[:, None, None]
        u = matvec3(Xinv, va)
        vau = np.sum(va * u, -1)
        Y = Ab + t2 * eye
        S = Y[None, :] - (t2 * t2) * Xinv[:, None]
        w = t2 * u[:, None, :] + vb[None, :, :]
        z = solve3(S, w)
        quad = cv - (vau[:, None] + np.sum(w * z, -1))
        detG = det3(X)[:, None] * det3(S)
        coul = coul + wq * (2.0 / math.sqrt(PI)) * (PI ** 3 / np.sqrt(detG) * np.exp(-quad))
    return (KNa[:, None] * KNb[None, :]) * coul


def boys_scaled_nodes(n=32):
    """The fused block's rule: Gauss-Legendre on u in [0,1), t^2 = rho c_k, c = u^2/(1-u^2),
    e = (w/2)(1-u^2)^-3/2 (gs_dft/coulomb/stream.py:341-347)."""
    x, w = np.polynomial.legendre.leggauss(n)
    u = (x + 1.0) / 2.0
    wu = w / 2.0
    return u * u / (1.0 - u * u), wu * (1.0 - u * u) ** -1.5


def eri_block_fused(q_splat, bi, bj, ki, kj, n_nodes=32):
    """(a|b) for bra pairs x ket pairs by the fused scalar kernel (gs_dft/coulomb/stream.py:406-458):
    C = A_a (A_a + A_b)^-1 A_b, its invariants I1, I2, I3, q2 = d.C d, q1 = I1 q2 - |C d|^2,
    q0 = I3 |d|^2, the per-(a, b) scale rho = I3^(1/3) / (1 + q2), and
    (a|b) = KN_a KN_b (2/sqrt(pi)) pi^3 sqrt(rho / det S) sum_k e_k exp(-s N(s)/D(s)) / sqrt(D(s)),
    s = rho c_k, D(s) = ((s + I1) s + I2) s + I3, N(s) = q0 + s (q1 + s q2)."""
    Aa, Pa, KNa = full_pair_quantities(q_splat, bi, bj)
    Ab, Pb, KNb = full_pair_quantities(q_splat, ki, kj)
    S = Aa[:, None] + Ab[None, :]
    detS = det3(S)
    C = np.einsum("akl,abln,bnm->abkm", Aa, adj3(S), Ab) / detS[..., None, None]
    C = 0.5 * (C + np.swapaxes(C, -1, -2))
    I1 = np.trace(C, axis1=-2, axis2=-1)
    I2 = (C[..., 0, 0] * C[..., 1, 1] + C[..., 1, 1] * C[..., 2, 2] + C[..., 2, 2] * C[..., 0, 0]
          - C[..., 0, 1] ** 2 - C[..., 0, 2] ** 2 - C[..., 1, 2] ** 2)
    I3 = (det3(Aa)[:, None] * det3(Ab)[None, :]) / detS
    d = Pa[:, None, :] - Pb[None, :, :]
    Cd = np.einsum("abkl,abl->abk", C, d)
    q2 = np.sum(d * Cd, -1)
    q1 = I1 * q2 - np.sum(Cd * Cd, -1)
    q0 = I3 * np.sum(d * d, -1)
    rho = np.cbrt(I3) / (1.0 + q2)
    acc = np.zeros_like(I1)
    for c, e in zip(*boys_scaled_nodes(n_nodes)):
        s = rho * c
        D = ((s + I1) * s + I2) * s + I3
        acc = acc + e * np.exp(-s * (q0 + s * (q1 + s * q2)) / D) / np.sqrt(D)
    pref = 2.0 * PI ** 3 / math.sqrt(PI)
    return (KNa[:, None] * KNb[None, :]) * pref * np.sqrt(rho / detS) * acc


def screened_coulomb_energy_exact(sys_arrays, pi, pj, valid, bra_chunk=128, block="schur"):
    """Exact E_J = 1/2 sum_{a,b} P_a P_b (a|b) over the listed pairs, P_a = valid_a sum_o occ_o
    C_io C_jo (gs_dft/coulomb/stream.py:294-320), with the Schur block (the reference's choice) or
    the fused 32-node block. Returns (E, Jvec) with Jvec_a = sum_b (a|b) P_b."""
    blk = eri_block_schur if block == "schur" else eri_block_fused
    quat, log_scale, centers, C, occ = sys_arrays
    q = full_quantities(quat, log_scale, centers)
    n = pi.shape[0]
    w = np.ones(n) if valid is None else np.asarray(valid, np.float64)
    Pw = w * np.sum(occ[None, :] * C[pi] * C[pj], axis=1)
    live = Pw != 0
    ki, kj, Pk = pi[live], pj[live], Pw[live]
    jv = np.zeros(n)
    for a in range(0, n, bra_chunk):
        sl = slice(a, a + bra_chunk)
        jv[sl] = blk(q, pi[sl], pj[sl], ki, kj) @ Pk
    return 0.5 * float(np.sum(jv * Pw)), jv

def screened_coulomb_exact_and_grad(sys_arrays, pi, pj, valid, bra_chunk=64, block="schur"):
    """Exact E_J (as ``screened_coulomb_energy_exact``), J per listed pair (0 on zero-weight
    entries) and the gradient of E_J with respect to (quat, log_scale, centers, C_occ), pair list
    frozen: the derivative the reference takes by autodiff of its streamed block
    (gs_dft/coulomb/stream.py:144-189, 294-320), written out. The 6x6 determinant of the Schur
    block is det A_a det A_b det(I + t^2 H) and its exponent t^2 d.(I + t^2 H)^-1 d, with
    H = A_a^-1 + A_b^-1 and d = P_a - P_b, so (a|b) = (2/sqrt(pi)) pi^3 g_a g_b F(H, d),
    g = KN det(A)^-1/2 and F = sum_t w_t det(I + t^2 H)^-1/2 exp(-t^2 d.K_t d), K_t = (I + t^2 H)^-1:
      dF/dH = sum_t f_t (-1/2 t^2 K_t + t^4 u_t u_t^T),  dF/dd = -2 sum_t f_t t^2 u_t,  u_t = K_t d.
    Each node's K_t is a direct 3x3 inverse here (no power expansion). ``block="fused"``: the
    32-node rule t^2 = rho c_k with F = sqrt(rho) sum_k e_k (...), rho = det(H)^-1/3/(1 + d.H^-1 d),
    which adds dF/drho (drho/dH, drho/dd), with d/ds of a node term f (-1/2 tr(K H) - |u|^2)."""
    fused = block == "fused"
    quat, log_scale, centers, C_occ, occ = sys_arrays
    qs = full_quantities(quat, log_scale, centers)
    n = pi.shape[0]
    w = np.ones(n) if valid is None else np.asarray(valid, np.float64)
    live = w != 0
    idx = np.nonzero(live)[0]
    ci, cj, cw = pi[live], pj[live], w[live]
    q = pair_density(C_occ, occ, ci, cj, cw)
    Ah, Pa, KNa = full_pair_quantities(qs, ci, cj)
    Ainv = np.linalg.inv(Ah)
    g = KNa / np.sqrt(det3(Ah))
    pref = (2.0 / math.sqrt(PI)) * PI ** 3
    nl = ci.shape[0]
    Jl = np.zeros(nl)
    GH = np.zeros((nl, 3, 3))
    GD = np.zeros((nl, 3))
    T = np.zeros(nl)
    eye = np.eye(3)
    wk = q * g                                                   # q_b g_b
    nodes = (list(zip(*boys_scaled_nodes(32))) if fused
             else [(t * t, wq) for t, wq in zip(QUAD_T, QUAD_W)])
    for a0 in range(0, nl, bra_chunk):
        sl = slice(a0, a0 + bra_chunk)
        H = Ainv[sl, None] + Ainv[None, :]                        # (B, K, 3, 3)
        d = Pa[sl, None, :] - Pa[None, :, :]
        F = np.zeros(H.shape[:2])
        gH = np.zeros(H.shape)
        gD = np.zeros(d.shape)
        rho = np.ones(H.shape[:2])
        if fused:
            Hinv = np.linalg.inv(H)
            w_ = np.einsum("bkij,bkj->bki", Hinv, d)
            q2 = np.sum(d * w_, -1)
            rho = np.cbrt(1.0 / np.linalg.det(H)) / (1.0 + q2)
            dF_drho = np.zeros(H.shape[:2])
        for c, wq in nodes:
            s2 = rho * c                                          # t^2 at this node
            X = eye + s2[..., None, None] * H
            K = np.linalg.inv(X)
            u = np.einsum("bkij,bkj->bki", K, d)
            f = wq / np.sqrt(np.linalg.det(X)) * np.exp(-s2 * np.sum(d * u, -1))
            F += f
            gH += f[..., None, None] * (-0.5 * s2[..., None, None] * K
                                        + (s2 * s2)[..., None, None] * u[..., :, None] * u[..., None, :])
            gD += (-2.0 * s2 * f)[..., None] * u
            if fused:
                trKH = np.einsum("bkij,bkji->bk", K, H)
                dF_drho += c * f * (-0.5 * trKH - np.sum(u * u, -1))
        if fused:
            sq = np.sqrt(rho)
            dFr = 0.5 * F / sq + sq * dF_drho
            F, gH, gD = sq * F, sq[..., None, None] * gH, sq[..., None] * gD
            kr = (dFr * rho)
            gH += kr[..., None, None] * (-Hinv / 3.0 + (w_[..., :, None] * w_[..., None, :])
                                         / (1.0 + q2)[..., None, None])
            gD += (-2.0 * kr / (1.0 + q2))[..., None] * w_
        T[sl] = F @ wk
        GH[sl] = np.einsum("bkij,k->bij", gH, wk)
        GD[sl] = np.einsum("bki,k->bi", gD, wk)
    Jl = pref * g * T
    E = 0.5 * float(np.sum(q * Jl))
    sc = (q * pref * g)
    Ainv_bar = sc[:, None, None] * GH
    Pbar = sc[:, None] * GD
    gbar = q * pref * T
    Abar = (-np.einsum("bij,bjk,bkl->bil", Ainv, Ainv_bar, Ainv)
            - (0.5 * gbar * g)[:, None, None] * Ainv)
    KNbar = gbar / np.sqrt(det3(Ah))
    M = centers.shape[0]
    gA = np.zeros((M, 3, 3))
    gmu = np.zeros((M, 3))
    gN = np.zeros(M)
    gC = np.zeros_like(C_occ)
    _scatter_pair_grads(qs, ci, cj, cw, Jl, Abar, Pbar, KNbar, C_occ, occ, gA, gmu, gN, gC)
    g_quat, g_log = chart_vjp(quat, log_scale, gA, gN)
    J = np.zeros(n)
    J[idx] = Jl
    return dict(E=E, J=J, g_quat=g_quat, g_log_scale=g_log, g_centers=gmu, g_C=gC, gA=gA,
                gmu=gmu, gN=gN)

# ----------------------------------------------------------------------------------------------
#  Screened RI-K  (gs_dft/coulomb/ri.py:497-544)
# ----------------------------------------------------------------------------------------------


def _exchange_D(q_splat, C, aux_q, pi, pj, valid, chunk=1024, omega=None):
    """D[P,o,o'] = sum_{live (i,k)} (P|ik) C_io C_ko' over the listed pairs (``valid`` a 0/1 mask,
    as the reference's ``cv & ov`` requires) (gs_dft/coulomb/ri.py:496-526); ``omega``: the
    long-range integrals."""
    beta, R, KN = aux_q
    n = pi.shape[0]
    live_all = np.ones(n, bool) if valid is None else (np.asarray(valid) != 0)
    D = np.zeros((beta.shape[0], C.shape[1], C.shape[1]))
    for a in range(0, n, chunk):
        sl = slice(a, a + chunk)
        live = live_all[sl]
        if not np.any(live):
            continue
        ci, cj = pi[sl][live], pj[sl][live]
        blk = full_isobra_block(beta, R, KN, *full_pair_quantities(q_splat, ci, cj), omega=omega)
        D += np.einsum("Ap,po,pq->Aoq", blk, C[ci], C[cj])
    return D


def exchange_energy_screened(sys_arrays, aux_q, lam, pi, pj, valid, chunk=1024, omega=None):
    """E_K = -tr((V + lam I)^-1 M), M_PQ = sum_{o,o'} D[P,o,o'] D[Q,o,o']
    (gs_dft/coulomb/ri.py:529-544; ``sys_arrays`` = (quat, log_scale, centers, C_occ, occ), occ
    unused as in the reference); ``omega``: the long-range exchange E_K[erf(omega r)/r] (metric
    and 3-centre integrals both attenuated). Returns (E_K, D)."""
    quat, log_scale, centers, C = sys_arrays[:4]
    q = full_quantities(quat, log_scale, centers)
    D = _exchange_D(q, C, aux_q, pi, pj, valid, chunk, omega)
    Vs = aux_metric(*aux_q, omega=omega)
    Vs[np.diag_indices_from(Vs)] += lam
    Mm = np.einsum("Aoq,Boq->AB", D, D)
    return -float(np.trace(np.linalg.solve(Vs, Mm))), D


def exchange_energy_and_grad(sys_arrays, aux_q, lam, pi, pj, valid, chunk=1024, omega=None):
    """E_K and its gradient with respect to (quat, log_scale, centers, C_occ), aux and pairs frozen.
    With Y = (V + lam I)^-1 D: dE/dD = -2 Y, dE/d(P|a) = -2 C_i^T Y_P C_k, and dE/dC from D's
    bilinear dependence on C_i, C_k."""
    quat, log_scale, centers, C = sys_arrays[:4]
    qs = full_quantities(quat, log_scale, centers)
    E, D = exchange_energy_screened(sys_arrays, aux_q, lam, pi, pj, valid, chunk, omega)
    beta, R, KN_aux = aux_q
    Vs = aux_metric(*aux_q, omega=omega)
    Vs[np.diag_indices_from(Vs)] += lam
    nA, no = D.shape[0], D.shape[1]
    Ybar = -2.0 * np.linalg.solve(Vs, D.reshape(nA, no * no)).reshape(nA, no, no)
    M = centers.shape[0]
    gA, gmu, gN = np.zeros((M, 3, 3)), np.zeros((M, 3)), np.zeros(M)
    gC = np.zeros_like(C)
    n = pi.shape[0]
    live_all = np.ones(n, bool) if valid is None else (np.asarray(valid) != 0)
    for a in range(0, n, chunk):
        sl = slice(a, a + chunk)
        live = live_all[sl]
        if not np.any(live):
            continue
        ci, cj = pi[sl][live], pj[sl][live]
        Ah, Pa, KNa = full_pair_quantities(qs, ci, cj)
        blk = full_isobra_block(beta, R, KN_aux, Ah, Pa, KNa, omega=omega)  # (N_aux, c)
        W = np.einsum("po,Aoq,pq->Ap", C[ci], Ybar, C[cj])                  # dE/d(P|a)
        _, Abar, Pbar, KNbar = _pair_vjp_integral(beta, R, KN_aux, None, Ah, Pa, KNa, None, W=W,
                                                  omega=omega)
        _scatter_pair_grads(qs, ci, cj, np.ones(ci.shape[0]), np.zeros(ci.shape[0]), Abar, Pbar,
                            KNbar, C, np.zeros(C.shape[1]), gA, gmu, gN, gC)
        T = np.einsum("Ap,Aoq->poq", blk, Ybar)                             # dE/dX[a,o,o']
        np.add.at(gC, ci, np.einsum("poq,pq->po", T, C[cj]))
        np.add.at(gC, cj, np.einsum("poq,po->pq", T, C[ci]))
    g_quat, g_log = chart_vjp(quat, log_scale, gA, gN)
    return dict(E=E, D=D, g_quat=g_quat, g_log_scale=g_log, g_centers=gmu, g_C=gC, gA=gA,
                gmu=gmu, gN=gN)

# ----------------------------------------------------------------------------------------------
#  Screened nuclear attraction on the pair list  (gs_dft/screening/pairs.py:348-370, 403-440)
# ----------------------------------------------------------------------------------------------

VNE_PREF = 2.0 * PI          # (2/sqrt(pi)) pi^1.5


def nuclear_pairs(q_splat, pi, pj, coords, charges):
    """V_ij = -N_iN_jK sum_A Z_A (2/sqrt(pi)) sum_t w_t pi^1.5 det(B)^-1/2
    exp(-(t^2 |d|^2 - t^4 d.adj(B).d / det B)), B = A_hat + t^2 I, d = P_ij - R_A: one
    reciprocal of det(B) per pair and node (gs_dft/screening/pairs.py:348-370)."""
    Ah, P, NK = full_pair_quantities(q_splat, pi, pj)
    d = P[:, None, :] - coords[None, :, :]
    d2 = np.sum(d * d, axis=-1)
    acc = np.zeros(d2.shape)
    eye = np.eye(3)
    for t, w in zip(QUAD_T, QUAD_W):
        t2 = t * t
        B = Ah + t2 * eye
        invdet = 1.0 / det3(B)
        quad = np.einsum("pak,pkl,pal->pa", d, adj3(B), d)
        expo = t2 * d2 - (t2 * t2) * quad * invdet[:, None]
        acc = acc + (w * PI ** 1.5) * np.sqrt(invdet)[:, None] * np.exp(-expo)
    acc = (2.0 / math.sqrt(PI)) * acc
    return -np.sum(charges[None, :] * acc, axis=1) * NK


def density_pairs(C, occ, pi, pj):
    """P_ij = sum_o occ_o C_io C_jo on the pair list (gs_dft/screening/pairs.py:403-406)."""
    return np.sum(occ[None, :] * C[pi] * C[pj], axis=1)


def external_energy(sys_arrays, pi, pj, valid, coords, charges, chunk=8192):
    """E_ext = sum_a valid_a P_a V_a over the listed pairs, chunked
    (gs_dft/screening/pairs.py:409-440; ``valid`` is the pair weight, pairs.py:325-327)."""
    quat, log_scale, centers, C, occ = sys_arrays
    q = full_quantities(quat, log_scale, centers)
    n = pi.shape[0]
    w = np.ones(n) if valid is None else np.asarray(valid, np.float64)
    E = 0.0
    for a in range(0, n, chunk):
        sl = slice(a, a + chunk)
        Pp = w[sl] * density_pairs(C, occ, pi[sl], pj[sl])
        E = E + float(np.sum(Pp * nuclear_pairs(q, pi[sl], pj[sl], coords, charges)))
    return E


def _pair_vjp_nuclear(coords, charges, A_pair, P_pair, KN_pair, qa):
    """For each pair: V_a and the cotangents of (A_hat, P_a, KN_a) of E = sum_a q_a V_a.

    With d = R_A - P, t^2|d|^2 - t^4 d.B^-1 d = t^2 d.A_hat B^-1 d, so per node and atom
    f = w det(B)^-1/2 exp(-t^2 d.A_hat B^-1 d) and
      df/dA_hat = f (-1/2 B^-1 - t^4 z z^T),   df/dP = 2 t^2 f A_hat z,   z = B^-1 d
    (the reference gets the same by JAX autodiff through pairs.py:356-370)."""
    n = A_pair.shape[0]
    d = coords[None, :, :] - P_pair[:, None, :]                     # (B, A, 3)
    F = np.zeros(d.shape[:2])
    GA = np.zeros((n, 3, 3))
    GP = np.zeros((n, 3))
    eye = np.eye(3)
    for t, w in zip(QUAD_T, QUAD_W):
        t2 = t * t
        B = A_pair + t2 * eye
        Binv = np.linalg.inv(B)
        z = np.einsum("bkl,bal->bak", Binv, d)
        ex = t2 * np.einsum("bak,bkl,bal->ba", d, A_pair, z)
        f = w * (1.0 / np.sqrt(np.linalg.det(B)))[:, None] * np.exp(-ex)
        F += f
        fz = charges[None, :] * f
        GA += (-0.5 * np.sum(fz, axis=1)[:, None, None] * Binv
               - (t2 * t2) * np.einsum("ba,bak,bal->bkl", fz, z, z))
        GP += 2.0 * t2 * np.einsum("bkl,bal,ba->bk", A_pair, z, fz)
    S = F @ charges
    c = -VNE_PREF * KN_pair
    V = c * S
    Abar = (qa * c)[:, None, None] * GA
    Pbar = (qa * c)[:, None] * GP
    KNbar = qa * (-VNE_PREF) * S
    return V, Abar, Pbar, KNbar


def external_energy_and_grad(sys_arrays, pi, pj, valid, coords, charges, chunk=1024):
    """E_ext, V per listed pair (0 on zero-weight entries; it is dE/dq_a) and the gradient of E_ext
    with respect to (quat, log_scale, centers, C_occ), pair list frozen."""
    quat, log_scale, centers, C_occ, occ = sys_arrays
    qs = full_quantities(quat, log_scale, centers)
    M = centers.shape[0]
    n = pi.shape[0]
    w = np.ones(n) if valid is None else np.asarray(valid, np.float64)
    V = np.zeros(n)
    gA = np.zeros((M, 3, 3))
    gmu = np.zeros((M, 3))
    gN = np.zeros(M)
    gC = np.zeros_like(C_occ)
    E = 0.0
    for a in range(0, n, chunk):
        sl = slice(a, a + chunk)
        ci, cj, cw = pi[sl], pj[sl], w[sl]
        live = cw != 0
        if not np.any(live):
            continue
        ci, cj, cw = ci[live], cj[live], cw[live]
        qa = pair_density(C_occ, occ, ci, cj, cw)
        Ah, Pa, KNa = full_pair_quantities(qs, ci, cj)
        Vc, Abar, Pbar, KNbar = _pair_vjp_nuclear(coords, charges, Ah, Pa, KNa, qa)
        V[np.arange(a, min(a + chunk, n))[live]] = Vc
        E += float(np.sum(qa * Vc))
        _scatter_pair_grads(qs, ci, cj, cw, Vc, Abar, Pbar, KNbar, C_occ, occ, gA, gmu, gN, gC)
    g_quat, g_log = chart_vjp(quat, log_scale, gA, gN)
    return dict(E=E, V=V, g_quat=g_quat, g_log_scale=g_log, g_centers=gmu, g_C=gC, gA=gA,
                gmu=gmu, gN=gN)

# ----------------------------------------------------------------------------------------------
#  Convenience: a full refresh + step for one system
# ----------------------------------------------------------------------------------------------


def refresh(quat, log_scale, centers, eps, lam, pad_to=None, unique=False, scales=(1.0,)):
    """Pair list, product aux (diagonal), metric and its factor (gs_dft/ks/energy.py:454-473)."""
    q = full_quantities(quat, log_scale, centers)
    pi, pj, valid, n_sig = neighbor_pairs(q, eps=eps, pad_to=pad_to, unique=unique)
    log_alpha, R = init_product_aux(q, scales=scales)
    aux_q = aux_quantities(log_alpha, R)
    V = aux_metric(*aux_q)
    L = aux_cholesky(V, lam)
    return dict(pi=pi, pj=pj, valid=valid, n_sig=n_sig, log_alpha=log_alpha, R=R,
                aux_q=aux_q, V=V, L=L)

# ----------------------------------------------------------------------------------------------
#  The same step with the O(N_aux x N_pairs) loops in C + OpenMP (gsdft_oracle_c.c): the checker at
#  sizes the NumPy loops cannot reach, and the multi-core CPU baseline.
# ----------------------------------------------------------------------------------------------
_CLIB = None


def c_lib():
    """Load (building with ``make`` if needed) oracle/libgsdft_oracle.so."""
    global _CLIB
    if _CLIB is None:
        import ctypes
        import os
        import subprocess
        here = os.path.dirname(os.path.abspath(__file__))
        path = os.path.join(here, "libgsdft_oracle.so")
        if not os.path.exists(path):
            subprocess.run(["make", "-C", here], check=True, capture_output=True)
        lib = ctypes.CDLL(path)
        P = ctypes.c_void_p
        lib.orc_set_nodes.argtypes = [P, P]
        lib.orc_set_threads.argtypes = [ctypes.c_int]
        lib.orc_get_threads.restype = ctypes.c_int
        # every host core the process may run on (torchrun sets OMP_NUM_THREADS=1 per rank)
        lib.orc_set_threads(len(os.sched_getaffinity(0)))
        lib.orc_gamma.argtypes = [P, ctypes.c_int64, P, P, P, ctypes.c_int64, P]
        lib.orc_vjp.argtypes = [P, ctypes.c_int64, P, P, P, ctypes.c_int64, P]
        I64, F64 = ctypes.c_int64, ctypes.c_double
        lib.orc_pairs_count.argtypes = [P, P, P, I64, F64, ctypes.c_int, F64, F64, P, P]
        lib.orc_pairs_fill.argtypes = [P, P, P, I64, F64, ctypes.c_int, F64, P, P, P, P]
        lib.orc_metric.argtypes = [P, P, P, I64, P]
        t = np.ascontiguousarray(QUAD_T)
        w = np.ascontiguousarray(QUAD_W)
        lib.orc_set_nodes(t.ctypes.data, w.ctypes.data)
        _CLIB = (lib, t, w)
    return _CLIB[0]


def pair_records(q_splat, C_occ, occ, pi, pj, valid):
    """Per live pair: [lam(3), U(9, columns = eigenvectors), P(3), KN, q] and the live indices."""
    w = np.asarray(valid, np.float64)
    live = np.nonzero(w != 0)[0]
    ci, cj = pi[live], pj[live]
    Ah, Pa, KN = full_pair_quantities(q_splat, ci, cj)
    Lam, U = np.linalg.eigh(Ah)
    qa = pair_density(C_occ, occ, ci, cj, w[live])
    rec = np.concatenate([Lam, U.reshape(-1, 9), Pa, KN[:, None], qa[:, None]], axis=1)
    return np.ascontiguousarray(rec), live


def c_threads():
    """OpenMP threads the C oracle runs with."""
    return int(c_lib().orc_get_threads())


def energy_and_grad_c(sys_arrays, aux_q, L, pi, pj, valid, want_grad=True):
    """energy_and_grad with the heavy loops in C/OpenMP. Same outputs."""
    lib = c_lib()
    quat, log_scale, centers, C_occ, occ = sys_arrays
    qs = full_quantities(quat, log_scale, centers)
    beta, R, KN_aux = (np.ascontiguousarray(a, dtype=np.float64) for a in aux_q)
    rec, live = pair_records(qs, C_occ, occ, pi, pj, valid)
    nl, na = rec.shape[0], beta.shape[0]
    gamma = np.zeros(na)
    lib.orc_gamma(rec.ctypes.data, nl, beta.ctypes.data, R.ctypes.data, KN_aux.ctypes.data, na,
                  gamma.ctypes.data)
    E, dvec = df_coulomb_solve(gamma, L)
    out = dict(E=E, gamma=gamma, d=dvec)
    if not want_grad:
        return out
    cP = np.ascontiguousarray(dvec * KN_aux)
    sums = np.zeros((nl, 13))
    lib.orc_vjp(rec.ctypes.data, nl, beta.ctypes.data, R.ctypes.data, cP.ctypes.data, na,
                sums.ctypes.data)
    Lam, U, KNa, qa = rec[:, 0:3], rec[:, 3:12].reshape(-1, 3, 3), rec[:, 15], rec[:, 16]
    kn = KNa * PREF
    qk = qa * kn
    Mkl = np.empty((nl, 3, 3))
    for (k, l), f in {(0, 0): 7, (1, 1): 8, (2, 2): 9, (0, 1): 10, (0, 2): 11, (1, 2): 12}.items():
        Mkl[:, k, l] = Mkl[:, l, k] = -qk * sums[:, f]
    for k in range(3):
        Mkl[:, k, k] -= 0.5 * qk * sums[:, 1 + k]
    Abar = np.einsum("bik,bkl,bjl->bij", U, Mkl, U)
    Pe = 2.0 * qk[:, None] * Lam * sums[:, 4:7]
    Pbar = np.einsum("bik,bk->bi", U, Pe)
    KNbar = qa * PREF * sums[:, 0]
    J = np.zeros(pi.shape[0])
    J[live] = kn * sums[:, 0]
    ci, cj = pi[live], pj[live]
    gAi, gAj, gmui, gmuj, gNi, gNj = _pair_chain(qs, ci, cj, Abar, Pbar, KNbar)
    M = centers.shape[0]
    gA, gmu, gN = np.zeros((M, 3, 3)), np.zeros((M, 3)), np.zeros(M)
    np.add.at(gA, ci, gAi)
    np.add.at(gA, cj, gAj)
    np.add.at(gmu, ci, gmui)
    np.add.at(gmu, cj, gmuj)
    np.add.at(gN, ci, gNi)
    np.add.at(gN, cj, gNj)
    w = np.asarray(valid, np.float64)[live]
    s = (J[live] * w)[:, None] * occ[None, :]
    gC = np.zeros_like(C_occ)
    np.add.at(gC, ci, s * C_occ[cj])
    np.add.at(gC, cj, s * C_occ[ci])
    g_quat, g_log = chart_vjp(quat, log_scale, gA, gN)
    out.update(J=J, g_quat=g_quat, g_log_scale=g_log, g_centers=gmu, g_C=gC, gA=gA, gmu=gmu,
               gN=gN)
    return out


def neighbor_pairs_c(q, eps, unique=False, band=1e-12):
    """The unpadded significant list of neighbor_pairs (pad_to=None) with the O(M^2) overlap sweep
    in C/OpenMP (gsdft_oracle_c.c::orc_pairs_*), for the large configurations. Same decisions as
    _significant_flat: |S| of the (min, max) orientation against eps, rows lexsorted.
    Returns (pi, pj, valid, n_sig, n_guard): n_guard counts candidates within relative ``band`` of
    eps (decisions that a last-bit change in the chart or the exponential could flip)."""
    lib = c_lib()
    A, mu, N = q
    M = int(mu.shape[0])
    A9 = np.ascontiguousarray(A.reshape(M, 9), dtype=np.float64)
    mu = np.ascontiguousarray(mu, dtype=np.float64)
    N = np.ascontiguousarray(N, dtype=np.float64)
    counts = np.zeros(M, np.int64)
    near = np.zeros(M, np.int64)
    pi15 = PI ** 1.5
    lib.orc_pairs_count(A9.ctypes.data, mu.ctypes.data, N.ctypes.data, M, float(eps), int(unique),
                        pi15, float(band), counts.ctypes.data, near.ctypes.data)
    offsets = np.zeros(M, np.int64)
    np.cumsum(counts[:-1], out=offsets[1:])
    n_sig = int(counts.sum())
    pi = np.empty(n_sig, np.int32)
    pj = np.empty(n_sig, np.int32)
    absS = np.empty(n_sig, np.float64)
    lib.orc_pairs_fill(A9.ctypes.data, mu.ctypes.data, N.ctypes.data, M, float(eps), int(unique),
                       pi15, offsets.ctypes.data, pi.ctypes.data, pj.ctypes.data, absS.ctypes.data)
    return pi, pj, pair_weights(pi, pj, unique), n_sig, int(near.sum())


def aux_metric_c(beta, R, KN):
    """aux_metric with the n^2 loop in C/OpenMP (C libm erf): the CPU baseline's refresh at the
    large configurations."""
    lib = c_lib()
    beta, R, KN = (np.ascontiguousarray(a, dtype=np.float64) for a in (beta, R, KN))
    n = int(beta.shape[0])
    V = np.empty((n, n))
    lib.orc_metric(beta.ctypes.data, R.ctypes.data, KN.ctypes.data, n, V.ctypes.data)
    return V
