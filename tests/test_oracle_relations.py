"""Relations the reference's own tests assert for this path, checked on the CPU oracle (they pin it
beyond the golden vectors): the DF energy is a lower bound of the exact Hartree energy and
approaches it as the aux set grows (tests/unit/test_coulomb_df.py:54-63,
tests/unit/test_aux_mult.py:28-49), the closed-form 3x3 algebra agrees with LAPACK
(tests/unit/test_linalg3.py:14-44), solving with the metric's Cholesky factor agrees with a general
solve (tests/unit/test_refresh_cholv.py:24-41), and the small-argument branch of F0 joins the closed
form (tests/unit/test_coulomb_stream.py:115-134)."""
import numpy as np
import pytest

import gsdft_oracle as O


def _system():
    from gs_dft_b200.systems import small_random_system
    s = small_random_system(24, 4, seed=0)
    arr = (s.quat, s.log_scale, s.centers, s.C_occ, s.occ)
    q = O.full_quantities(s.quat, s.log_scale, s.centers)
    M = s.M
    pi = np.repeat(np.arange(M), M).astype(np.int32)     # every ordered pair: no screening
    pj = np.tile(np.arange(M), M).astype(np.int32)
    return s, arr, q, pi, pj


@pytest.fixture(scope="module")
def exact_and_df():
    s, arr, q, pi, pj = _system()
    E_exact, _ = O.screened_coulomb_energy_exact(arr, pi, pj, None)
    out = {}
    for scales in ((1.0,), (1.0, 2.0), (0.5, 1.0, 2.0)):
        la, R = O.init_product_aux(q, scales=scales)
        aq = O.aux_quantities(la, R)
        L = O.aux_cholesky(O.aux_metric(*aq), s.lam)
        E_df, _, _ = O.energy(arr, aq, L, pi, pj, np.ones(pi.size))
        out[scales] = (E_df, aq[0].shape[0])
    return s.M, E_exact, out


def test_df_energy_is_a_lower_bound(exact_and_df):
    M, E_exact, out = exact_and_df
    for scales, (E_df, _) in out.items():
        assert E_df <= E_exact * (1 + 1e-12), (scales, E_df, E_exact)


def test_bigger_aux_moves_df_toward_exact(exact_and_df):
    """Nested aux sets (scales (1), (1, 2), (0.5, 1, 2)): n_aux = mult x M and the DF gap shrinks."""
    M, E_exact, out = exact_and_df
    gaps = []
    for scales in ((1.0,), (1.0, 2.0), (0.5, 1.0, 2.0)):
        E_df, n_aux = out[scales]
        assert n_aux == len(scales) * M
        gaps.append(E_exact - E_df)
    assert gaps[0] >= gaps[1] >= gaps[2] >= -1e-12 * abs(E_exact), gaps


def test_closed_form_3x3_matches_lapack():
    rng = np.random.default_rng(0)
    B = rng.standard_normal((64, 3, 3))
    A = np.einsum("nkl,nml->nkm", B, B) + 0.5 * np.eye(3)     # SPD like A_i + A_j + t^2 I
    b = rng.standard_normal((64, 3))
    assert np.max(np.abs(O.det3(A) - np.linalg.det(A))) < 1e-12
    inv = O.adj3(A) / O.det3(A)[:, None, None]
    assert np.max(np.abs(inv - np.linalg.inv(A))) < 1e-12
    assert np.max(np.abs(O.solve3(A, b) - np.linalg.solve(A, b[..., None])[..., 0])) < 1e-12


def test_cholesky_solve_matches_general_solve():
    s, arr, q, pi, pj = _system()
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    V = O.aux_metric(*aq)
    L = O.aux_cholesky(V, s.lam)
    gamma = O.df_coulomb_gamma_screened(q, s.C_occ, s.occ, aq, pi, pj, np.ones(pi.size))
    E_chol, d_chol = O.df_coulomb_solve(gamma, L)
    Vs = V + s.lam * np.eye(V.shape[0])
    d_solve = np.linalg.solve(Vs, gamma)
    assert abs(E_chol - 0.5 * float(gamma @ d_solve)) < 1e-10 * abs(E_chol)


def test_boys_small_argument_branch_joins_closed_form():
    T = np.array([1e-8 * (1 - 1e-6), 1e-8 * (1 + 1e-6)])
    F = O.boys0(T)
    closed = 0.5 * np.sqrt(np.pi / T) * np.vectorize(__import__("math").erf)(np.sqrt(T))
    np.testing.assert_allclose(F, closed, rtol=1e-14)


@pytest.mark.parametrize("block", ["schur", "fused"])
def test_exact_coulomb_gradient_is_the_derivative_of_the_block_energy(block):
    """The closed-form exact-E_J gradient (direct 3x3 inverses per node) against Richardson
    central differences of the oracle's block energy on a seeded 8-splat system: the Schur-
    complement block, and the fused block in the reference's invariant form (C = A_a S^-1 A_b,
    I1, I2, I3, q0, q1, q2, rho). The formulations of (a|b) are independent, so this pins the
    derivative (with the fused rule's per-(a, b) scale) and the algebra that turns either form
    into det(I + t^2 H)."""
    from gs_dft_b200.systems import small_random_system
    s = small_random_system(8, 2, seed=5, spread=1.0)
    x0 = [s.quat.copy(), s.log_scale.copy(), s.centers.copy(), s.C_occ.copy(), s.occ.copy()]
    q = O.full_quantities(*x0[:3])
    pi, pj, v = O.neighbor_pairs(q, eps=1e-7)[:3]
    res = O.screened_coulomb_exact_and_grad(tuple(x0), pi, pj, v, block=block)
    E0, J0 = O.screened_coulomb_energy_exact(tuple(x0), pi, pj, v, block=block)
    np.testing.assert_allclose(res["E"], E0, rtol=1e-13)
    np.testing.assert_allclose(res["J"], J0, rtol=1e-12, atol=1e-14 * np.abs(J0).max())

    def fd(k, h):
        g = np.zeros_like(x0[k])
        for idx in np.ndindex(x0[k].shape):
            xp = [a.copy() for a in x0]
            xm = [a.copy() for a in x0]
            xp[k][idx] += h
            xm[k][idx] -= h
            g[idx] = (O.screened_coulomb_energy_exact(tuple(xp), pi, pj, v, block=block)[0]
                      - O.screened_coulomb_energy_exact(tuple(xm), pi, pj, v, block=block)[0]) / (2 * h)
        return g

    for k, name in enumerate(["g_quat", "g_log_scale", "g_centers", "g_C"]):
        ref = (4 * fd(k, 5e-4) - fd(k, 1e-3)) / 3
        np.testing.assert_allclose(res[name], ref, rtol=0, atol=1e-9 * np.abs(ref).max())


def _df_problem(seed=11, M=14, n_occ=3):
    from gs_dft_b200.systems import small_random_system
    s = small_random_system(M, n_occ, seed=seed, spread=1.2)
    arr = (s.quat, s.log_scale, s.centers, s.C_occ, s.occ)
    return s, arr


def _df_energy_and_grad(arr, pi, pj, w, lam):
    q = O.full_quantities(*arr[:3])
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    L = O.aux_cholesky(O.aux_metric(*aq), lam)
    return O.energy_and_grad(arr, aq, L, pi, pj, w)


def test_unique_weighted_list_equals_ordered_list():
    """The unique list (j >= i, weights 2 - delta_ij) gives the ordered list's E_J and gradients:
    the reference's unique-mode identity (tests/unit/test_pair_tricks.py:81-100, rtol 1e-10)."""
    s, arr = _df_problem()
    q = O.full_quantities(*arr[:3])
    pi, pj, v, _ = O.neighbor_pairs(q, eps=1e-7)
    ui, uj, uw, _ = O.neighbor_pairs(q, eps=1e-7, unique=True)
    a = _df_energy_and_grad(arr, pi, pj, np.asarray(v, np.float64), s.lam)
    b = _df_energy_and_grad(arr, ui, uj, np.asarray(uw, np.float64), s.lam)
    np.testing.assert_allclose(b["E"], a["E"], rtol=1e-10)
    for k in ("gamma", "g_quat", "g_log_scale", "g_centers", "g_C"):
        np.testing.assert_allclose(b[k], a[k], rtol=1e-10, atol=1e-12 * np.abs(a[k]).max())


def test_full_ordered_list_equals_dense_density_fit():
    """With eps < 0 (every ordered pair) the screened gamma and E_J equal the dense density fit
    gamma_P = sum_ij P_ij (P|ij) with the dense density P = C diag(occ) C^T (the reference's
    tests/unit/test_coulomb_df.py:107-126, rtol 1e-9)."""
    s, arr = _df_problem(seed=12, M=10)
    quat, log_scale, centers, C, occ = arr
    q = O.full_quantities(quat, log_scale, centers)
    pi, pj, v, _ = O.neighbor_pairs(q, eps=-1.0)
    assert pi.size == s.M * s.M
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    L = O.aux_cholesky(O.aux_metric(*aq), s.lam)
    E, gamma, _ = O.energy(arr, aq, L, pi, pj, np.ones(pi.size))
    P = (C * occ[None, :]) @ C.T
    ii, jj = np.meshgrid(np.arange(s.M), np.arange(s.M), indexing="ij")
    blk = O.full_isobra_block(*aq, *O.full_pair_quantities(q, ii.ravel(), jj.ravel()))
    gamma_dense = blk @ P.ravel()
    np.testing.assert_allclose(gamma, gamma_dense, rtol=1e-12, atol=1e-14 * np.abs(gamma).max())
    E_dense, _ = O.df_coulomb_solve(gamma_dense, L)
    np.testing.assert_allclose(E, E_dense, rtol=1e-9)


def _quat_mul(a, b):
    w1, x1, y1, z1 = a[..., 0], a[..., 1], a[..., 2], a[..., 3]
    w2, x2, y2, z2 = b[..., 0], b[..., 1], b[..., 2], b[..., 3]
    return np.stack([w1 * w2 - x1 * x2 - y1 * y2 - z1 * z2,
                     w1 * x2 + x1 * w2 + y1 * z2 - z1 * y2,
                     w1 * y2 - x1 * z2 + y1 * w2 + z1 * x2,
                     w1 * z2 + x1 * y2 - y1 * x2 + z1 * w2], -1)


def test_rotation_invariance_and_gradient_equivariance():
    """A global rotation Q of every splat (centres Q mu, orientations Q R(q)) leaves E_J unchanged
    and rotates the centre gradient (g -> Q g), the log-scale gradient staying put: the chart's
    equivariance that the reference checks (tests/unit/test_splat_chart.py:19-52), through the whole
    DF energy and its analytic gradient."""
    s, arr = _df_problem(seed=13)
    quat, log_scale, centers, C, occ = arr
    qQ = np.array([0.8, -0.3, 0.4, 0.2])
    qQ = qQ / np.linalg.norm(qQ)
    Q = O.quat_to_rotation(qQ[None])[0]
    quat_n = quat / np.linalg.norm(quat, axis=-1, keepdims=True)
    rot = (_quat_mul(np.broadcast_to(qQ, quat_n.shape), quat_n), log_scale, centers @ Q.T, C, occ)
    np.testing.assert_allclose(O.quat_to_rotation(rot[0]), Q @ O.quat_to_rotation(quat_n),
                               atol=1e-14)

    def run(a):
        qq = O.full_quantities(*a[:3])
        pi, pj, v, _ = O.neighbor_pairs(qq, eps=1e-7)
        return pi, pj, _df_energy_and_grad(a, pi, pj, np.asarray(v, np.float64), s.lam)

    pi0, pj0, r0 = run(arr)
    pi1, pj1, r1 = run(rot)
    np.testing.assert_array_equal(pi0, pi1)
    np.testing.assert_array_equal(pj0, pj1)
    np.testing.assert_allclose(r1["E"], r0["E"], rtol=1e-11)
    np.testing.assert_allclose(r1["g_centers"], r0["g_centers"] @ Q.T, rtol=1e-9,
                               atol=1e-11 * np.abs(r0["g_centers"]).max())
    np.testing.assert_allclose(r1["g_log_scale"], r0["g_log_scale"], rtol=1e-9,
                               atol=1e-11 * np.abs(r0["g_log_scale"]).max())
    np.testing.assert_allclose(r1["g_C"], r0["g_C"], rtol=1e-9, atol=1e-11 * np.abs(r0["g_C"]).max())
