"""The CPU oracle against golden vectors produced by executing the reference's own source
(``tests/golden/make_golden.py``). These pin the oracle before it is trusted as the checker."""
import numpy as np
import pytest

import gsdft_oracle as O
from conftest import load_golden

CASES = ["ref_rand24.npz", "ref_rand48.npz", "ref_co2.npz"]


def _q(g):
    return O.full_quantities(g["quat"], g["log_scale"], g["centers"])


@pytest.mark.parametrize("case", CASES)
def test_chart_matches_reference(case):
    g = load_golden(case)
    A, _, N = _q(g)
    np.testing.assert_allclose(A, g["A"], rtol=0, atol=1e-13 * np.abs(g["A"]).max())
    np.testing.assert_allclose(N, g["N"], rtol=1e-14)


@pytest.mark.parametrize("case", CASES)
def test_pair_lists_bit_exact(case):
    g = load_golden(case)
    q = _q(g)
    eps = float(g["eps"])
    n = g["ord_pi"].size
    pi, pj, v, n_sig = O.neighbor_pairs(q, eps=eps)
    assert n_sig == n
    np.testing.assert_array_equal(pi, g["ord_pi"])
    np.testing.assert_array_equal(pj, g["ord_pj"])
    assert v.dtype == bool and v.all()
    pi, pj, v, _ = O.neighbor_pairs(q, eps=eps, pad_to=n + 37)
    np.testing.assert_array_equal(pi, g["pad_pi"])
    np.testing.assert_array_equal(pj, g["pad_pj"])
    np.testing.assert_array_equal(v, g["pad_v"])
    pi, pj, w, _ = O.neighbor_pairs(q, eps=eps, unique=True)
    np.testing.assert_array_equal(pi, g["uni_pi"])
    np.testing.assert_array_equal(pj, g["uni_pj"])
    np.testing.assert_array_equal(w, g["uni_w"])
    M = q[1].shape[0]
    pi, pj, v, _ = O.neighbor_pairs(q, eps=-1.0, pad_to=M * M + 11)
    np.testing.assert_array_equal(pi, g["all_pi"])
    np.testing.assert_array_equal(pj, g["all_pj"])
    np.testing.assert_array_equal(v, g["all_v"])


@pytest.mark.parametrize("case", CASES)
def test_overflow_keeps_the_reference_set(case):
    """Overflow ranks by |S|. The oracle shares one overlap per unordered pair; the reference
    evaluates both orientations. The kept sets agree except where an (i,j)/(j,i) twin straddles
    the cut, which this asserts is at most one twin swap."""
    g = load_golden(case)
    q = _q(g)
    eps = float(g["eps"])
    M = q[1].shape[0]
    for key, unique in (("over", False), ("uover", True)):
        ref_pi, ref_pj = g[f"{key}_pi"], g[f"{key}_pj"]
        pad = ref_pi.size
        pi, pj, _, _ = O.neighbor_pairs(q, eps=eps, pad_to=pad, unique=unique)
        got = set(zip(pi.tolist(), pj.tolist()))
        want = set(zip(ref_pi.tolist(), ref_pj.tolist()))
        diff = got ^ want
        if unique:
            assert not diff
        else:
            assert len(diff) <= 2
            if diff:
                (a, b), (c, d) = sorted(diff)
                assert (a, b) == (d, c), "only a transposed twin may differ"
        flat = pi.astype(np.int64) * M + pj
        assert np.all(np.diff(flat) > 0)


@pytest.mark.parametrize("case", CASES)
def test_aux_metric_factor_gamma_energy(case):
    g = load_golden(case)
    q = _q(g)
    la, R = O.init_product_aux(q)
    np.testing.assert_allclose(la, g["aux_log_alpha"], rtol=0, atol=1e-14)
    np.testing.assert_allclose(R, g["aux_R"], rtol=0, atol=1e-13)
    aq = O.aux_quantities(g["aux_log_alpha"], g["aux_R"])
    V = O.aux_metric(*aq)
    np.testing.assert_allclose(V, g["V"], rtol=1e-13, atol=1e-13 * np.abs(g["V"]).max())
    L = O.aux_cholesky(V, float(g["lam"]))
    gamma = O.df_coulomb_gamma_screened(q, g["C_occ"], g["occ"], aq, g["pad_pi"], g["pad_pj"],
                                        g["pad_v"], chunk=512)
    np.testing.assert_allclose(gamma, g["gamma"], rtol=1e-12, atol=1e-12 * np.abs(g["gamma"]).max())
    E, d = O.df_coulomb_solve(gamma, L)
    np.testing.assert_allclose(E, float(g["E"]), rtol=1e-12)
    gu = O.df_coulomb_gamma_screened(q, g["C_occ"], g["occ"], aq, g["uni_pi"], g["uni_pj"],
                                     g["uni_w"], chunk=512)
    np.testing.assert_allclose(gu, g["gamma_unique"], rtol=1e-12,
                               atol=1e-12 * np.abs(g["gamma"]).max())
    # unique-weight gamma equals the ordered gamma (gs-dft tests/unit/test_pair_tricks.py:81-100)
    np.testing.assert_allclose(gu, gamma, rtol=1e-10, atol=1e-12)


def test_gradient_matches_reference_finite_differences():
    g = load_golden("ref_grad.npz")
    q = _q(g)
    pi, pj, v, _ = O.neighbor_pairs(q, eps=float(g["eps"]))
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    L = O.aux_cholesky(O.aux_metric(*aq), float(g["lam"]))
    res = O.energy_and_grad((g["quat"], g["log_scale"], g["centers"], g["C_occ"], g["occ"]),
                            aq, L, pi, pj, v)
    np.testing.assert_allclose(res["E"], float(g["E"]), rtol=1e-13)
    for k in ("g_quat", "g_log_scale", "g_centers", "g_C"):
        ref = g[k]
        # Richardson central differences are good to ~1e-10 of the largest component here.
        np.testing.assert_allclose(res[k], ref, rtol=0, atol=2e-9 * np.abs(ref).max())


def test_node_reverse_matches_reference_nodes_bwd():
    g = load_golden("ref_nodes_bwd.npz")
    coul = O.isobra_nodes(g["beta"], g["dp2"], g["Lam"])
    np.testing.assert_allclose(coul, g["coul"], rtol=1e-14)
    d_beta, d_dp2, d_Lam = O.isobra_nodes_bwd(g["beta"], g["dp2"], g["Lam"], g["gI"])
    np.testing.assert_allclose(d_beta, g["d_beta"], rtol=1e-13, atol=1e-15)
    np.testing.assert_allclose(d_dp2, g["d_dp2"], rtol=1e-13, atol=1e-15)
    np.testing.assert_allclose(d_Lam, g["d_Lam"], rtol=1e-13, atol=1e-15)


def test_pad_rule_and_stripe():
    """pad_to = ceil(pad n0 / G) G (gs_dft/ks/train.py:356-359); striping deals pairs round-robin
    so each device block has the same valid:dummy ratio (gs_dft/ks/shard.py:146-166)."""
    assert O.pad_rule(1000, 2.0, 8) == 2000
    assert O.pad_rule(1001, 2.0, 8) == 2008
    pi = np.arange(24, dtype=np.int32)
    v = np.arange(24) < 10
    spi, spj, sv = O.stripe_pairs(pi, pi, v, 4)
    blocks = sv.reshape(4, 6)
    counts = blocks.sum(1)
    assert counts.max() - counts.min() <= 1
    for b in blocks:                       # valid entries at each block's front
        k = b.sum()
        assert b[:k].all() and not b[k:].any()
    assert O.stripe_pairs(pi, pi, v, 5)[0] is pi      # n % G != 0 leaves the list alone


@pytest.mark.parametrize("case", CASES)
def test_nuclear_pairs_and_external_energy_match_reference(case):
    """V_ij on the ordered list and E_ext on the padded ordered and the unique lists, against the
    executed reference (gs_dft/screening/pairs.py:348-370, 409-440)."""
    g = load_golden(case)
    r = load_golden("ref_vne.npz")
    name = case[4:-4]
    q = _q(g)
    X, Z = r[f"{name}_atoms"], r[f"{name}_charges"]
    V = O.nuclear_pairs(q, g["ord_pi"], g["ord_pj"], X, Z)
    ref = r[f"{name}_V"]
    np.testing.assert_allclose(V, ref, rtol=1e-12, atol=1e-13 * np.abs(ref).max())
    arr = (g["quat"], g["log_scale"], g["centers"], g["C_occ"], g["occ"])
    E = O.external_energy(arr, g["pad_pi"], g["pad_pj"], g["pad_v"], X, Z)
    np.testing.assert_allclose(E, float(r[f"{name}_E"]), rtol=1e-12)
    Eu = O.external_energy(arr, g["uni_pi"], g["uni_pj"], g["uni_w"], X, Z)
    np.testing.assert_allclose(Eu, float(r[f"{name}_E_unique"]), rtol=1e-12)
    np.testing.assert_allclose(Eu, E, rtol=1e-11)         # unique weights reproduce the ordered sum


def test_external_gradient_matches_reference_finite_differences():
    """The hand-derived gradient of E_ext (the reference's is JAX autodiff) against Richardson
    central differences of the executed reference energy."""
    r = load_golden("ref_vne.npz")
    arr = (r["grad_quat"], r["grad_log_scale"], r["grad_centers"], r["grad_C_occ"], r["grad_occ"])
    q = O.full_quantities(*arr[:3])
    pi, pj, v, _ = O.neighbor_pairs(q, eps=float(r["eps"]))
    res = O.external_energy_and_grad(arr, pi, pj, v, r["grad_atoms"], r["grad_charges"])
    np.testing.assert_allclose(res["E"], float(r["grad_E"]), rtol=1e-13)
    for k in ("g_quat", "g_log_scale", "g_centers", "g_C"):
        ref = r["grad_" + k]
        np.testing.assert_allclose(res[k], ref, rtol=0, atol=2e-9 * np.abs(ref).max())


@pytest.mark.parametrize("case", CASES)
def test_exchange_energy_matches_reference(case):
    """Screened RI-K E_K on the padded ordered list against the executed reference
    (gs_dft/coulomb/ri.py:497-544). Tolerance 1e-9 relative: E_K = -sum_oq D_oq.(V + lam I)^-1 D_oq
    amplifies last-bit differences in D and V by the metric's conditioning (cond(V + lam I) = 1.5e7
    for CO2); two LU solves on metrics equal to 1e-13 already differ by 3.5e-10 there."""
    g = load_golden(case)
    r = load_golden("ref_k.npz")
    q = _q(g)
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    arr = (g["quat"], g["log_scale"], g["centers"], g["C_occ"], g["occ"])
    E, _ = O.exchange_energy_screened(arr, aq, float(g["lam"]), g["pad_pi"], g["pad_pj"],
                                      g["pad_v"])
    np.testing.assert_allclose(E, float(r[f"{case[4:-4]}_E_K"]), rtol=1e-9)


def test_exchange_gradient_matches_reference_finite_differences():
    r = load_golden("ref_k.npz")
    arr = (r["grad_quat"], r["grad_log_scale"], r["grad_centers"], r["grad_C_occ"], r["grad_occ"])
    q = O.full_quantities(*arr[:3])
    pi, pj, v, _ = O.neighbor_pairs(q, eps=float(r["eps"]))
    la, R = O.init_product_aux(q)
    res = O.exchange_energy_and_grad(arr, O.aux_quantities(la, R), float(r["lam"]), pi, pj, v)
    np.testing.assert_allclose(res["E"], float(r["grad_E_K"]), rtol=1e-12)
    for k in ("g_quat", "g_log_scale", "g_centers", "g_C"):
        ref = r["grad_" + k]
        np.testing.assert_allclose(res[k], ref, rtol=0, atol=5e-9 * np.abs(ref).max())


@pytest.mark.parametrize("case", CASES)
def test_exact_coulomb_energy_matches_reference(case):
    """Screened exact E_J (Schur (pair|pair) kernel) against the executed reference
    (gs_dft/coulomb/stream.py:249-320); CO2 on its first 2000 ordered pairs."""
    g = load_golden(case)
    r = load_golden("ref_exact.npz")
    name = case[4:-4]
    arr = (g["quat"], g["log_scale"], g["centers"], g["C_occ"], g["occ"])
    if name == "co2":
        E, _ = O.screened_coulomb_energy_exact(arr, r["co2_sub_pi"], r["co2_sub_pj"], None)
    else:
        E, _ = O.screened_coulomb_energy_exact(arr, g["pad_pi"], g["pad_pj"], g["pad_v"])
    np.testing.assert_allclose(E, float(r[f"{name}_E"]), rtol=1e-12)
    if name == "rand48":
        Eu, _ = O.screened_coulomb_energy_exact(arr, g["uni_pi"], g["uni_pj"], g["uni_w"])
        np.testing.assert_allclose(Eu, float(r["rand48_E_unique"]), rtol=1e-12)


@pytest.mark.parametrize("block", ["schur", "fused"])
def test_exact_coulomb_gradient_matches_reference(block):
    """The oracle's closed-form gradient of the screened exact E_J against Richardson central
    differences of the executed reference (10 splats, padded ordered list, pair list frozen): its
    ``screened_coulomb_energy`` (Schur block) and the same sum over ``full_eri_block_fused``."""
    r = load_golden("ref_exact_grad.npz")
    pre = "" if block == "schur" else "fused_"
    arr = (r["quat"], r["log_scale"], r["centers"], r["C_occ"], r["occ"])
    res = O.screened_coulomb_exact_and_grad(arr, r["pi"], r["pj"], r["valid"], block=block)
    np.testing.assert_allclose(res["E"], float(r[pre + "E"]), rtol=1e-12)
    for k in ("g_quat", "g_log_scale", "g_centers", "g_C"):
        ref = r[pre + k]
        np.testing.assert_allclose(res[k], ref, rtol=0, atol=5e-9 * np.abs(ref).max())


def test_exact_coulomb_fused_block_energy_matches_reference():
    """The fused 32-node block's sum on rand24's padded ordered list against the executed
    reference's ``full_eri_block_fused``; the fused and Schur rules agree to quadrature accuracy."""
    g = load_golden("ref_rand24.npz")
    r = load_golden("ref_exact_grad.npz")
    arr = (g["quat"], g["log_scale"], g["centers"], g["C_occ"], g["occ"])
    E, _ = O.screened_coulomb_energy_exact(arr, g["pad_pi"], g["pad_pj"], g["pad_v"], block="fused")
    np.testing.assert_allclose(E, float(r["rand24_fused_E"]), rtol=1e-12)
    Es = float(load_golden("ref_exact.npz")["rand24_E"])
    np.testing.assert_allclose(E, Es, rtol=1e-6)


@pytest.mark.parametrize("case", CASES)
def test_long_range_exchange_energy_matches_reference(case):
    """The long-range RI-K E_K[erf(omega r)/r] (omega = 0.3: the 12-node segment rule on
    [0, omega] and the attenuated metric, gs_dft/coulomb/ri.py:149,232-235,267-275) on the padded
    ordered list against the executed reference. The attenuated metric is far worse conditioned
    than the 1/r one (cond(V + lam I) = 1e7, 1e8 and 6e10 for the three systems), and E_K passes
    that to its last bits: on CO2 an LU and a Cholesky solve of the same D already differ by 5e-7.
    Tolerance: relative max(1e-9, 1e-16 cond)."""
    g = load_golden(case)
    r = load_golden("ref_k_lr.npz")
    q = _q(g)
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    arr = (g["quat"], g["log_scale"], g["centers"], g["C_occ"], g["occ"])
    E, _ = O.exchange_energy_screened(arr, aq, float(r["lam"]), g["pad_pi"], g["pad_pj"],
                                      g["pad_v"], omega=float(r["omega"]))
    V = O.aux_metric(*aq, omega=float(r["omega"]))
    V[np.diag_indices_from(V)] += float(r["lam"])
    rtol = max(1e-9, 1e-16 * np.linalg.cond(V))
    np.testing.assert_allclose(E, float(r[f"{case[4:-4]}_E_K_lr"]), rtol=rtol)


def test_long_range_exchange_gradient_matches_reference_finite_differences():
    """The oracle's long-range RI-K gradient against Richardson central differences of the
    executed reference (10 splats). The attenuated metric's condition number (1e6 here, against
    1e3 for 1/r) puts the differences' noise floor near 4e-8 absolute: tolerance 2e-7 of the
    largest entry or of 1."""
    r = load_golden("ref_k_lr.npz")
    arr = (r["grad_quat"], r["grad_log_scale"], r["grad_centers"], r["grad_C_occ"],
           np.ones(r["grad_C_occ"].shape[1]))
    q = O.full_quantities(*arr[:3])
    pi, pj, v, _ = O.neighbor_pairs(q, eps=float(r["eps"]))
    la, R = O.init_product_aux(q)
    res = O.exchange_energy_and_grad(arr, O.aux_quantities(la, R), float(r["lam"]), pi, pj, v,
                                     omega=float(r["omega"]))
    np.testing.assert_allclose(res["E"], float(r["grad_E_K"]), rtol=1e-10)
    for k in ("g_quat", "g_log_scale", "g_centers", "g_C"):
        ref = r["grad_" + k]
        np.testing.assert_allclose(res[k], ref, rtol=0, atol=2e-7 * max(np.abs(ref).max(), 1.0))
