"""CUDA path vs the CPU oracle on seeded inputs, through the C ABI (``gs_dft_b200`` host layer).

Tolerances: integer and index work (pair lists, plans) is bit-exact; FP64 values agree within the
north-star bound, relative 1e-10 with an absolute floor of 1e-12 times the array's scale (E_J,
gamma, J, gradients). Golden cases come from executing the reference's own source
(tests/golden/make_golden.py)."""
import numpy as np
import pytest

import gsdft_oracle as O
from conftest import load_golden

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL, ATOL_REL = 1e-10, 1e-12


def close(got, want, rtol=RTOL, atol_rel=ATOL_REL):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    scale = max(np.abs(want).max(), 1e-300) if want.size else 1.0
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol_rel * scale)


@pytest.fixture(scope="module")
def g():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gs_dft_b200
    gs_dft_b200._lib.lib.load()
    return gs_dft_b200


def dev(a, dtype=torch.float64):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device="cuda")


def host(t):
    return t.detach().cpu().numpy()


def splats(g, d):
    return g.Splat(dev(d["quat"]), dev(d["log_scale"]), dev(d["centers"]))


CASES = ["ref_rand24.npz", "ref_rand48.npz", "ref_co2.npz"]


@pytest.mark.parametrize("case", CASES)
def test_chart(g, case):
    d = load_golden(case)
    s = splats(g, d)
    A, _, N = O.full_quantities(d["quat"], d["log_scale"], d["centers"])
    close(host(s.A), A, rtol=1e-14, atol_rel=1e-15)
    close(host(s.norm), N, rtol=1e-14)


@pytest.mark.parametrize("case", CASES)
def test_pair_lists_bit_exact(g, case):
    d = load_golden(case)
    s = splats(g, d)
    q = O.full_quantities(d["quat"], d["log_scale"], d["centers"])
    eps = float(d["eps"])
    M = s.n_basis
    n = d["ord_pi"].size
    assert g.screening.count_significant(s, eps) == n
    for pad, unique, keys in ((None, False, ("ord_pi", "ord_pj")), (n + 37, False, ("pad_pi", "pad_pj")),
                              (None, True, ("uni_pi", "uni_pj"))):
        pi, pj, v = g.neighbor_pairs(s, eps=eps, pad_to=pad, unique=unique)
        opi, opj, ov, _ = O.neighbor_pairs(q, eps=eps, pad_to=pad, unique=unique)
        np.testing.assert_array_equal(host(pi), opi)
        np.testing.assert_array_equal(host(pj), opj)
        np.testing.assert_array_equal(host(v), ov)
        np.testing.assert_array_equal(host(pi), d[keys[0]])   # and the reference's own list
        np.testing.assert_array_equal(host(pj), d[keys[1]])
    # overflow: keep the pad largest |S|, ties by flat index, re-lexsorted
    for unique in (False, True):
        nn = O.count_significant(q, M, eps, unique)
        pad = nn // 2 + 1
        pi, pj, v = g.neighbor_pairs(s, eps=eps, pad_to=pad, unique=unique)
        opi, opj, ov, _ = O.neighbor_pairs(q, eps=eps, pad_to=pad, unique=unique)
        np.testing.assert_array_equal(host(pi), opi)
        np.testing.assert_array_equal(host(pj), opj)
    # eps < 0: every ordered pair, padded
    pi, pj, v = g.neighbor_pairs(s, eps=-1.0, pad_to=M * M + 11)
    np.testing.assert_array_equal(host(pi), d["all_pi"])
    np.testing.assert_array_equal(host(pj), d["all_pj"])
    np.testing.assert_array_equal(host(v), d["all_v"])


def test_pair_list_guard_band(g):
    """No screening decision sits within 1e-12 relative of eps on the golden systems, so the
    bit-exact agreement above does not hinge on last-bit rounding."""
    for case in CASES:
        d = load_golden(case)
        q = O.full_quantities(d["quat"], d["log_scale"], d["centers"])
        M = q[1].shape[0]
        pi = np.repeat(np.arange(M), M)
        pj = np.tile(np.arange(M), M)
        s = O.canonical_abs_overlap(q, pi, pj)
        assert np.sum(np.abs(s / float(d["eps"]) - 1.0) < 1e-12) == 0


def test_overflow_beyond_headroom_raises(g):
    d = load_golden("ref_rand24.npz")
    s = splats(g, d)
    n = d["ord_pi"].size
    with pytest.raises(ValueError):
        g.neighbor_pairs(s, eps=float(d["eps"]), pad_to=n // 3)


@pytest.mark.parametrize("case", CASES)
def test_aux_metric_factor(g, case):
    d = load_golden(case)
    s = splats(g, d)
    aux = g.init_product_aux(s)
    close(host(aux.log_alpha), d["aux_log_alpha"], rtol=1e-13, atol_rel=1e-14)
    close(host(aux.centers), d["aux_R"], rtol=1e-12, atol_rel=1e-13)
    V = g.aux_metric(aux)
    close(host(V), d["V"], rtol=1e-12, atol_rel=1e-13)
    L = g.aux_cholesky(aux, float(d["lam"]))
    Lo = O.aux_cholesky(O.aux_metric(*O.aux_quantities(host(aux.log_alpha), host(aux.centers))),
                        float(d["lam"]))
    close(host(L), Lo, rtol=1e-8, atol_rel=1e-9)       # a factor of an ill-conditioned V
    assert np.all(np.triu(host(L), 1) == 0.0)


@pytest.mark.parametrize("case", CASES)
def test_gamma_energy_vs_reference(g, case):
    d = load_golden(case)
    s = splats(g, d)
    aux = g.init_product_aux(s)
    L = g.aux_cholesky(aux, float(d["lam"]))
    pi, pj, v = dev(d["pad_pi"], torch.int32), dev(d["pad_pj"], torch.int32), dev(d["pad_v"], torch.bool)
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    gamma = g.df_coulomb_gamma_screened(s, C, occ, aux, pi, pj, valid=v)
    close(host(gamma), d["gamma"])
    E = g.df_coulomb_solve(gamma, aux, cholV=L)
    close(float(E), float(d["E"]))
    E2 = g.df_coulomb_energy_screened(s, C, occ, aux, pi, pj, valid=v, cholV=L)
    close(float(E2), float(d["E"]))
    # unique weights reproduce the ordered gamma (gs-dft tests/unit/test_pair_tricks.py:81-100)
    gu = g.df_coulomb_gamma_screened(s, C, occ, aux, dev(d["uni_pi"], torch.int32),
                                     dev(d["uni_pj"], torch.int32), valid=dev(d["uni_w"]))
    close(host(gu), d["gamma_unique"])


@pytest.mark.parametrize("cfg,M", [(1, None), (2, 1500)])
def test_inverse_factor_solve(g, cfg, M):
    """gsdft_j_solve_inv (two triangular mat-vecs on the packed [L^-1 | L^-T]) against cho_solve on the same
    factor (copied to the host), against the substitution path, and bitwise across calls;
    oversize n is rejected. The factor is the device's own: cond(V + lam I) reaches ~1e9 here, so
    last-ulp differences between two metrics move d far more than the solve method does (the
    end-to-end tests compare E and gradients with the reference)."""
    from gs_dft_b200._lib import lib, ptr, stream_handle
    from gs_dft_b200.systems import make_config
    sy = make_config(cfg, M)
    s = g.Splat(dev(sy.quat), dev(sy.log_scale), dev(sy.centers))
    aux = g.init_product_aux(s)
    L = g.aux_cholesky(aux, 1e-8)
    n = int(L.shape[0])
    aq = O.aux_quantities(host(aux.log_alpha), host(aux.centers))
    V = O.aux_metric(*aq)
    Lo = host(L)
    rng = np.random.default_rng(cfg)
    gam_h = V @ rng.standard_normal(n) + np.abs(rng.standard_normal(n))
    E_ref, d_ref = O.df_coulomb_solve(gam_h, Lo)
    gam = dev(gam_h)
    Linv = torch.empty((n, n), dtype=torch.float64, device="cuda")
    st = stream_handle(gam.device)
    lib.call("gsdft_j_solve_inverse", ptr(L), n, ptr(Linv), st)
    # packed: lower triangle = L^-1, strict upper = its mirror (L^-T)
    Lih = host(Linv)
    np.testing.assert_array_equal(np.triu(Lih, 1), np.tril(Lih, -1).T)
    close(np.tril(Lih) @ Lo, np.eye(n), rtol=0, atol_rel=1e-6)
    wb = lib.gsdft_j_solve_inv_workspace_size(n)
    ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(2):
        d_, E_ = torch.empty(n, dtype=torch.float64, device="cuda"), torch.empty(1, dtype=torch.float64, device="cuda")
        lib.call("gsdft_j_solve_inv", ptr(Linv), ptr(L), ptr(gam), n, ptr(d_), ptr(E_), ptr(ws), wb, st)
        outs.append((host(d_), float(E_)))
    close(outs[0][0], d_ref)
    close(outs[0][1], E_ref)
    assert np.array_equal(outs[0][0], outs[1][0]) and outs[0][1] == outs[1][1]
    d2, E2 = torch.empty(n, dtype=torch.float64, device="cuda"), torch.empty(1, dtype=torch.float64, device="cuda")
    lib.call("gsdft_j_solve", ptr(L), ptr(gam), n, ptr(d2), ptr(E2), None, 0, st)
    close(outs[0][0], host(d2))
    close(outs[0][1], float(E2))
    with pytest.raises(g._lib.GsdftError):
        lib.call("gsdft_j_solve_inverse", ptr(L), g._lib.SOLVE_INV_MAX + 1, ptr(Linv), st)


def _oracle_grad(d, pi, pj, v):
    q = O.full_quantities(d["quat"], d["log_scale"], d["centers"])
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    L = O.aux_cholesky(O.aux_metric(*aq), float(d["lam"]))
    return O.energy_and_grad((d["quat"], d["log_scale"], d["centers"], d["C_occ"], d["occ"]),
                             aq, L, pi, pj, v)


@pytest.mark.parametrize("case", ["ref_rand24.npz", "ref_rand48.npz", "ref_co2.npz"])
@pytest.mark.parametrize("unique", [False, True])
def test_energy_and_gradient_vs_oracle(g, case, unique):
    d = load_golden(case)
    key = ("uni_pi", "uni_pj", "uni_w") if unique else ("pad_pi", "pad_pj", "pad_v")
    pi, pj, v = d[key[0]], d[key[1]], d[key[2]]
    ref = _oracle_grad(d, pi, pj, v)
    s = splats(g, d)
    for t in (s.quat, s.log_scale, s.centers):
        t.requires_grad_(True)
    C = dev(d["C_occ"]).requires_grad_(True)
    occ = dev(d["occ"])
    aux = g.init_product_aux(s)
    L = g.aux_cholesky(aux, float(d["lam"]))
    vt = dev(v) if unique else dev(v, torch.bool)
    E = g.df_coulomb_energy_screened(s, C, occ, aux, dev(pi, torch.int32), dev(pj, torch.int32),
                                     valid=vt, cholV=L)
    E.backward()
    close(float(E), ref["E"])
    close(host(s.quat.grad), ref["g_quat"])
    close(host(s.log_scale.grad), ref["g_log_scale"])
    close(host(s.centers.grad), ref["g_centers"])
    close(host(C.grad), ref["g_C"])


def test_gradient_matches_reference_finite_differences(g):
    d = load_golden("ref_grad.npz")
    q = O.full_quantities(d["quat"], d["log_scale"], d["centers"])
    pi, pj, v, _ = O.neighbor_pairs(q, eps=float(d["eps"]))
    s = splats(g, d)
    for t in (s.quat, s.log_scale, s.centers):
        t.requires_grad_(True)
    C = dev(d["C_occ"]).requires_grad_(True)
    aux = g.init_product_aux(s)
    L = g.aux_cholesky(aux, float(d["lam"]))
    E = g.df_coulomb_energy_screened(s, C, dev(d["occ"]), aux, dev(pi, torch.int32),
                                     dev(pj, torch.int32), valid=dev(v, torch.bool), cholV=L)
    E.backward()
    close(float(E), float(d["E"]), rtol=1e-12)
    for got, k in ((s.quat.grad, "g_quat"), (s.log_scale.grad, "g_log_scale"),
                   (s.centers.grad, "g_centers"), (C.grad, "g_C")):
        np.testing.assert_allclose(host(got), d[k], rtol=0, atol=2e-9 * np.abs(d[k]).max())


def test_engine_step_j_vector_and_determinism(g):
    """J_a = sum_P (P|a) d_P per list entry (0 on padding); two steps are bit-identical."""
    d = load_golden("ref_rand48.npz")
    pi, pj, v = d["pad_pi"], d["pad_pj"], d["pad_v"]
    ref = _oracle_grad(d, pi, pj, v)
    s = splats(g, d)
    aux = g.init_product_aux(s)
    L = g.aux_cholesky(aux, float(d["lam"]))
    beta, R, KN = aux.quantities()
    eng = g.RIJEngine(dev(pi, torch.int32), dev(pj, torch.int32), dev(v), s.n_basis,
                      d["C_occ"].shape[1], beta, R.contiguous(), KN, L)
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    outs = []
    for _ in range(2):
        o = eng.step(s.quat, s.log_scale, s.centers, C, occ)
        outs.append({k: host(t).copy() for k, t in o.items()})
    close(outs[0]["J"][:pi.size], ref["J"])
    for k in outs[0]:
        np.testing.assert_array_equal(outs[0][k], outs[1][k])
    from gs_dft_b200.coulomb.engine import check_device_status
    check_device_status()


def test_sub_list_linearity(g):
    """gamma is linear in the pair list: gamma(list) = gamma(first half) + gamma(second half)."""
    d = load_golden("ref_co2.npz")
    s = splats(g, d)
    aux = g.init_product_aux(s)
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    pi, pj = dev(d["ord_pi"], torch.int32), dev(d["ord_pj"], torch.int32)
    n = pi.shape[0]
    full = g.df_coulomb_gamma_screened(s, C, occ, aux, pi, pj)
    h = n // 2
    a = g.df_coulomb_gamma_screened(s, C, occ, aux, pi[:h], pj[:h])
    b = g.df_coulomb_gamma_screened(s, C, occ, aux, pi[h:], pj[h:])
    close(host(a + b), host(full), rtol=1e-12)


def test_refresh_and_coulomb_ks(g):
    """refresh(ks, basis) + ks(model, state) through the drop-in surface, against the oracle."""
    d = load_golden("ref_rand48.npz")
    s = splats(g, d)
    ks = g.CoulombKS(coulomb=g.df(), screen=g.pairlist(eps=float(d["eps"])))
    pad = ks.initial_pad(s)
    st = g.refresh(ks, s, pad_to=pad)
    assert st.pairs[0].shape[0] == pad
    st2 = g.refresh(ks, s, like=st)
    assert st2.pairs[0].shape[0] == pad
    model = g.SplatModel(basis=s, C=dev(d["C_occ"]), occupations=dev(d["occ"]))
    E = ks(model, st)
    q = O.full_quantities(d["quat"], d["log_scale"], d["centers"])
    pi, pj, v, _ = O.neighbor_pairs(q, eps=float(d["eps"]), pad_to=pad)
    ref = _oracle_grad(d, pi, pj, v)
    close(float(E), ref["E"])


def test_ethanol_slice_vs_oracle(g):
    """Configuration 1 (ethanol, M=600): the full refresh on the GPU, the pair list checked
    bit-exactly against the oracle's, and the step on a 3000-pair slice checked against the oracle
    (the full 600 x n_sig oracle would take minutes)."""
    from gs_dft_b200.systems import make_config
    sy = make_config(1)
    s = g.Splat(dev(sy.quat), dev(sy.log_scale), dev(sy.centers))
    pi, pj, v = g.neighbor_pairs(s, eps=sy.eps)
    q = O.full_quantities(sy.quat, sy.log_scale, sy.centers)
    opi, opj, ov, n_sig = O.neighbor_pairs(q, eps=sy.eps)
    np.testing.assert_array_equal(host(pi), opi)
    np.testing.assert_array_equal(host(pj), opj)
    sl = slice(0, 3000)
    C, occ = dev(sy.C_occ), dev(sy.occ)
    for t in (s.quat, s.log_scale, s.centers):
        t.requires_grad_(True)
    Ct = C.clone().requires_grad_(True)
    aux = g.init_product_aux(s)
    L = g.aux_cholesky(aux, sy.lam)
    E = g.df_coulomb_energy_screened(s, Ct, occ, aux, pi[sl].contiguous(), pj[sl].contiguous(),
                                     valid=v[sl].contiguous(), cholV=L)
    E.backward()
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    Lo = O.aux_cholesky(O.aux_metric(*aq), sy.lam)
    ref = O.energy_and_grad((sy.quat, sy.log_scale, sy.centers, sy.C_occ, sy.occ), aq, Lo,
                            opi[sl], opj[sl], ov[sl])
    close(float(E), ref["E"])
    close(host(s.quat.grad), ref["g_quat"])
    close(host(s.log_scale.grad), ref["g_log_scale"])
    close(host(s.centers.grad), ref["g_centers"])
    close(host(Ct.grad), ref["g_C"])


def test_twin_merge_matches_unmerged_and_halves_the_work(g):
    """(i,j) and (j,i) carry the same integral: the plan evaluates each live transposed twin once
    with the summed weight. Outputs agree with the unmerged evaluation (and with the oracle, which
    evaluates every ordered entry) to 1e-10; a unique list has no twins to merge."""
    d = load_golden("ref_co2.npz")
    pi, pj, v = d["pad_pi"], d["pad_pj"], d["pad_v"]
    s = splats(g, d)
    aux = g.init_product_aux(s)
    L = g.aux_cholesky(aux, float(d["lam"]))
    beta, R, KN = aux.quantities()
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    outs = {}
    for merge in (True, False):
        eng = g.RIJEngine(dev(pi, torch.int32), dev(pj, torch.int32), dev(v), s.n_basis,
                          d["C_occ"].shape[1], beta, R.contiguous(), KN, L, merge_twins=merge)
        o = eng.step(s.quat, s.log_scale, s.centers, C, occ)
        outs[merge] = ({k: host(t).copy() for k, t in o.items()}, eng.plan)
    n_live = int(v.sum())
    n_diag = int(np.sum((pi == pj) & v))
    assert outs[False][1].n_rep_total == n_live
    assert outs[True][1].n_rep_total == n_diag + (n_live - n_diag) // 2
    for k in ("E", "gamma", "J", "g_quat", "g_log_scale", "g_centers", "g_C"):
        close(outs[True][0][k], outs[False][0][k])
    ref = _oracle_grad(d, pi, pj, v)
    close(outs[True][0]["J"][:pi.size], ref["J"])
    ui, uj, uw = d["uni_pi"], d["uni_pj"], d["uni_w"]
    eng = g.RIJEngine(dev(ui, torch.int32), dev(uj, torch.int32), dev(uw), s.n_basis,
                      d["C_occ"].shape[1], beta, R.contiguous(), KN, L)
    assert eng.plan.n_rep_total == int((uw != 0).sum())


def test_sharded_slices_cover_the_representatives(g):
    """Rank slices of the plan partition the representatives contiguously and evenly."""
    d = load_golden("ref_rand48.npz")
    pi, pj, v = dev(d["pad_pi"], torch.int32), dev(d["pad_pj"], torch.int32), dev(d["pad_v"])
    from gs_dft_b200.coulomb.engine import make_plan
    M = d["quat"].shape[0]
    full = make_plan(pi, pj, v, M)
    for world in (2, 3, 8):
        sl = [make_plan(pi, pj, v, M, r, world) for r in range(world)]
        assert sl[0].r0 == 0 and sl[-1].r1 == full.n_rep_total
        assert all(sl[k].r1 == sl[k + 1].r0 for k in range(world - 1))
        sizes = [p.n_rep for p in sl]
        assert max(sizes) - min(sizes) <= 1
        got = np.concatenate([host(p.rep_pos[:p.n_rep]) for p in sl])
        np.testing.assert_array_equal(got, host(full.rep_pos[:full.n_rep]))


def test_graph_replay_matches_eager_step(g):
    """The step captured as a CUDA graph replays to the same bits as the eager step, and follows
    new parameters copied into the captured input tensors."""
    from gs_dft_b200.coulomb.engine import StepGraph
    d = load_golden("ref_rand48.npz")
    s = splats(g, d)
    aux = g.init_product_aux(s)
    L = g.aux_cholesky(aux, float(d["lam"]))
    beta, R, KN = aux.quantities()
    eng = g.RIJEngine(dev(d["pad_pi"], torch.int32), dev(d["pad_pj"], torch.int32), dev(d["pad_v"]),
                      s.n_basis, d["C_occ"].shape[1], beta, R.contiguous(), KN, L)
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    step = lambda: eng.step(s.quat, s.log_scale, s.centers, C, occ)
    eager = {k: host(t).copy() for k, t in step().items()}
    graph = StepGraph(step)
    out = graph.replay()
    torch.cuda.synchronize()
    for k in eager:
        np.testing.assert_array_equal(host(out[k]), eager[k])
    with torch.no_grad():
        s.centers.add_(0.01)
    eager2 = {k: host(t).copy() for k, t in step().items()}
    out = graph.replay()
    torch.cuda.synchronize()
    for k in eager2:
        np.testing.assert_array_equal(host(out[k]), eager2[k])
    assert not np.array_equal(eager2["E"], eager["E"])


def test_two_forwards_then_backward_of_the_first(g):
    """The engine a refresh state caches serves every forward: a backward after a second forward
    at other orbitals re-runs its own forward first, so E(C1) and E(C2) in one loss get their own
    gradients (checked against the oracle)."""
    d = load_golden("ref_rand48.npz")
    pi, pj, v = d["pad_pi"], d["pad_pj"], d["pad_v"]
    s = splats(g, d)
    ks = g.CoulombKS(coulomb=g.df(), screen=g.pairlist(eps=float(d["eps"])))
    st = g.refresh(ks, s, pad_to=int(pi.size))
    C1 = d["C_occ"]
    C2 = np.linalg.qr(C1 + 0.05 * np.random.default_rng(1).standard_normal(C1.shape))[0]
    Ct1, Ct2 = dev(C1).requires_grad_(True), dev(C2).requires_grad_(True)
    occ = dev(d["occ"])
    E1 = ks(g.SplatModel(basis=s, C=Ct1, occupations=occ), st)
    E2 = ks(g.SplatModel(basis=s, C=Ct2, occupations=occ), st)
    E1.backward()                 # the engine's buffers hold E2's forward at this point
    q = O.full_quantities(d["quat"], d["log_scale"], d["centers"])
    opi, opj, ov, _ = O.neighbor_pairs(q, eps=float(d["eps"]), pad_to=int(pi.size))
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    Lo = O.aux_cholesky(O.aux_metric(*aq), float(d["lam"]))
    for Ch, Et, Ctg in ((C1, E1, Ct1), (C2, E2, Ct2)):
        ref = O.energy_and_grad((d["quat"], d["log_scale"], d["centers"], Ch, d["occ"]), aq, Lo,
                                opi, opj, ov)
        close(float(Et), ref["E"])
        if Ctg is Ct1:
            close(host(Ctg.grad), ref["g_C"])
    E2.backward()
    ref2 = O.energy_and_grad((d["quat"], d["log_scale"], d["centers"], C2, d["occ"]), aq, Lo,
                             opi, opj, ov)
    close(host(Ct2.grad), ref2["g_C"])
