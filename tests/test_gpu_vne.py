"""Screened nuclear attraction on the GPU (``gsdft_vne`` behind ``screened_nuclear_pairs`` /
``screened_external_energy`` / ``RIJEngine(atoms=...)``) against the executed reference's golden
vectors (tests/golden/ref_vne.npz) and the oracle.

Tolerances as for RI-J: relative 1e-10 with an absolute floor of 1e-12 x the array's scale;
gradients against the reference's finite differences to their accuracy (2e-9 of the scale)."""
import numpy as np
import pytest

import gsdft_oracle as O
from conftest import load_golden

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

CASES = ["ref_rand24.npz", "ref_rand48.npz", "ref_co2.npz"]


def close(got, want, rtol=1e-10, atol_rel=1e-12):
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


def _case(g, case):
    d = load_golden(case)
    r = load_golden("ref_vne.npz")
    name = case[4:-4]
    s = g.Splat(dev(d["quat"]), dev(d["log_scale"]), dev(d["centers"]))
    return d, s, r[f"{name}_atoms"], r[f"{name}_charges"], r, name


@pytest.mark.parametrize("case", CASES)
def test_nuclear_pairs_and_external_energy_vs_reference(g, case):
    d, s, X, Z, r, name = _case(g, case)
    V = g.screened_nuclear_pairs(s, dev(d["ord_pi"], torch.int32), dev(d["ord_pj"], torch.int32),
                                 X, Z)
    close(host(V), r[f"{name}_V"])
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    E = g.screened_external_energy(s, C, occ, dev(d["pad_pi"], torch.int32),
                                   dev(d["pad_pj"], torch.int32), X, Z,
                                   valid=dev(d["pad_v"], torch.bool))
    close(float(E), float(r[f"{name}_E"]))
    Eu = g.screened_external_energy(s, C, occ, dev(d["uni_pi"], torch.int32),
                                    dev(d["uni_pj"], torch.int32), X, Z, valid=dev(d["uni_w"]))
    close(float(Eu), float(r[f"{name}_E_unique"]))


@pytest.mark.parametrize("case", CASES)
def test_density_pairs(g, case):
    d = load_golden(case)
    P = g.density_pairs(dev(d["C_occ"]), dev(d["occ"]), dev(d["ord_pi"], torch.int32),
                        dev(d["ord_pj"], torch.int32))
    close(host(P), O.density_pairs(d["C_occ"], d["occ"], d["ord_pi"], d["ord_pj"]), rtol=1e-13)


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("unique", [False, True])
def test_external_energy_and_gradient_vs_oracle(g, case, unique):
    d, s, X, Z, _, _ = _case(g, case)
    key = ("uni_pi", "uni_pj", "uni_w") if unique else ("pad_pi", "pad_pj", "pad_v")
    pi, pj, v = d[key[0]], d[key[1]], d[key[2]]
    ref = O.external_energy_and_grad((d["quat"], d["log_scale"], d["centers"], d["C_occ"],
                                      d["occ"]), pi, pj, v, X, Z)
    for t in (s.quat, s.log_scale, s.centers):
        t.requires_grad_(True)
    C = dev(d["C_occ"]).requires_grad_(True)
    vt = dev(v) if unique else dev(v, torch.bool)
    E = g.screened_external_energy(s, C, dev(d["occ"]), dev(pi, torch.int32), dev(pj, torch.int32),
                                   X, Z, valid=vt)
    E.backward()
    close(float(E), ref["E"])
    close(host(s.quat.grad), ref["g_quat"])
    close(host(s.log_scale.grad), ref["g_log_scale"])
    close(host(s.centers.grad), ref["g_centers"])
    close(host(C.grad), ref["g_C"])


def test_external_gradient_vs_reference_finite_differences(g):
    r = load_golden("ref_vne.npz")
    q = O.full_quantities(r["grad_quat"], r["grad_log_scale"], r["grad_centers"])
    pi, pj, v, _ = O.neighbor_pairs(q, eps=float(r["eps"]))
    s = g.Splat(dev(r["grad_quat"]), dev(r["grad_log_scale"]), dev(r["grad_centers"]))
    for t in (s.quat, s.log_scale, s.centers):
        t.requires_grad_(True)
    C = dev(r["grad_C_occ"]).requires_grad_(True)
    E = g.screened_external_energy(s, C, dev(r["grad_occ"]), dev(pi, torch.int32),
                                   dev(pj, torch.int32), r["grad_atoms"], r["grad_charges"],
                                   valid=dev(v, torch.bool))
    E.backward()
    close(float(E), float(r["grad_E"]), rtol=1e-12)
    for got, k in ((s.quat.grad, "g_quat"), (s.log_scale.grad, "g_log_scale"),
                   (s.centers.grad, "g_centers"), (C.grad, "g_C")):
        want = r["grad_" + k]
        np.testing.assert_allclose(host(got), want, rtol=0, atol=2e-9 * np.abs(want).max())


def _engine(g, d, s, X, Z, merge=True, with_rij=True):
    from gs_dft_b200.screening import atom_records
    pi, pj, v = d["pad_pi"], d["pad_pj"], d["pad_v"]
    kw = {}
    if with_rij:
        aux = g.init_product_aux(s)
        L = g.aux_cholesky(aux, float(d["lam"]))
        beta, R, KN = aux.quantities()
        kw = dict(beta=beta, R=R.contiguous(), KN=KN, L=L)
    return g.RIJEngine(dev(pi, torch.int32), dev(pj, torch.int32), dev(v), s.n_basis,
                       d["C_occ"].shape[1], merge_twins=merge, atoms=atom_records(X, Z, "cuda"),
                       **kw)


def test_combined_step_carries_both_terms(g):
    """One engine step with atoms: E_J and E_ne each as the oracle's, the gradient and J = dE/dq
    of their sum; twin merging on and off agree; two steps are bit-identical."""
    d, s, X, Z, _, _ = _case(g, "ref_rand48.npz")
    pi, pj, v = d["pad_pi"], d["pad_pj"], d["pad_v"]
    arr = (d["quat"], d["log_scale"], d["centers"], d["C_occ"], d["occ"])
    q = O.full_quantities(*arr[:3])
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    Lo = O.aux_cholesky(O.aux_metric(*aq), float(d["lam"]))
    rj = O.energy_and_grad(arr, aq, Lo, pi, pj, v)
    rn = O.external_energy_and_grad(arr, pi, pj, v, X, Z)
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    outs = {}
    for merge in (True, False):
        eng = _engine(g, d, s, X, Z, merge)
        runs = []
        for _ in range(2):
            o = eng.step(s.quat, s.log_scale, s.centers, C, occ)
            runs.append({k: host(t).copy() for k, t in o.items()})
        for k in runs[0]:
            np.testing.assert_array_equal(runs[0][k], runs[1][k])
        outs[merge] = runs[0]
    o = outs[True]
    close(float(o["E"][0]), rj["E"])
    close(float(o["E_ne"][0]), rn["E"])
    close(o["V"][:pi.size], rn["V"] * (v != 0))
    close(o["J"][:pi.size], rj["J"] + rn["V"] * (v != 0))
    for k in ("g_quat", "g_log_scale", "g_centers", "g_C"):
        close(o[k], rj[k] + rn[k])
        close(outs[False][k], o[k])


def test_external_only_engine_and_external_ks(g):
    """An engine without the RI-J term (beta=None), and ExternalKS on a refresh state, both equal
    screened_external_energy."""
    d, s, X, Z, r, name = _case(g, "ref_co2.npz")
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    eng = _engine(g, d, s, X, Z, with_rij=False)
    o = eng.step(s.quat, s.log_scale, s.centers, C, occ)
    close(float(o["E_ne"][0]), float(r[f"{name}_E"]))
    ref = O.external_energy_and_grad((d["quat"], d["log_scale"], d["centers"], d["C_occ"],
                                      d["occ"]), d["pad_pi"], d["pad_pj"], d["pad_v"], X, Z)
    close(host(o["g_centers"]), ref["g_centers"])
    ks = g.CoulombKS(coulomb=g.df(), screen=g.pairlist(eps=float(d["eps"])))
    st = g.refresh(ks, s, pad_to=int(d["pad_pi"].size))
    model = g.SplatModel(basis=s, C=C, occupations=occ)
    Ek = g.ExternalKS(X, Z)(model, st)
    close(float(Ek), float(r[f"{name}_E"]))


def test_ethanol_external_energy_vs_oracle(g):
    """Configuration 1 (ethanol, M = 600, 296,744 live pairs, 9 nuclei): V on the full list and E_ne
    against the oracle."""
    from gs_dft_b200.systems import make_config
    sy = make_config(1)
    s = g.Splat(dev(sy.quat), dev(sy.log_scale), dev(sy.centers))
    pi, pj, v = g.neighbor_pairs(s, eps=sy.eps)
    V = g.screened_nuclear_pairs(s, pi, pj, sy.atoms, sy.charges)
    q = O.full_quantities(sy.quat, sy.log_scale, sy.centers)
    hp, hq = host(pi), host(pj)
    Vo = np.concatenate([O.nuclear_pairs(q, hp[k:k + 20000], hq[k:k + 20000], sy.atoms, sy.charges)
                         for k in range(0, hp.size, 20000)])
    close(host(V), Vo)
    E = g.screened_external_energy(s, dev(sy.C_occ), dev(sy.occ), pi, pj, sy.atoms, sy.charges,
                                   valid=v)
    Eo = O.external_energy((sy.quat, sy.log_scale, sy.centers, sy.C_occ, sy.occ), hp, hq,
                           host(v), sy.atoms, sy.charges, chunk=20000)
    close(float(E), Eo)


def test_sharded_slices_sum_to_the_whole(g):
    """Engines on the rank slices of a 3-way partition: their E_ne partials and gradient
    contributions sum to the single-engine values."""
    d, s, X, Z, _, _ = _case(g, "ref_co2.npz")
    from gs_dft_b200.screening import atom_records
    pi, pj, v = dev(d["pad_pi"], torch.int32), dev(d["pad_pj"], torch.int32), dev(d["pad_v"])
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    atoms = atom_records(X, Z, "cuda")

    def run(rank, world):
        eng = g.RIJEngine(pi, pj, v, s.n_basis, C.shape[1], atoms=atoms, rank=rank, world=world)
        eng.prepare(s.quat, s.log_scale, s.centers, C, occ)
        eng.backward_local(s.centers, C, occ)
        return float(eng.E_ne[0]), host(eng.gmu).copy(), host(eng.gA6).copy()

    E1, gmu1, gA1 = run(0, 1)
    parts = [run(r, 3) for r in range(3)]
    close(sum(p[0] for p in parts), E1, rtol=1e-12)
    close(sum(p[1] for p in parts), gmu1, rtol=1e-11)
    close(sum(p[2] for p in parts), gA1, rtol=1e-11)
