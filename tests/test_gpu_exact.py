"""Screened exact Hartree energy on the GPU (``screened_coulomb_energy`` over ``gsdft_exact_j``)
and its gradient (``gsdft_exact_j_vjp`` + the pair chain) against the executed reference's golden
values (tests/golden/ref_exact.npz, ref_exact_grad.npz) and the oracle. Tolerance: relative 1e-10
against the oracle (the RI-J bound; no metric solve is involved); 5e-9 of the largest entry against
the reference's finite differences."""
import numpy as np
import pytest

import gsdft_oracle as O
from conftest import load_golden

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gs_dft_b200
    gs_dft_b200._lib.lib.load()
    return gs_dft_b200


def dev(a, dtype=torch.float64):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device="cuda")


def _lists(d, r, name):
    if name == "co2":
        return r["co2_sub_pi"], r["co2_sub_pj"], None
    return d["pad_pi"], d["pad_pj"], d["pad_v"]


@pytest.mark.parametrize("case", ["ref_rand24.npz", "ref_rand48.npz", "ref_co2.npz"])
def test_exact_energy_vs_reference_and_oracle(g, case):
    d = load_golden(case)
    r = load_golden("ref_exact.npz")
    name = case[4:-4]
    pi, pj, v = _lists(d, r, name)
    s = g.Splat(dev(d["quat"]), dev(d["log_scale"]), dev(d["centers"]))
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    vt = None if v is None else dev(v, torch.bool)
    E = g.screened_coulomb_energy(s, C, occ, dev(pi, torch.int32), dev(pj, torch.int32), valid=vt)
    np.testing.assert_allclose(float(E), float(r[f"{name}_E"]), rtol=1e-10)
    arr = (d["quat"], d["log_scale"], d["centers"], d["C_occ"], d["occ"])
    Eo, jv = O.screened_coulomb_energy_exact(arr, pi, pj, v)
    np.testing.assert_allclose(float(E), Eo, rtol=1e-10)
    # J per representative equals the oracle's J at the representative's list position
    E2, J, plan = g.screened_coulomb_energy(s, C, occ, dev(pi, torch.int32), dev(pj, torch.int32),
                                            valid=vt, return_j=True)
    pos = plan.rep_pos[:plan.n_rep].cpu().numpy()
    np.testing.assert_allclose(J.cpu().numpy(), jv[pos], rtol=1e-10,
                               atol=1e-12 * np.abs(jv).max())
    assert float(E2) == float(E)          # deterministic


def test_exact_unique_list_and_twin_merge(g):
    d = load_golden("ref_rand48.npz")
    r = load_golden("ref_exact.npz")
    s = g.Splat(dev(d["quat"]), dev(d["log_scale"]), dev(d["centers"]))
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    Eu = g.screened_coulomb_energy(s, C, occ, dev(d["uni_pi"], torch.int32),
                                   dev(d["uni_pj"], torch.int32), valid=dev(d["uni_w"]))
    np.testing.assert_allclose(float(Eu), float(r["rand48_E_unique"]), rtol=1e-10)
    pi, pj, v = dev(d["pad_pi"], torch.int32), dev(d["pad_pj"], torch.int32), dev(d["pad_v"], torch.bool)
    Em = g.screened_coulomb_energy(s, C, occ, pi, pj, valid=v, merge_twins=True)
    Eu2 = g.screened_coulomb_energy(s, C, occ, pi, pj, valid=v, merge_twins=False)
    np.testing.assert_allclose(float(Em), float(Eu2), rtol=1e-12)
    ks_term = g.ScreenedExactCoulomb()
    st = g.SplatState(pairs=(pi, pj, v))
    e_j, e_k = ks_term.energy(s, C, None, occ, st)
    assert float(e_j) == float(Em) and float(e_k) == 0.0


def _leaf(a):
    return dev(a).requires_grad_(True)


def _grads(g, quat, log_scale, centers, C, occ, pi, pj, v, term=False, block="schur"):
    """E and the autograd gradient of the exact E_J (direct call, or through the KS term)."""
    s = g.Splat(_leaf(quat), _leaf(log_scale), _leaf(centers))
    Ct = _leaf(C)
    pit, pjt = dev(pi, torch.int32), dev(pj, torch.int32)
    vt = None if v is None else dev(v)
    if term:
        E, _ = g.ScreenedExactCoulomb().energy(s, Ct, None, dev(occ), g.SplatState(pairs=(pit, pjt, vt)))
    else:
        E = g.screened_coulomb_energy(s, Ct, dev(occ), pit, pjt, valid=vt, block=block)
    E.backward()
    return float(E), {"g_quat": s.quat.grad, "g_log_scale": s.log_scale.grad,
                      "g_centers": s.centers.grad, "g_C": Ct.grad}


def _close(got, want, rtol, what):
    got = got.detach().cpu().numpy() if torch.is_tensor(got) else np.asarray(got)
    np.testing.assert_allclose(got, want, rtol=rtol, atol=rtol * 1e-2 * np.abs(want).max(),
                               err_msg=what)


@pytest.mark.parametrize("block", ["schur", "fused"])
def test_exact_gradient_vs_reference_fd(g, block):
    """gsdft_exact_j_vjp + the pair chain against Richardson central differences of the executed
    reference (10 splats, padded ordered list): screened_coulomb_energy (Schur block) and the same
    sum over full_eri_block_fused (the 32-node rule)."""
    r = load_golden("ref_exact_grad.npz")
    pre = "" if block == "schur" else "fused_"
    E, gr = _grads(g, r["quat"], r["log_scale"], r["centers"], r["C_occ"], r["occ"], r["pi"],
                   r["pj"], r["valid"], block=block)
    np.testing.assert_allclose(E, float(r[pre + "E"]), rtol=1e-10)
    for k, v in gr.items():
        ref = r[pre + k]
        np.testing.assert_allclose(v.cpu().numpy(), ref, rtol=0, atol=5e-9 * np.abs(ref).max(),
                                   err_msg=k)


@pytest.mark.parametrize("case,block", [("ref_rand24.npz", "schur"), ("ref_co2.npz", "schur"),
                                        ("ref_rand24.npz", "fused"), ("ref_co2.npz", "fused")])
def test_exact_gradient_vs_oracle(g, case, block):
    """The exact-E_J gradient against the oracle's closed form (direct 3x3 inverses per node) at
    relative 1e-10, for both rules: rand24's padded ordered list (twins merged on the GPU,
    zero-weight padding) and the first 600 ordered pairs of CO2 (unmatched twins)."""
    d = load_golden(case)
    if case == "ref_co2.npz":
        r = load_golden("ref_exact.npz")
        pi, pj, v = r["co2_sub_pi"][:600], r["co2_sub_pj"][:600], None
    else:
        pi, pj, v = d["pad_pi"], d["pad_pj"], d["pad_v"]
    arr = (d["quat"], d["log_scale"], d["centers"], d["C_occ"], d["occ"])
    ref = O.screened_coulomb_exact_and_grad(arr, pi, pj, v, block=block)
    E, gr = _grads(g, *arr, pi, pj, v, block=block)
    np.testing.assert_allclose(E, ref["E"], rtol=1e-10)
    for k, t in gr.items():
        _close(t, ref[k], 1e-10, f"{case} {block} {k}")
    if case == "ref_rand24.npz" and block == "fused":
        np.testing.assert_allclose(E, float(load_golden("ref_exact_grad.npz")["rand24_fused_E"]),
                                   rtol=1e-10)


def test_exact_term_is_differentiable_and_forward_token(g):
    """ScreenedExactCoulomb's energy carries the gradient (the same as the direct call), and a
    backward after another forward on the same engine re-runs its own forward first."""
    d = load_golden("ref_rand24.npz")
    arr = (d["quat"], d["log_scale"], d["centers"], d["C_occ"], d["occ"])
    pi, pj, v = d["pad_pi"], d["pad_pj"], d["pad_v"]
    E1, g1 = _grads(g, *arr, pi, pj, v)
    E2, g2 = _grads(g, *arr, pi, pj, v, term=True)
    assert E1 == E2
    for k in g1:
        assert torch.equal(g1[k], g2[k]), k
    from gs_dft_b200.coulomb.stream import _ScreenedExactEnergy, exact_engine
    s = g.Splat(_leaf(d["quat"]), _leaf(d["log_scale"]), _leaf(d["centers"]))
    C = _leaf(d["C_occ"])
    occ = dev(d["occ"])
    eng = exact_engine(s, C, dev(pi, torch.int32), dev(pj, torch.int32), dev(v))
    Ea = _ScreenedExactEnergy.apply(s.quat, s.log_scale, s.centers, C, occ, eng)
    with torch.no_grad():
        C2 = C * 1.1
    Eb = _ScreenedExactEnergy.apply(s.quat, s.log_scale, s.centers, C2, occ, eng)
    assert float(Eb) != float(Ea)
    Ea.backward()
    for k, t in (("g_quat", s.quat.grad), ("g_log_scale", s.log_scale.grad),
                 ("g_centers", s.centers.grad), ("g_C", C.grad)):
        assert torch.equal(t, g1[k]), k
