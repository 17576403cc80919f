"""Screened exact Hartree energy on the GPU (``screened_coulomb_energy`` over ``gsdft_exact_j``)
against the executed reference's golden values (tests/golden/ref_exact.npz) and the oracle.
Tolerance: relative 1e-10 (the RI-J bound; no metric solve is involved)."""
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


def test_screened_exact_term_refuses_a_gradient(g):
    """The exact E_J has no reverse pass on this path: with inputs that require grad the term
    raises instead of returning an energy whose gradient would silently be missing."""
    d = load_golden("ref_rand24.npz")
    s = g.Splat(dev(d["quat"]), dev(d["log_scale"]), dev(d["centers"]).requires_grad_(True))
    st = g.SplatState(pairs=(dev(d["pad_pi"], torch.int32), dev(d["pad_pj"], torch.int32),
                             dev(d["pad_v"], torch.bool)))
    C, occ = dev(d["C_occ"]), dev(d["occ"])
    with pytest.raises(NotImplementedError):
        g.ScreenedExactCoulomb().energy(s, C, None, occ, st)
    with torch.no_grad():
        e_j, _ = g.ScreenedExactCoulomb().energy(s, C, None, occ, st)
    assert np.isfinite(float(e_j))
