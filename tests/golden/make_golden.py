"""Generate the golden vectors in this directory by EXECUTING THE REFERENCE'S OWN SOURCE.

JAX is not installable here, so the reference modules (gs_dft/basis/spectral.py, isotropic.py,
gs_dft/screening/pairs.py, gs_dft/coulomb/ri.py, stream.py, gs_dft/integrals/*.py) are imported
unmodified from a checkout of andresguzco/gs-dft and run under ``jaxshim`` (a NumPy stand-in for the
JAX API subset they use). Inputs are the seeded synthetic systems of ``gs_dft_b200.systems``.

Run from the repository root, with the reference checkout at ``jaxshim.REFERENCE_ROOT``:

    python tests/golden/make_golden.py

Outputs (compressed .npz, a few hundred KB in all):
  * ``ref_<case>.npz``  — chart (A, N), pair lists in every mode, product aux, metric, factor,
    gamma, E_J and d for three systems;
  * ``ref_grad.npz``    — the gradient of E_J w.r.t. (quat, log_scale, centers, C_occ) by
    Richardson-extrapolated central differences of the executed reference energy (pair list,
    aux and factor frozen, as in training);
  * ``ref_nodes_bwd.npz`` — the reference's hand-written node reverse pass on one block;
  * ``ref_vne.npz``     — the screened nuclear attraction: V_ij on the ordered list
    (``screened_nuclear_pairs``), E_ext on the padded ordered and the unique lists
    (``screened_external_energy``) for the three systems, and the gradient of E_ext by
    Richardson-extrapolated central differences of the executed reference on a 10-splat system.

  * ``ref_k.npz``       — screened RI-K: E_K (``df_exchange_energy_screened``) on the padded ordered
    list of the three systems, and its gradient by Richardson central differences of the executed
    reference on the 10-splat system.

  * ``ref_exact.npz``   — the screened exact Hartree energy (``screened_coulomb_energy``, the
    Schur (pair|pair) kernel) on the padded ordered lists of the two random systems, the unique
    list of the 48-splat one, and the first 2000 ordered pairs of CO2 (the full CO2 list takes the
    NumPy stand-in half an hour).

  * ``ref_exact_grad.npz`` — the gradient of the screened exact Hartree energy w.r.t. (quat,
    log_scale, centers, C_occ) by Richardson central differences of the executed reference
    (``screened_coulomb_energy``) on the 10-splat system, pair list frozen; the same for the sum
    over the fused 32-node block (``full_eri_block_fused``), and that sum's value on rand24's
    padded ordered list.

  * ``ref_k_lr.npz``    — the long-range (range-separated) RI-K E_K[erf(omega r)/r], omega = 0.3,
    on the same lists, and its gradient by Richardson central differences on the 10-splat system.

``python tests/golden/make_golden.py vne`` (or ``k``, ``k_lr``, ``exact``, ``exact_grad``)
regenerates only that file.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(ROOT, "gs-dft_b200"))

import jaxshim  # noqa: E402
from gs_dft_b200.systems import make_config, small_random_system  # noqa: E402

J = jaxshim.as_jarr


def _modules():
    return (jaxshim.load("gs_dft.basis.spectral"), jaxshim.load("gs_dft.basis.isotropic"),
            jaxshim.load("gs_dft.screening.pairs"), jaxshim.load("gs_dft.coulomb.ri"))


def _cases():
    return {
        "rand24": small_random_system(24, 4, seed=0),
        "rand48": small_random_system(48, 5, seed=1, spread=4.0, n_atoms=6),
        "co2": make_config(0),
    }


def make_case(name, s, eps=1e-7, lam=1e-8):
    spec, iso, pairs, ri = _modules()
    sp = spec.Splat(quat=J(s.quat), log_scale=J(s.log_scale), centers=J(s.centers))
    out = dict(quat=s.quat, log_scale=s.log_scale, centers=s.centers, C_occ=s.C_occ, occ=s.occ,
               eps=eps, lam=lam)
    out["A"] = np.asarray(sp.A)
    out["N"] = np.asarray(sp.norm)
    M = s.M
    pi, pj, v = pairs.neighbor_pairs(sp, eps=eps)
    n = int(pi.shape[0])
    out.update(ord_pi=np.asarray(pi), ord_pj=np.asarray(pj), ord_v=np.asarray(v))
    pi2, pj2, v2 = pairs.neighbor_pairs(sp, eps=eps, pad_to=n + 37)
    out.update(pad_pi=np.asarray(pi2), pad_pj=np.asarray(pj2), pad_v=np.asarray(v2))
    pi3, pj3, v3 = pairs.neighbor_pairs(sp, eps=eps, pad_to=n // 2 + 1)
    out.update(over_pi=np.asarray(pi3), over_pj=np.asarray(pj3), over_v=np.asarray(v3))
    ui, uj, uw = pairs.neighbor_pairs(sp, eps=eps, unique=True)
    nu = int(ui.shape[0])
    out.update(uni_pi=np.asarray(ui), uni_pj=np.asarray(uj), uni_w=np.asarray(uw))
    ui2, uj2, uw2 = pairs.neighbor_pairs(sp, eps=eps, unique=True, pad_to=nu // 2 + 3)
    out.update(uover_pi=np.asarray(ui2), uover_pj=np.asarray(uj2), uover_w=np.asarray(uw2))
    fi, fj, fv = pairs.neighbor_pairs(sp, eps=-1.0, pad_to=M * M + 11)
    out.update(all_pi=np.asarray(fi), all_pj=np.asarray(fj), all_v=np.asarray(fv))
    aux = iso.init_product_aux(sp)
    out.update(aux_log_alpha=np.asarray(aux.log_alpha), aux_R=np.asarray(aux.centers))
    out["V"] = np.asarray(ri.aux_metric(aux))
    L = ri.aux_cholesky(aux, lam)
    out["L"] = np.asarray(L)
    C, occ = J(s.C_occ), J(s.occ)
    g = ri.df_coulomb_gamma_screened(sp, C, occ, aux, pi2, pj2, chunk=512, valid=v2)
    out["gamma"] = np.asarray(g)
    out["E"] = float(ri.df_coulomb_solve(g, aux, cholV=L))
    from scipy.linalg import cho_solve
    out["d"] = cho_solve((np.asarray(L), True), np.asarray(g))
    gu = ri.df_coulomb_gamma_screened(sp, C, occ, aux, ui, uj, chunk=512, valid=uw)
    out["gamma_unique"] = np.asarray(gu)
    np.savez_compressed(os.path.join(HERE, f"ref_{name}.npz"), **out)
    print(f"{name}: M={M} n_sig={n} unique={nu} E={out['E']:.15g}")


def make_grad(eps=1e-7, lam=1e-8):
    spec, iso, pairs, ri = _modules()
    s = small_random_system(10, 3, seed=3, spread=1.0, n_atoms=3)
    sp0 = spec.Splat(quat=J(s.quat), log_scale=J(s.log_scale), centers=J(s.centers))
    pi, pj, v = pairs.neighbor_pairs(sp0, eps=eps)
    aux = iso.init_product_aux(sp0)
    L = ri.aux_cholesky(aux, lam)

    def energy(quat, ls, cen, C):
        sp = spec.Splat(quat=J(quat), log_scale=J(ls), centers=J(cen))
        return float(ri.df_coulomb_energy_screened(sp, J(C), J(s.occ), aux, pi, pj, chunk=64,
                                                   valid=v, cholV=L))

    x0 = [s.quat.copy(), s.log_scale.copy(), s.centers.copy(), s.C_occ.copy()]

    def fd(k, h):
        g = np.zeros_like(x0[k])
        for idx in np.ndindex(x0[k].shape):
            xp = [a.copy() for a in x0]
            xm = [a.copy() for a in x0]
            xp[k][idx] += h
            xm[k][idx] -= h
            g[idx] = (energy(*xp) - energy(*xm)) / (2 * h)
        return g

    out = dict(quat=s.quat, log_scale=s.log_scale, centers=s.centers, C_occ=s.C_occ, occ=s.occ,
               eps=eps, lam=lam, E=energy(*x0))
    for k, name in enumerate(["g_quat", "g_log_scale", "g_centers", "g_C"]):
        h = 1e-3
        out[name] = (4 * fd(k, h / 2) - fd(k, h)) / 3          # Richardson, O(h^4)
    np.savez_compressed(os.path.join(HERE, "ref_grad.npz"), **out)
    print("grad: M=10 E=", out["E"])


def make_nodes_bwd():
    _, _, _, ri = _modules()
    rng = np.random.default_rng(7)
    A, B = 9, 13
    beta = np.exp(rng.normal(0.0, 1.0, A))
    Lam = np.exp(rng.normal(0.0, 1.0, (B, 3)))
    dp2 = rng.uniform(0.0, 6.0, (A, B, 3))
    gI = rng.normal(0.0, 1.0, (A, B))
    nodes = ri._isobra_nodes
    coul = np.asarray(nodes(J(beta), J(dp2), J(Lam)))
    d_beta, d_dp2, d_Lam = nodes.bwd((J(beta), J(dp2), J(Lam)), J(gI))
    np.savez_compressed(os.path.join(HERE, "ref_nodes_bwd.npz"), beta=beta, Lam=Lam, dp2=dp2,
                        gI=gI, coul=coul, d_beta=np.asarray(d_beta), d_dp2=np.asarray(d_dp2),
                        d_Lam=np.asarray(d_Lam))
    print("nodes_bwd: done")


def make_vne(eps=1e-7):
    spec, _, pairs, _ = _modules()
    out = {}
    for name, s in _cases().items():
        sp = spec.Splat(quat=J(s.quat), log_scale=J(s.log_scale), centers=J(s.centers))
        X, Z = J(s.atoms), J(s.charges)
        C, occ = J(s.C_occ), J(s.occ)
        pi, pj, _ = pairs.neighbor_pairs(sp, eps=eps)
        n = int(pi.shape[0])
        out[f"{name}_V"] = np.asarray(pairs.screened_nuclear_pairs(sp, pi, pj, X, Z))
        pi2, pj2, v2 = pairs.neighbor_pairs(sp, eps=eps, pad_to=n + 37)
        out[f"{name}_E"] = float(pairs.screened_external_energy(sp, C, occ, pi2, pj2, X, Z, v2,
                                                                chunk=256))
        ui, uj, uw = pairs.neighbor_pairs(sp, eps=eps, unique=True)
        out[f"{name}_E_unique"] = float(pairs.screened_external_energy(sp, C, occ, ui, uj, X, Z,
                                                                       uw, chunk=256))
        out[f"{name}_atoms"] = s.atoms
        out[f"{name}_charges"] = s.charges
        print(f"vne {name}: n={n} E_ext={out[f'{name}_E']:.15g}")

    s = small_random_system(10, 3, seed=3, spread=1.0, n_atoms=3)
    sp0 = spec.Splat(quat=J(s.quat), log_scale=J(s.log_scale), centers=J(s.centers))
    pi, pj, v = pairs.neighbor_pairs(sp0, eps=eps)
    X, Z = J(s.atoms), J(s.charges)

    def energy(quat, ls, cen, C):
        sp = spec.Splat(quat=J(quat), log_scale=J(ls), centers=J(cen))
        return float(pairs.screened_external_energy(sp, J(C), J(s.occ), pi, pj, X, Z, v, chunk=64))

    x0 = [s.quat.copy(), s.log_scale.copy(), s.centers.copy(), s.C_occ.copy()]

    def fd(k, h):
        g = np.zeros_like(x0[k])
        for idx in np.ndindex(x0[k].shape):
            xp = [a.copy() for a in x0]
            xm = [a.copy() for a in x0]
            xp[k][idx] += h
            xm[k][idx] -= h
            g[idx] = (energy(*xp) - energy(*xm)) / (2 * h)
        return g

    out.update(grad_quat=s.quat, grad_log_scale=s.log_scale, grad_centers=s.centers,
               grad_C_occ=s.C_occ, grad_occ=s.occ, grad_atoms=s.atoms, grad_charges=s.charges,
               grad_E=energy(*x0), eps=eps)
    for k, name in enumerate(["g_quat", "g_log_scale", "g_centers", "g_C"]):
        h = 1e-3
        out["grad_" + name] = (4 * fd(k, h / 2) - fd(k, h)) / 3      # Richardson, O(h^4)
    np.savez_compressed(os.path.join(HERE, "ref_vne.npz"), **out)
    print("vne grad: M=10 E_ext=", out["grad_E"])


def make_k(eps=1e-7, lam=1e-8):
    spec, iso, pairs, ri = _modules()
    out = {}
    for name, s in _cases().items():
        sp = spec.Splat(quat=J(s.quat), log_scale=J(s.log_scale), centers=J(s.centers))
        pi, pj, _ = pairs.neighbor_pairs(sp, eps=eps)
        n = int(pi.shape[0])
        pi2, pj2, v2 = pairs.neighbor_pairs(sp, eps=eps, pad_to=n + 37)
        aux = iso.init_product_aux(sp)
        out[f"{name}_E_K"] = float(ri.df_exchange_energy_screened(sp, J(s.C_occ), aux, pi2, pj2,
                                                                   lam=lam, chunk=512, valid=v2))
        print(f"k {name}: E_K={out[f'{name}_E_K']:.15g}")

    s = small_random_system(10, 3, seed=3, spread=1.0, n_atoms=3)
    sp0 = spec.Splat(quat=J(s.quat), log_scale=J(s.log_scale), centers=J(s.centers))
    pi, pj, v = pairs.neighbor_pairs(sp0, eps=eps)
    aux = iso.init_product_aux(sp0)

    def energy(quat, ls, cen, C):
        sp = spec.Splat(quat=J(quat), log_scale=J(ls), centers=J(cen))
        return float(ri.df_exchange_energy_screened(sp, J(C), aux, pi, pj, lam=lam, chunk=64,
                                                    valid=v))

    x0 = [s.quat.copy(), s.log_scale.copy(), s.centers.copy(), s.C_occ.copy()]

    def fd(k, h):
        g = np.zeros_like(x0[k])
        for idx in np.ndindex(x0[k].shape):
            xp = [a.copy() for a in x0]
            xm = [a.copy() for a in x0]
            xp[k][idx] += h
            xm[k][idx] -= h
            g[idx] = (energy(*xp) - energy(*xm)) / (2 * h)
        return g

    out.update(grad_quat=s.quat, grad_log_scale=s.log_scale, grad_centers=s.centers,
               grad_C_occ=s.C_occ, grad_occ=s.occ, grad_E_K=energy(*x0), eps=eps, lam=lam)
    for k, name in enumerate(["g_quat", "g_log_scale", "g_centers", "g_C"]):
        h = 1e-3
        out["grad_" + name] = (4 * fd(k, h / 2) - fd(k, h)) / 3      # Richardson, O(h^4)
    np.savez_compressed(os.path.join(HERE, "ref_k.npz"), **out)
    print("k grad: M=10 E_K=", out["grad_E_K"])


def make_k_lr(eps=1e-7, lam=1e-8, omega=0.3):
    """The long-range exchange E_K[erf(omega r)/r] (``df_exchange_energy_screened(..., omega)``) on
    the padded ordered list of the three systems, and its gradient by Richardson central
    differences of the executed reference on the 10-splat system."""
    spec, iso, pairs, ri = _modules()
    out = {"omega": omega, "lam": lam, "eps": eps}
    for name, s in _cases().items():
        sp = spec.Splat(quat=J(s.quat), log_scale=J(s.log_scale), centers=J(s.centers))
        pi, pj, _ = pairs.neighbor_pairs(sp, eps=eps)
        n = int(pi.shape[0])
        pi2, pj2, v2 = pairs.neighbor_pairs(sp, eps=eps, pad_to=n + 37)
        aux = iso.init_product_aux(sp)
        out[f"{name}_E_K_lr"] = float(ri.df_exchange_energy_screened(
            sp, J(s.C_occ), aux, pi2, pj2, lam=lam, chunk=512, valid=v2, omega=omega))
        print(f"k lr {name}: E_K={out[f'{name}_E_K_lr']:.15g}", flush=True)

    s = small_random_system(10, 3, seed=3, spread=1.0, n_atoms=3)
    sp0 = spec.Splat(quat=J(s.quat), log_scale=J(s.log_scale), centers=J(s.centers))
    pi, pj, v = pairs.neighbor_pairs(sp0, eps=eps)
    aux = iso.init_product_aux(sp0)

    def energy(quat, ls, cen, C):
        sp = spec.Splat(quat=J(quat), log_scale=J(ls), centers=J(cen))
        return float(ri.df_exchange_energy_screened(sp, J(C), aux, pi, pj, lam=lam, chunk=64,
                                                    valid=v, omega=omega))

    x0 = [s.quat.copy(), s.log_scale.copy(), s.centers.copy(), s.C_occ.copy()]

    def fd(k, h):
        g = np.zeros_like(x0[k])
        for idx in np.ndindex(x0[k].shape):
            xp = [a.copy() for a in x0]
            xm = [a.copy() for a in x0]
            xp[k][idx] += h
            xm[k][idx] -= h
            g[idx] = (energy(*xp) - energy(*xm)) / (2 * h)
        return g

    out.update(grad_quat=s.quat, grad_log_scale=s.log_scale, grad_centers=s.centers,
               grad_C_occ=s.C_occ, grad_E_K=energy(*x0))
    for k, name in enumerate(["g_quat", "g_log_scale", "g_centers", "g_C"]):
        h = 1e-3
        out["grad_" + name] = (4 * fd(k, h / 2) - fd(k, h)) / 3      # Richardson, O(h^4)
    np.savez_compressed(os.path.join(HERE, "ref_k_lr.npz"), **out)
    print("k lr grad: M=10 E_K=", out["grad_E_K"])


def make_exact(eps=1e-7):
    spec, _, pairs, _ = _modules()
    cs = jaxshim.load("gs_dft.coulomb.stream")
    out = {}
    for name, s in _cases().items():
        sp = spec.Splat(quat=J(s.quat), log_scale=J(s.log_scale), centers=J(s.centers))
        C, occ = J(s.C_occ), J(s.occ)
        pi, pj, _ = pairs.neighbor_pairs(sp, eps=eps)
        n = int(pi.shape[0])
        if name == "co2":
            pi, pj, v = pi[:2000], pj[:2000], None
            out["co2_sub_pi"], out["co2_sub_pj"] = np.asarray(pi), np.asarray(pj)
        else:
            pi, pj, v = pairs.neighbor_pairs(sp, eps=eps, pad_to=n + 37)
        out[f"{name}_E"] = float(cs.screened_coulomb_energy(sp, C, occ, pi, pj, valid=v,
                                                            bra_chunk=128))
        print(f"exact {name}: E_J={out[f'{name}_E']:.15g}", flush=True)
        if name == "rand48":
            ui, uj, uw = pairs.neighbor_pairs(sp, eps=eps, unique=True)
            out["rand48_E_unique"] = float(cs.screened_coulomb_energy(sp, C, occ, ui, uj,
                                                                      valid=uw, bra_chunk=128))
    np.savez_compressed(os.path.join(HERE, "ref_exact.npz"), **out)


def make_exact_grad(eps=1e-7):
    spec, _, pairs, _ = _modules()
    cs = jaxshim.load("gs_dft.coulomb.stream")
    s = small_random_system(10, 3, seed=3, spread=1.0, n_atoms=3)
    sp0 = spec.Splat(quat=J(s.quat), log_scale=J(s.log_scale), centers=J(s.centers))
    pi, pj, _ = pairs.neighbor_pairs(sp0, eps=eps)
    n = int(pi.shape[0])
    pi, pj, v = pairs.neighbor_pairs(sp0, eps=eps, pad_to=n + 7)

    def energy(quat, ls, cen, C):
        sp = spec.Splat(quat=J(quat), log_scale=J(ls), centers=J(cen))
        return float(cs.screened_coulomb_energy(sp, J(C), J(s.occ), pi, pj, valid=v,
                                                bra_chunk=32))

    def energy_fused(quat, ls, cen, C):
        # the same sum over the fused block (the reference's screened energy is Schur-only)
        sp = spec.Splat(quat=J(quat), log_scale=J(ls), centers=J(cen))
        Pw = np.asarray(v, np.float64) * np.sum(s.occ[None, :] * C[np.asarray(pi)]
                                                * C[np.asarray(pj)], axis=1)
        blk = np.asarray(cs.full_eri_block_fused(sp, pi, pj, pi, pj))
        return 0.5 * float(Pw @ (blk @ Pw))

    x0 = [s.quat.copy(), s.log_scale.copy(), s.centers.copy(), s.C_occ.copy()]

    def fd(fn, k, h):
        g = np.zeros_like(x0[k])
        for idx in np.ndindex(x0[k].shape):
            xp = [a.copy() for a in x0]
            xm = [a.copy() for a in x0]
            xp[k][idx] += h
            xm[k][idx] -= h
            g[idx] = (fn(*xp) - fn(*xm)) / (2 * h)
        return g

    out = dict(quat=s.quat, log_scale=s.log_scale, centers=s.centers, C_occ=s.C_occ, occ=s.occ,
               pi=np.asarray(pi), pj=np.asarray(pj), valid=np.asarray(v), E=energy(*x0),
               fused_E=energy_fused(*x0), eps=eps)
    for prefix, fn in (("", energy), ("fused_", energy_fused)):
        for k, name in enumerate(["g_quat", "g_log_scale", "g_centers", "g_C"]):
            h = 1e-3
            out[prefix + name] = (4 * fd(fn, k, h / 2) - fd(fn, k, h)) / 3   # Richardson, O(h^4)
    # the fused block's energy on rand24's padded ordered list
    r24 = _cases()["rand24"]
    sp = spec.Splat(quat=J(r24.quat), log_scale=J(r24.log_scale), centers=J(r24.centers))
    qi, qj, _ = pairs.neighbor_pairs(sp, eps=eps)
    qi, qj, qv = pairs.neighbor_pairs(sp, eps=eps, pad_to=int(qi.shape[0]) + 37)
    Pw = np.asarray(qv, np.float64) * np.sum(r24.occ[None, :] * r24.C_occ[np.asarray(qi)]
                                             * r24.C_occ[np.asarray(qj)], axis=1)
    blk = np.asarray(cs.full_eri_block_fused(sp, qi, qj, qi, qj))
    out["rand24_fused_E"] = 0.5 * float(Pw @ (blk @ Pw))
    np.savez_compressed(os.path.join(HERE, "ref_exact_grad.npz"), **out)
    print("exact grad: M=10 E_J=", out["E"], "fused", out["fused_E"], "rand24 fused",
          out["rand24_fused_E"])


if __name__ == "__main__":
    if sys.argv[1:] == ["exact"]:
        make_exact()
        sys.exit(0)
    if sys.argv[1:] == ["vne"]:
        make_vne()
        sys.exit(0)
    if sys.argv[1:] == ["k"]:
        make_k()
        sys.exit(0)
    if sys.argv[1:] == ["exact_grad"]:
        make_exact_grad()
        sys.exit(0)
    if sys.argv[1:] == ["k_lr"]:
        make_k_lr()
        sys.exit(0)
    for name, s in _cases().items():
        make_case(name, s)
    make_grad()
    make_nodes_bwd()
    make_vne()
    make_k()
    make_k_lr()
    make_exact()
    make_exact_grad()
