"""The CUDA path at the benchmark's large configurations, against the CPU oracle.

Configuration 2 is (H2O)64 (M = 3,000 splats, n_occ = 320, 1.16e6 significant pairs) and
configuration 3 is (H2O)343 (M = 20,000, n_occ = 1,715, 1.29e7 significant pairs): the sizes the
metric is quoted on. They run the code paths the small golden systems never reach: q and g_C as
DMMA tiles over 64-splat row blocks (n_occ >= 64), int64 flat pair keys over 4e8
candidates, the packed inverse factor above N_aux = 16,384, and node screening, which only pays on
spatially extended systems.

* Pair lists: the whole significant list, bit-exact against the oracle's C sweep
  (``neighbor_pairs_c``, itself checked against the NumPy oracle on CPU); no candidate lies within
  1e-12 relative of eps, so the agreement does not hinge on a last-bit rounding.
* Steps: E, gamma, J and every gradient on a seeded random subset of the significant list (all aux),
  within relative 1e-10 (absolute floor 1e-12 of the array's scale) of the C oracle's step. Both
  sides solve with the device's own factor (copied to the host), so the comparison measures the
  integrals and the reverse pass, not two factorisations of a metric with cond ~ 1e9.
* Node screening: on (the default) against off, and the counted node evaluations.
"""
import numpy as np
import pytest

import gsdft_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

RTOL, ATOL_REL = 1e-10, 1e-12


def close(got, want, rtol=RTOL, atol_rel=ATOL_REL, what=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    scale = max(np.abs(want).max(), 1e-300) if want.size else 1.0
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol_rel * scale, err_msg=what)


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


_SYSTEMS = {}


def system(g, cfg):
    """Configuration ``cfg`` on the device: splats, the GPU's significant list (unpadded), aux and
    factor. Cached per module (the factor of configuration 3 is 3.2 GB)."""
    if cfg not in _SYSTEMS:
        from gs_dft_b200.systems import make_config
        _SYSTEMS.clear()
        torch.cuda.empty_cache()
        sy = make_config(cfg)
        s = g.Splat(dev(sy.quat), dev(sy.log_scale), dev(sy.centers))
        pi, pj, v = g.neighbor_pairs(s, eps=sy.eps)
        aux = g.init_product_aux(s)
        L = g.aux_cholesky(aux, sy.lam)
        _SYSTEMS[cfg] = (sy, s, pi, pj, v, aux, L)
    return _SYSTEMS[cfg]


@pytest.mark.parametrize("cfg", [2, 3])
def test_pair_list_bit_exact_large(g, cfg):
    sy, s, pi, pj, v, _, _ = system(g, cfg)
    q = O.full_quantities(sy.quat, sy.log_scale, sy.centers)
    opi, opj, ov, n_sig, n_guard = O.neighbor_pairs_c(q, sy.eps)
    assert n_guard == 0, f"{n_guard} candidates within 1e-12 of eps"
    assert int(pi.shape[0]) == n_sig
    assert g.screening.count_significant(s, sy.eps) == n_sig
    np.testing.assert_array_equal(host(pi), opi)
    np.testing.assert_array_equal(host(pj), opj)
    np.testing.assert_array_equal(host(v), ov)
    if cfg == 2:
        # unique mode (j >= i, weights 2 - delta_ij), and the tail padding of the pad rule
        upi, upj, uw = g.neighbor_pairs(s, eps=sy.eps, unique=True)
        opi2, opj2, ow2, _, _ = O.neighbor_pairs_c(q, sy.eps, unique=True)
        np.testing.assert_array_equal(host(upi), opi2)
        np.testing.assert_array_equal(host(upj), opj2)
        np.testing.assert_array_equal(host(uw), ow2)
        pad = 2 * n_sig + 5
        ppi, ppj, pv = g.neighbor_pairs(s, eps=sy.eps, pad_to=pad)
        assert int(ppi.shape[0]) == pad
        np.testing.assert_array_equal(host(ppi[:n_sig]), opi)
        assert not host(ppi[n_sig:]).any() and not host(pv[n_sig:]).any()


def test_pair_list_bit_exact_north_star(g):
    """Configuration 4 ((H2O)914, M = 53,000: 2.8e9 candidates, the north-star system): the whole
    significant list of the GPU bit-exact against the oracle's C sweep, and its count equal to
    BASELINE.md's 36,896,926. Pairs only (no aux or factor: the metric alone is 22.5 GB)."""
    from gs_dft_b200.systems import make_config
    _SYSTEMS.clear()
    torch.cuda.empty_cache()
    sy = make_config(4)
    s = g.Splat(dev(sy.quat), dev(sy.log_scale), dev(sy.centers))
    pi, pj, v = g.neighbor_pairs(s, eps=sy.eps)
    q = O.full_quantities(sy.quat, sy.log_scale, sy.centers)
    opi, opj, ov, n_sig, n_guard = O.neighbor_pairs_c(q, sy.eps)
    assert n_guard == 0, f"{n_guard} candidates within 1e-12 of eps"
    assert n_sig == 36_896_926 and int(pi.shape[0]) == n_sig
    np.testing.assert_array_equal(host(pi), opi)
    np.testing.assert_array_equal(host(pj), opj)
    np.testing.assert_array_equal(host(v), ov)


def _subset(n, k, seed):
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(n, size=min(k, n), replace=False))


def _engine_step(g, sy, s, pi, pj, aux, L, C_occ, screening=True):
    """One engine step (the product path: packed inverse-factor solve) on the listed pairs, with
    the node evaluations it counted."""
    import ctypes
    from gs_dft_b200._lib import lib
    beta, R, KN = aux.quantities()
    lib.call("gsdft_set_node_screening", 1 if screening else 0)
    try:
        eng = g.RIJEngine(pi, pj, torch.ones(int(pi.shape[0]), dtype=torch.float64, device="cuda"),
                          sy.M, C_occ.shape[1], beta, R.contiguous(), KN, L)
        f, r = ctypes.c_uint64(0), ctypes.c_uint64(0)
        lib.call("gsdft_node_evals", ctypes.byref(f), ctypes.byref(r), 1)
        o = eng.step(s.quat, s.log_scale, s.centers, dev(C_occ), dev(sy.occ))
        out = {k: host(t).copy() for k, t in o.items()}
        lib.call("gsdft_node_evals", ctypes.byref(f), ctypes.byref(r), 1)
        out["evals"] = (int(f.value), int(r.value))
        out["units"] = eng.plan.n_rep * eng.n_aux
        out["block"] = eng.blocks is not None
        del eng
    finally:
        lib.call("gsdft_set_node_screening", 1)
    return out


@pytest.mark.parametrize("cfg,k", [(2, 6000), (3, 3000)])
def test_step_subset_vs_oracle_large(g, cfg, k):
    """E_J, gamma, J and the gradients (quat, log_scale, centres, C_occ) on a random subset of the
    configuration's significant pairs, all aux, against the C oracle; n_occ = 320 / 1715 runs q
    and g_C as row-block DMMA tiles (SDDMM and SpMM). Node screening on (the
    product default) and off agree with each other to 1e-12 and with the oracle to 1e-10."""
    sy, s, pi, pj, v, aux, L = system(g, cfg)
    sel = _subset(int(pi.shape[0]), k, seed=cfg)
    spi, spj = host(pi)[sel], host(pj)[sel]
    dpi, dpj = dev(spi, torch.int32), dev(spj, torch.int32)
    on = _engine_step(g, sy, s, dpi, dpj, aux, L, sy.C_occ, screening=True)
    off = _engine_step(g, sy, s, dpi, dpj, aux, L, sy.C_occ, screening=False)
    Lh = host(L)
    aq = tuple(host(t) for t in aux.quantities())
    ref = O.energy_and_grad_c((sy.quat, sy.log_scale, sy.centers, sy.C_occ, sy.occ), aq, Lh,
                              spi, spj, np.ones(spi.size, bool))
    for key, rk in (("E", "E"), ("gamma", "gamma"), ("J", "J"), ("g_quat", "g_quat"),
                    ("g_log_scale", "g_log_scale"), ("g_centers", "g_centers"), ("g_C", "g_C")):
        got = on[key][:spi.size] if key == "J" else on[key]
        close(got, ref[rk], what=f"cfg{cfg} {key} vs oracle")
        close(got, off[key][:spi.size] if key == "J" else off[key], rtol=1e-12, atol_rel=1e-14,
              what=f"cfg{cfg} {key} screening on vs off")
    units = on["units"]
    assert off["evals"] == (20 * units, 20 * units)
    f, r = on["evals"]
    assert 4 * units <= f < 20 * units and 4 * units <= r < 20 * units


@pytest.mark.parametrize("n_occ", [24, 40, 100])
def test_orbital_count_branches(g, n_occ):
    """Ethanol's geometry with 24 (thread-per-pair q, 32-wide register density gradient), 40
    (warp-per-pair q, chunked density gradient) and 100 (row-block DMMA tiles, with a ragged last
    orbital tile and a ragged last row block) occupied orbitals, on a 3000-pair subset."""
    from gs_dft_b200.systems import make_config
    sy = make_config(1)
    C = np.linalg.qr(np.random.default_rng(n_occ).standard_normal((sy.M, n_occ)))[0]
    sy.C_occ, sy.occ = np.ascontiguousarray(C), np.full(n_occ, 2.0)
    s = g.Splat(dev(sy.quat), dev(sy.log_scale), dev(sy.centers))
    pi, pj, _ = g.neighbor_pairs(s, eps=sy.eps)
    aux = g.init_product_aux(s)
    L = g.aux_cholesky(aux, sy.lam)
    sel = _subset(int(pi.shape[0]), 3000, seed=n_occ)
    spi, spj = host(pi)[sel], host(pj)[sel]
    out = _engine_step(g, sy, s, dev(spi, torch.int32), dev(spj, torch.int32), aux, L, sy.C_occ)
    from gs_dft_b200.coulomb.engine import BLOCK_MIN_OCC
    assert out["block"] == (n_occ >= BLOCK_MIN_OCC) and (sy.M % 64 != 0 or n_occ < 64)
    aq = tuple(host(t) for t in aux.quantities())
    ref = O.energy_and_grad_c((sy.quat, sy.log_scale, sy.centers, sy.C_occ, sy.occ), aq, host(L),
                              spi, spj, np.ones(spi.size, bool))
    for key in ("E", "gamma", "g_quat", "g_log_scale", "g_centers", "g_C"):
        close(out[key], ref[key], what=f"n_occ={n_occ} {key}")
    close(out["J"][:spi.size], ref["J"], what=f"n_occ={n_occ} J")


def test_metric_rows_and_inverse_factor_large(g):
    """Configuration 3 (N_aux = 20,000, above the 16,384 of the unpacked inverse): sampled rows of
    the metric against the oracle's closed form; the packed inverse factor's solve against the
    substitution solve on the same factor and against the host's cho_solve. The inverse and the
    substitution carry different rounding through cond(L); the recorded agreement is the
    accuracy of the per-step solve at this size."""
    from gs_dft_b200._lib import lib, ptr, stream_handle
    sy, s, pi, pj, v, aux, L = system(g, 3)
    n = int(L.shape[0])
    beta, R, KN = (host(t) for t in aux.quantities())
    rows = _subset(n, 16, seed=7)
    V = g.aux_metric(aux)
    Vo = O.coulomb_block(beta[rows], R[rows], KN[rows], beta, R, KN)
    close(host(V[rows]), Vo, rtol=1e-12, atol_rel=1e-14)
    del V
    rng = np.random.default_rng(3)
    gam_h = np.abs(rng.standard_normal(n)) + 0.1
    gam = dev(gam_h)
    st = stream_handle(gam.device)
    Linv = torch.empty((n, n), dtype=torch.float64, device="cuda")
    lib.call("gsdft_j_solve_inverse", ptr(L), n, ptr(Linv), st)
    wb = lib.gsdft_j_solve_inv_workspace_size(n)
    ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
    d1 = torch.empty(n, dtype=torch.float64, device="cuda")
    E1 = torch.empty(1, dtype=torch.float64, device="cuda")
    lib.call("gsdft_j_solve_inv", ptr(Linv), ptr(L), ptr(gam), n, ptr(d1), ptr(E1), ptr(ws), wb, st)
    d2 = torch.empty(n, dtype=torch.float64, device="cuda")
    E2 = torch.empty(1, dtype=torch.float64, device="cuda")
    lib.call("gsdft_j_solve", ptr(L), ptr(gam), n, ptr(d2), ptr(E2), None, 0, st)
    del Linv
    torch.cuda.empty_cache()
    E_ref, d_ref = O.df_coulomb_solve(gam_h, host(L))
    close(float(E1), E_ref)
    close(float(E2), E_ref)
    close(host(d1), d_ref, rtol=1e-9, atol_rel=1e-11)
    close(host(d2), d_ref, rtol=1e-9, atol_rel=1e-11)


def test_cost_balanced_rank_slices(g):
    """Configuration 2 split over 2 and 8 ranks by estimated cost: the slices are contiguous and
    cover every representative, the ranks' estimated costs agree to within a few percent, and the
    ranks' partial gammas sum to the one-device gamma."""
    from gs_dft_b200.coulomb.engine import make_plan
    sy, s, pi, pj, v, aux, L = system(g, 2)
    beta, R, KN = aux.quantities()
    w = torch.ones(int(pi.shape[0]), dtype=torch.float64, device="cuda")
    C, occ = dev(sy.C_occ), dev(sy.occ)
    one = g.RIJEngine(pi, pj, w, sy.M, sy.n_occ, beta, R.contiguous(), KN, L)
    gam = host(one.forward_local(s.quat, s.log_scale, s.centers, C, occ)).copy()
    cost = one._cost_fn(s.quat, s.log_scale, s.centers)(one.plan.rep_pos, one.plan.n_rep)
    cost = host(cost)
    assert cost.min() > 0
    for world in (2, 8):
        total = np.zeros_like(gam)
        prev = 0
        rank_cost = []
        for rank in range(world):
            eng = g.RIJEngine(pi, pj, w, sy.M, sy.n_occ, beta, R.contiguous(), KN, L, rank=rank,
                              world=world, balance=(s.quat, s.log_scale, s.centers))
            assert eng.plan.r0 == prev
            prev = eng.plan.r1
            rank_cost.append(int(cost[eng.plan.r0:eng.plan.r1].sum()))
            total += host(eng.forward_local(s.quat, s.log_scale, s.centers, C, occ))
        assert prev == one.plan.n_rep_total
        assert max(rank_cost) / min(rank_cost) < 1.02
        close(total, gam, rtol=1e-12, atol_rel=1e-14)


def test_sharded_step_sums_to_one_device_with_row_blocks(g):
    """Configuration 2 (n_occ = 320: q and g_C on the row-block tiles) split over 2 ranks by
    estimated cost, emulated in one process: the partial gammas summed, each rank's solve and
    reverse pass on its slice, and the partial splat cotangents and g_C summed equal the one-device
    step (each rank builds its row blocks over its own representatives only)."""
    sy, s, pi, pj, v, aux, L = system(g, 2)
    beta, R, KN = aux.quantities()
    w = torch.ones(int(pi.shape[0]), dtype=torch.float64, device="cuda")
    C, occ = dev(sy.C_occ), dev(sy.occ)
    one = g.RIJEngine(pi, pj, w, sy.M, sy.n_occ, beta, R.contiguous(), KN, L)
    assert one.blocks is not None
    ref = {k: host(t).copy() for k, t in one.step(s.quat, s.log_scale, s.centers, C, occ).items()}
    del one
    ranks = [g.RIJEngine(pi, pj, w, sy.M, sy.n_occ, beta, R.contiguous(), KN, L, rank=r, world=2,
                         balance=(s.quat, s.log_scale, s.centers)) for r in range(2)]
    gam = sum(e.forward_local(s.quat, s.log_scale, s.centers, C, occ).clone() for e in ranks)
    parts = {"gA6": 0.0, "gmu": 0.0, "gN": 0.0, "g_C": 0.0}
    for e in ranks:
        assert e.blocks is not None
        e.gamma.copy_(gam)
        e.solve()
        gA6, gmu, gN, gC = e.backward_local(s.centers, C, occ)
        for k, t in (("gA6", gA6), ("gmu", gmu), ("gN", gN), ("g_C", gC[:, :sy.n_occ])):
            parts[k] = parts[k] + host(t)
    close(float(ranks[0].E[0]), ref["E"][0], rtol=1e-12)
    close(parts["g_C"], ref["g_C"], rtol=1e-10, atol_rel=1e-12)
    close(parts["gmu"], ref["g_centers"], rtol=1e-10, atol_rel=1e-12)
    close(parts["gA6"], ref["gA6"], rtol=1e-10, atol_rel=1e-12)
    close(parts["gN"], ref["gN"], rtol=1e-10, atol_rel=1e-12)
