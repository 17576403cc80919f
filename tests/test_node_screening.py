"""CPU checks behind two large-configuration features of the CUDA path (no GPU needed).

1. The oracle's C pair-list sweep (``neighbor_pairs_c``, the checker of the GPU list at
   configurations 2-4) gives exactly the NumPy oracle's lists, and the reference's own lists of the
   golden systems.
2. Node screening: the integral kernels stop a warp's 20-node Laplace sum once every one of its
   (aux, pair) terms has an exponent more than 2^-kNodeSkipLog2 below its first node's
   (``csrc/common.cuh``), checked after the same nodes. Emulated here per (aux, pair) — which stops
   no later than a warp, so it truncates at least as much — with the kernels' constants, on (aux,
   pair) samples of the water
   clusters: every node sum the kernels accumulate (the value and the reverse pass's weighted sums)
   is unchanged to below one rounding.
"""
import os
import re

import numpy as np
import pytest

import gsdft_oracle as O
from conftest import ROOT, load_golden


def _kernel_constants():
    """(threshold in log2 units, first checked node, check cadence) as the kernels are built."""
    src = open(os.path.join(ROOT, "gs-dft_b200", "csrc", "common.cuh")).read()
    thr = float(re.search(r"kNodeSkipLog2\s*=\s*([0-9.]+)", src).group(1))
    first = int(re.search(r"#define GSDFT_SKIP_FIRST (\d+)", src).group(1))
    every = int(re.search(r"#define GSDFT_SKIP_EVERY (\d+)", src).group(1))
    return thr, first, every


@pytest.mark.parametrize("case", ["ref_rand24.npz", "ref_rand48.npz", "ref_co2.npz"])
def test_c_pair_sweep_matches_reference_lists(case):
    d = load_golden(case)
    q = O.full_quantities(d["quat"], d["log_scale"], d["centers"])
    eps = float(d["eps"])
    pi, pj, v, n, guard = O.neighbor_pairs_c(q, eps)
    np.testing.assert_array_equal(pi, d["ord_pi"])
    np.testing.assert_array_equal(pj, d["ord_pj"])
    assert n == d["ord_pi"].size and guard == 0
    upi, upj, uw, _, _ = O.neighbor_pairs_c(q, eps, unique=True)
    np.testing.assert_array_equal(upi, d["uni_pi"])
    np.testing.assert_array_equal(upj, d["uni_pj"])
    np.testing.assert_array_equal(uw, d["uni_w"])


@pytest.mark.parametrize("cfg", [1, 2])
def test_c_pair_sweep_matches_numpy_oracle(cfg):
    from gs_dft_b200.systems import make_config
    s = make_config(cfg)
    q = O.full_quantities(s.quat, s.log_scale, s.centers)
    for unique in (False, True):
        a = O.neighbor_pairs_c(q, s.eps, unique=unique)
        b = O.neighbor_pairs(q, eps=s.eps, unique=unique)
        for x, y in zip(a[:3], b[:3]):
            np.testing.assert_array_equal(x, y)
        assert a[3] == b[3]


def _node_terms(beta, R, lam, U, P):
    """Per node n and (aux, pair): the log2 exponent x_n t_n^2 the kernels test, and the terms of
    the node sums they accumulate: f, f/G_k, t^2 f/G_k, t^4 f/(G_k G_l)."""
    t2 = O.QUAD_T ** 2
    d = R[:, None, :] - P[None, :, :]
    y = np.einsum("bki,abk->abi", U, d)
    b = beta[:, None, None]
    L = lam[None]
    ex, terms = [], []
    for n in range(t2.size):
        G = b * L + t2[n] * (b + L)
        E = t2[n] * np.sum(b * L * y * y / G, axis=-1)           # natural-log exponent
        f = O.QUAD_W[n] / np.sqrt(G.prod(-1)) * np.exp(-E)
        iG = 1.0 / G
        z = (t2[n] ** 2) * f[..., None, None] * iG[..., :, None] * iG[..., None, :]
        terms.append(np.concatenate([f[..., None], f[..., None] * iG, t2[n] * f[..., None] * iG,
                                     z.reshape(*z.shape[:2], 9)], axis=-1))
        ex.append(-E / np.log(2.0))
    return np.array(ex), np.array(terms)


@pytest.mark.parametrize("cfg", [2, 3])
def test_node_screening_changes_no_sum(cfg):
    from gs_dft_b200.systems import make_config
    thr, first, every = _kernel_constants()
    checked = np.zeros(O.QUAD_T.size, bool)
    checked[first:O.QUAD_T.size - 1:every] = True
    s = make_config(cfg)
    q = O.full_quantities(s.quat, s.log_scale, s.centers)
    la, R = O.init_product_aux(q)
    beta, R, _ = O.aux_quantities(la, R)
    M = s.M
    rng = np.random.default_rng(cfg)
    pairs = []
    for i in rng.choice(M, 4, replace=False):
        js = np.arange(M)
        sv = O.canonical_abs_overlap(q, np.full(M, i), js)
        pairs += [(i, j) for j in js[sv > s.eps]]
    pairs = np.array(pairs)
    sel = pairs[rng.choice(len(pairs), 256, replace=False)]
    Ah, P, _ = O.full_pair_quantities(q, sel[:, 0], sel[:, 1])
    lam, U = np.linalg.eigh(Ah)
    skipped_any = 0
    for chunk in range(4):
        aux = rng.choice(M, 96, replace=False)
        ex, terms = _node_terms(beta[aux], R[aux], lam, U, P)
        # the first checked node at which the exponent is thr below node 0's: nodes after it drop
        far = (ex - ex[0]) < -thr
        far[~checked] = False
        stop = np.where(far.any(0), far.argmax(0) + 1, ex.shape[0])       # nodes evaluated
        keep = np.arange(ex.shape[0])[:, None, None] < stop[None]
        full = terms.sum(0)
        trunc = np.where(keep[..., None], terms, 0.0).sum(0)
        scale = np.abs(full)
        err = np.abs(trunc - full) / np.where(scale > 0, scale, 1.0)
        assert err.max() <= 2 ** -52, f"relative truncation error {err.max():.3e}"
        skipped_any += int((stop < ex.shape[0]).sum())
    assert skipped_any > 0          # the rule does drop nodes on these extended systems
