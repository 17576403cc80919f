"""The library's dense FP64 routines on the tensor cores (DMMA), against host LAPACK / NumPy on the
same inputs: the GEMM in every transpose combination with ragged sizes, the blocked Cholesky of
V + lam I (including the not-positive-definite error), the packed inverse factor, and the one-shot
blocked triangular solve. Well-conditioned random matrices bound the comparison at the level of
rounding; the aux metrics themselves are covered end to end in test_gpu_parity.py and
test_gpu_large.py."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gs_dft_b200
    gs_dft_b200._lib.lib.load()
    return gs_dft_b200


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float64, device="cuda")


def host(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("ta", [0, 1])
@pytest.mark.parametrize("tb", [0, 1])
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (64, 64, 16), (70, 130, 37), (257, 63, 1000),
                                   (5, 300, 4100)])
def test_gemm_matches_host(g, ta, tb, M, N, K):
    from gs_dft_b200._lib import lib, ptr, stream_handle
    rng = np.random.default_rng(M * 7 + N * 3 + K + 11 * ta + 13 * tb)
    A = rng.standard_normal((K, M) if ta else (M, K))
    B = rng.standard_normal((N, K) if tb else (K, N))
    C0 = rng.standard_normal((M, N))
    want = 0.75 * (A.T if ta else A) @ (B.T if tb else B) - 0.5 * C0
    dA, dB, dC = dev(A), dev(B), dev(C0)
    lib.call("gsdft_dense_gemm", ta, tb, M, N, K, 0.75, ptr(dA), A.shape[1], ptr(dB), B.shape[1],
             -0.5, ptr(dC), N, stream_handle(dC.device))
    got = host(dC)
    # FP64 sums of K products: error ~ K u |A||B|
    tol = 1e-15 * K * np.abs(A).max() * np.abs(B).max() + 1e-14
    np.testing.assert_allclose(got, want, rtol=0, atol=tol)
    assert got.shape == (M, N)


@pytest.mark.parametrize("ta", [0, 1])
@pytest.mark.parametrize("tb", [0, 1])
@pytest.mark.parametrize("M,N,K,pad", [(258, 130, 38, 0), (300, 200, 150, 0), (512, 64, 1000, 0),
                                       (384, 192, 77, 1)])
def test_pipelined_gemm_matches_host(g, ta, tb, M, N, K, pad):
    """Sizes that take the pipelined kernel (M >= 128, N >= 64, even leading dimensions): ragged
    last tiles in M, N and K, and an odd K stored with a padded (even) leading dimension, whose
    last 16-byte chunk per row holds one element of the operand."""
    from gs_dft_b200._lib import lib, ptr, stream_handle
    rng = np.random.default_rng(M + 3 * N + 7 * K + 11 * ta + 13 * tb)
    A = rng.standard_normal((K, M) if ta else (M, K))
    B = rng.standard_normal((N, K) if tb else (K, N))
    C0 = rng.standard_normal((M, N))
    want = 0.75 * (A.T if ta else A) @ (B.T if tb else B) - 0.5 * C0

    def padded(X):
        # pad columns with NaN (never read) up to an even leading dimension, at least one column
        extra = (1 if X.shape[1] % 2 else 2) if pad else 0
        P = np.full((X.shape[0], X.shape[1] + extra), np.nan)
        P[:, :X.shape[1]] = X
        return P
    Ap, Bp = padded(A), padded(B)
    assert Ap.shape[1] % 2 == 0 and Bp.shape[1] % 2 == 0
    dA, dB, dC = dev(Ap), dev(Bp), dev(C0)
    lib.call("gsdft_dense_gemm", ta, tb, M, N, K, 0.75, ptr(dA), Ap.shape[1], ptr(dB), Bp.shape[1],
             -0.5, ptr(dC), N, stream_handle(dC.device))
    got = host(dC)
    tol = 1e-15 * K * np.abs(A).max() * np.abs(B).max() + 1e-14
    np.testing.assert_allclose(got, want, rtol=0, atol=tol)


def _spd(n, seed, cond=1e4):
    rng = np.random.default_rng(seed)
    Q, _ = np.linalg.qr(rng.standard_normal((n, n)))
    ev = np.geomspace(1.0, 1.0 / cond, n)
    V = (Q * ev) @ Q.T
    return 0.5 * (V + V.T)


@pytest.mark.parametrize("n", [1, 63, 64, 65, 300, 1000, 2051])
def test_cholesky_inverse_and_solve(g, n):
    from gs_dft_b200._lib import lib, ptr, stream_handle
    from gs_dft_b200.coulomb.ri import cholesky_inplace
    V = _spd(n, n)
    lam = 1e-8
    Lref = np.linalg.cholesky(V + lam * np.eye(n))
    dL = cholesky_inplace(dev(V), lam)
    L = host(dL)
    assert np.all(np.triu(L, 1) == 0.0)
    # a factor of a cond-1e4 matrix: entries agree to ~cond^(1/2) u
    np.testing.assert_allclose(L, Lref, rtol=0, atol=1e-12 * np.abs(Lref).max())
    st = stream_handle(dL.device)
    X = torch.empty((n, n), dtype=torch.float64, device="cuda")
    lib.call("gsdft_j_solve_inverse", ptr(dL), n, ptr(X), st)
    Xh = host(X)
    np.testing.assert_array_equal(np.triu(Xh, 1), np.tril(Xh, -1).T)
    np.testing.assert_allclose(np.tril(Xh) @ L, np.eye(n), rtol=0, atol=1e-10)
    rng = np.random.default_rng(n + 1)
    gam = rng.standard_normal(n)
    from scipy.linalg import cho_solve
    d_ref = cho_solve((L, True), gam)
    E_ref = 0.5 * gam @ d_ref
    gam_d = dev(gam)
    for name, args in (("gsdft_j_solve", (ptr(dL),)), ("gsdft_j_solve_inv", (ptr(X), ptr(dL))),
                       ("gsdft_j_solve_inv", (ptr(X), None))):
        d = torch.empty(n, dtype=torch.float64, device="cuda")
        E = torch.empty(1, dtype=torch.float64, device="cuda")
        wb = max(int(lib.gsdft_j_solve_inv_workspace_size(n)), 256)
        ws = torch.empty(wb, dtype=torch.uint8, device="cuda")
        lib.call(name, *args, ptr(gam_d), n, ptr(d), ptr(E), ptr(ws), wb, st)
        np.testing.assert_allclose(host(d), d_ref, rtol=0, atol=1e-10 * np.abs(d_ref).max())
        np.testing.assert_allclose(float(E), E_ref, rtol=1e-11)


def test_cholesky_rejects_an_indefinite_matrix(g):
    from gs_dft_b200.coulomb.ri import cholesky_inplace
    V = _spd(200, 5)
    V[150, 150] = -1.0
    with pytest.raises(ValueError, match="not positive definite"):
        cholesky_inplace(dev(V), 1e-8)


@pytest.mark.parametrize("M,n_occ,n_pairs", [(200, 65, 3000), (130, 128, 700), (64, 300, 1)])
def test_block_density_and_gradient(g, M, n_occ, n_pairs):
    """q and g_C as row-block DMMA tiles (SDDMM, SpMM) against NumPy on a random pair pattern:
    ragged last row block and orbital tile, row blocks without partners (splats 64..127 pair with
    nothing when M = 200), a single pair, representatives with i = j. q_a = w_a sum_o occ_o C_io
    C_jo; g_C[s] = occ (sum_{a: i_a = s} v_a C_{j_a} + sum_{a: j_a = s} v_a C_{i_a})."""
    from gs_dft_b200._lib import lib, ptr, stream_handle
    from gs_dft_b200.coulomb.engine import row_blocks
    rng = np.random.default_rng(M + n_occ)
    live = np.r_[np.arange(0, min(M, 64)), np.arange(128, M)]
    pairs = {(int(rng.choice(live)), int(rng.choice(live))) for _ in range(n_pairs)}
    pairs |= {(int(live[-1]), int(live[-1]))}
    pi = np.array(sorted(p[0] for p in pairs))
    pj = np.array([p[1] for p in sorted(pairs)])
    n = pi.size
    C = rng.standard_normal((M, n_occ))
    occ = rng.uniform(0.5, 2.0, n_occ)
    w = rng.choice([1.0, 2.0], n)
    v = rng.standard_normal(n)
    dpi = torch.as_tensor(pi, dtype=torch.int32, device="cuda")
    dpj = torch.as_tensor(pj, dtype=torch.int32, device="cuda")
    by_i, by_j = row_blocks(dpi, dpj, M), row_blocks(dpj, dpi, M)
    dC, docc, dw, dv = dev(C), dev(occ), dev(w), dev(v)
    st = stream_handle(dC.device)
    rec = torch.zeros((n, 18), dtype=torch.float64, device="cuda")
    rec[:, 17] = 3.0   # GSDFT_REC_KN
    buf = torch.empty(max(by_i.buf_len, by_j.buf_len), dtype=torch.float64, device="cuda")
    lib.call("gsdft_block_density", ptr(dC), ptr(docc), M, n_occ, by_i.n_blocks, ptr(by_i.boff),
             ptr(by_i.nj), ptr(by_i.joff), ptr(by_i.jidx), by_i.max_nj, ptr(by_i.cell), ptr(dw), n,
             ptr(buf), ptr(rec), st)
    q_ref = w * np.einsum("ao,o,ao->a", C[pi], occ, C[pj])
    scale = np.abs(C).max() ** 2 * occ.max() * n_occ * 1e-15 * 2
    np.testing.assert_allclose(host(rec[:, 16]), q_ref, rtol=0, atol=scale)
    np.testing.assert_allclose(host(rec[:, 15]), 3.0 * q_ref, rtol=0, atol=3 * scale)
    gC = dev(rng.standard_normal((M, n_occ)))   # overwritten (beta = 0 first)
    for k, bl in enumerate((by_i, by_j)):
        lib.call("gsdft_block_density_grad", ptr(dv), ptr(bl.cell), n, ptr(dC), ptr(docc), M,
                 n_occ, bl.n_blocks, ptr(bl.boff), ptr(bl.nj), ptr(bl.joff), ptr(bl.jidx),
                 bl.buf_len, ptr(buf), float(k), ptr(gC), st)
    want = np.zeros((M, n_occ))
    np.add.at(want, pi, v[:, None] * C[pj])
    np.add.at(want, pj, v[:, None] * C[pi])
    want *= occ
    tol = 1e-14 * (np.abs(v).sum() * np.abs(C).max() * occ.max() + 1)
    np.testing.assert_allclose(host(gC), want, rtol=0, atol=tol)
    assert not host(gC)[64:128].any()
