"""The no-allocation forward entry point, ``gsdft_j_forward_noalloc``, through the C ABI.

It serves callers that cannot allocate device memory (or hand in a workspace) when they call: its
scratch is a fixed 8 MiB device array inside the library. Checked against the workspace entry point
``gsdft_j_forward`` on the same pair records, on two calls in a row (the array keeps the first
call's contents, which must not leak into the second), within the parity tolerance of the suite,
relative 1e-10. Collected last so that a failure here stops a ``-x`` run only after every other test
has run; it sets up its own inputs, so it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

from conftest import load_golden

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gs_dft_b200 as g
    d = load_golden("ref_co2.npz")
    t = lambda a, dt=torch.float64: torch.as_tensor(np.ascontiguousarray(a), dtype=dt, device="cuda")
    s = g.Splat(t(d["quat"]), t(d["log_scale"]), t(d["centers"]))
    aux = g.init_product_aux(s)
    L = g.aux_cholesky(aux, float(d["lam"]))
    beta, R, KN = aux.quantities()
    R = R.contiguous()
    eng = g.RIJEngine(t(d["pad_pi"], torch.int32), t(d["pad_pj"], torch.int32), t(d["pad_v"]),
                      s.n_basis, d["C_occ"].shape[1], beta, R, KN, L)
    # existing entry point (caller workspace): pair prep + gsdft_j_forward
    ref = eng.forward_local(s.quat, s.log_scale, s.centers, t(d["C_occ"]), t(d["occ"])).clone()
    torch.cuda.synchronize()
    return g, eng, beta, R, KN, ref


def _noalloc(g, eng, beta, R, KN, out, n_aux=None):
    from gs_dft_b200._lib import lib, ptr, stream_handle
    n_aux = int(beta.shape[0]) if n_aux is None else n_aux
    lib.call("gsdft_j_forward_noalloc", ptr(eng.rec), eng.plan.n_rep, ptr(beta), ptr(R), ptr(KN),
             n_aux, ptr(out), stream_handle())


def test_noalloc_forward_matches_workspace_forward_twice(setup):
    g, eng, beta, R, KN, ref = setup
    want = ref.cpu().numpy()
    scale = np.abs(want).max()
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        _noalloc(g, eng, beta, R, KN, out)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-10, atol=1e-12 * scale)


def test_noalloc_rejects_more_aux_than_its_scratch(setup):
    from gs_dft_b200._lib import GsdftError
    g, eng, beta, R, KN, ref = setup
    out = torch.empty_like(ref)
    with pytest.raises(GsdftError) as e:
        _noalloc(g, eng, beta, R, KN, out, n_aux=(1 << 20) + 1)   # rejected before any launch
    assert e.value.code == 1 and "exceeds the fixed scratch" in str(e.value)
