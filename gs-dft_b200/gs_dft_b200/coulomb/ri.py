"""Screened RI-J: the reference's function surface, on the B200 kernels.

Mirror of gs_dft/coulomb/ri.py: ``aux_quantities`` (:238-240), ``aux_metric`` (:267-275),
``shift_diag`` / ``aux_cholesky`` (:243-264), ``df_coulomb_gamma_screened`` (:436-469),
``df_coulomb_solve`` (:472-482), ``df_coulomb_energy_screened`` (:485-494). Same names, argument
meaning and return values. ``df_coulomb_energy_screened`` is differentiable (torch autograd) in the
splat parameters and ``C_occ``, with the aux, pair list and factor frozen — what the reference's
``jax.value_and_grad`` of the trainer differentiates (gs_dft/ks/train.py:367-382).

``chunk`` and ``skip_pad`` are accepted for signature compatibility: the device path never forms a
(N_aux, chunk) block, and always skips zero-weight (padding) pairs, which contribute exactly zero.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _check
from .._lib import lib, ptr, stream_handle

from .engine import RIJEngine

F64 = torch.float64


def aux_quantities(aux):
    """(beta, R, KN) of the isotropic aux."""
    return aux.quantities()


def aux_metric(aux, omega=None) -> torch.Tensor:
    """V_PQ = (P|Q), exact s-s Coulomb with F0 from erf, (N_aux, N_aux) row-major; with ``omega``
    the long-range (P|erf(omega r)/r|Q) (gs_dft/coulomb/ri.py:267-275)."""
    beta, R, KN = aux.quantities()
    n = int(beta.shape[0])
    V = torch.empty((n, n), dtype=F64, device=beta.device)
    if omega:
        lib.call("gsdft_aux_metric_lr", ptr(beta), ptr(R.contiguous()), ptr(KN), n, float(omega),
                 ptr(V), stream_handle(beta.device))
    else:
        lib.call("gsdft_aux_metric", ptr(beta), ptr(R.contiguous()), ptr(KN), n, ptr(V),
                 stream_handle(beta.device))
    return V


def shift_diag(V: torch.Tensor, lam: float) -> torch.Tensor:
    """V + lam I by adding to the diagonal (no dense identity)."""
    out = V.clone()
    out.diagonal().add_(lam)
    return out


def cholesky_inplace(V: torch.Tensor, lam: float) -> torch.Tensor:
    """V <- lower Cholesky factor of V + lam I (row-major), in place."""
    n = int(V.shape[0])
    ws_bytes = lib.gsdft_aux_cholesky_workspace_size(n)
    if ws_bytes == 0:
        raise RuntimeError("gsdft_aux_cholesky_workspace_size failed: "
                           + lib.gsdft_last_error_string().decode())
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=V.device)
    try:
        lib.call("gsdft_aux_cholesky", ptr(V), n, float(lam), ptr(ws), ws_bytes,
                 stream_handle(V.device))
    except RuntimeError as exc:
        if getattr(exc, "code", None) == 4:
            raise ValueError(str(exc)) from exc
        raise
    return V


def aux_cholesky(aux, lam: float, omega=None) -> torch.Tensor:
    """Lower Cholesky factor of (V + lam I) (the long-range metric with ``omega``); V is factored
    in its own buffer (gs_dft/coulomb/ri.py:259-264)."""
    return cholesky_inplace(aux_metric(aux, omega), lam)


def _pairs_w(pi, pj, valid):
    n = int(pi.shape[0])
    w = (torch.ones(n, dtype=F64, device=pi.device) if valid is None
         else valid.to(F64).contiguous())
    return pi.to(torch.int32).contiguous(), pj.to(torch.int32).contiguous(), w


def _engine(splats, C_occ, aux, pi, pj, valid, L):
    beta, R, KN = aux.quantities()
    pi, pj, w = _pairs_w(pi, pj, valid)
    # one-shot calls: substitution solve, no O(n_aux^3) inverse
    return RIJEngine(pi, pj, w, splats.n_basis, int(C_occ.shape[1]), beta, R.contiguous(), KN, L,
                     inverse_solve=False)


def df_coulomb_gamma_screened(splats, C_occ, occ, aux, pi, pj, chunk=2048, valid=None,
                              skip_pad=False):
    """gamma_P = sum_a (P|a) q_a over the listed pairs (q_a = valid_a sum_o occ_o C_io C_jo)."""
    eng = _engine(splats, C_occ, aux, pi, pj, valid, L=None)
    g = eng.forward_local(splats.quat.detach().contiguous(), splats.log_scale.detach().contiguous(),
                          splats.centers.detach().contiguous(),
                          C_occ.detach().to(F64).contiguous(),
                          occ.detach().to(F64).contiguous())
    return g.clone()


def df_coulomb_solve(gamma, aux, lam=1e-8, cholV=None):
    """E_J^DF = 1/2 gamma^T (V + lam I)^-1 gamma; with ``cholV`` (the lower factor) one pair of
    triangular solves, otherwise the metric is built and factored first."""
    L = cholV if cholV is not None else aux_cholesky(aux, lam)
    n = int(gamma.shape[0])
    _check.f64(L, "cholV", (n, n))
    gamma = _check.f64(gamma.detach().to(F64).contiguous(), "gamma", (n,))
    d = torch.empty_like(gamma)
    E = torch.empty(1, dtype=F64, device=gamma.device)
    lib.call("gsdft_j_solve", ptr(L), ptr(gamma), n, ptr(d), ptr(E), None, 0,
             stream_handle(gamma.device))
    return E[0]


class _ScreenedDFEnergy(torch.autograd.Function):
    """E_J as a function of (quat, log_scale, centers, C_occ); aux, pairs and factor frozen."""

    @staticmethod
    def forward(ctx, quat, log_scale, centers, C_occ, occ, eng):
        q, ls, c = quat.detach().contiguous(), log_scale.detach().contiguous(), centers.detach().contiguous()
        C, oc = C_occ.detach().to(F64).contiguous(), occ.detach().to(F64).contiguous()
        eng.forward_local(q, ls, c, C, oc)
        E, _ = eng.solve()
        ctx.eng, ctx.token = eng, eng.last_forward
        ctx.save_for_backward(q, ls, c, C, oc)
        return E[0].clone()

    @staticmethod
    def backward(ctx, gE):
        q, ls, c, C, oc = ctx.saved_tensors
        eng = ctx.eng
        gE = gE.detach().to(F64).reshape(1).contiguous()
        if eng.last_forward is not ctx.token:   # another forward used the engine since
            eng.forward_local(q, ls, c, C, oc)
            eng.solve()
            ctx.token = eng.last_forward
        eng.backward_local(c, C, oc, g_E=gE)
        g_quat, g_log = eng.chart(q, ls)
        g_C = eng.g_C[:, :eng.n_occ].clone()
        return g_quat.clone(), g_log.clone(), eng.gmu.clone(), g_C, None, None


def df_coulomb_energy_screened(splats, C_occ, occ, aux, pi, pj, lam=1e-8, chunk=2048, valid=None,
                               cholV=None, skip_pad=False):
    """E_J^DF over the listed (significant) pairs; differentiable in the splat parameters and
    ``C_occ`` through torch autograd."""
    L = cholV if cholV is not None else aux_cholesky(aux, lam)
    eng = _engine(splats, C_occ, aux, pi, pj, valid, L)
    return _ScreenedDFEnergy.apply(splats.quat, splats.log_scale, splats.centers, C_occ, occ, eng)
