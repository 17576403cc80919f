"""Isotropic auxiliary splats and the frozen product aux.

Mirror of gs_dft/basis/isotropic.py:22-39 (``IsotropicSplat``) and :81-116 (``init_product_aux``);
the arithmetic runs in ``gsdft_product_aux`` / ``gsdft_aux_quantities`` (CUDA).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from .. import _check
from .._lib import lib, ptr, stream_handle
from .spectral import Splat, full_quantities

F64 = torch.float64


@dataclass
class IsotropicSplat:
    """Isotropic Gaussians g(r) = N exp(-alpha |r - centre|^2), N = (2 alpha / pi)^(3/4)."""

    log_alpha: torch.Tensor
    centers: torch.Tensor

    def __post_init__(self):
        n = int(self.log_alpha.shape[0]) if isinstance(self.log_alpha, torch.Tensor) else -1
        self.log_alpha = _check.f64(self.log_alpha, "log_alpha", (n,), contiguous=False).contiguous()
        self.centers = _check.f64(self.centers, "aux centers", (n, 3), contiguous=False).contiguous()

    @property
    def n_basis(self) -> int:
        return int(self.log_alpha.shape[0])

    def quantities(self):
        """(alpha, centers, norm) on the device (gs_dft/coulomb/ri.py:238-240)."""
        n = self.n_basis
        beta = torch.empty(n, dtype=F64, device=self.log_alpha.device)
        KN = torch.empty(n, dtype=F64, device=self.log_alpha.device)
        lib.call("gsdft_aux_quantities", ptr(self.log_alpha), n, ptr(beta), ptr(KN),
                 stream_handle(self.log_alpha.device))
        return beta, self.centers, KN

    @property
    def alpha(self) -> torch.Tensor:
        return self.quantities()[0]

    @property
    def norm(self) -> torch.Tensor:
        return self.quantities()[2]


def init_product_aux(basis: Splat, pi=None, pj=None, valid=None, *, scales=(1.0,),
                     diagonal_only=True) -> IsotropicSplat:
    """One isotropic aux per kept pair product at the product centre, alpha = det(A_i+A_j)^(1/3)*s
    for each scale s. ``diagonal_only`` (default) keeps the M self-products."""
    if not scales:
        raise ValueError("init_product_aux needs at least one scale")
    A9, mu, N = full_quantities(basis)
    M = basis.n_basis
    dev = mu.device
    if diagonal_only or pi is None:
        pi = pj = w = None
        n = M
    else:
        pi = pi.to(torch.int32).contiguous()
        pj = pj.to(torch.int32).contiguous()
        _check.pair_indices(pi, pj, M)
        n = int(pi.shape[0])
        w = (torch.ones(n, dtype=F64, device=dev) if valid is None
             else valid.to(F64).contiguous())
    ns = len(scales)
    log_alpha = torch.empty(n * ns, dtype=F64, device=dev)
    R = torch.empty((n * ns, 3), dtype=F64, device=dev)
    sc = (ctypes.c_double * ns)(*[float(s) for s in scales])
    lib.call("gsdft_product_aux", ptr(A9), ptr(mu), ptr(N), M, ptr(pi), ptr(pj), ptr(w), n, sc,
             ns, ptr(log_alpha), ptr(R), stream_handle(dev))
    return IsotropicSplat(log_alpha=log_alpha, centers=R)
