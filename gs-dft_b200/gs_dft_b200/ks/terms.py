"""Strategy values for the screened DF Coulomb, mirror of gs_dft/ks/terms.py:48-139 (specs and
factories) and :236-256 (``ScreenedProductDFCoulomb``)."""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class DFSpec:
    """Frozen pair-product density-fitting backend (see :func:`df`)."""

    scales: tuple = (1.0,)
    diagonal: bool = True
    lam: float = 1e-8
    chunk: int = 2048


SCREEN_PAD = 2.0
"""Default pair-list pad multiplier (gs_dft/ks/terms.py:68)."""


@dataclass(frozen=True)
class Pairlist:
    """Significant-overlap pair screening (see :func:`pairlist`)."""

    eps: float = 1e-7
    pad: float = SCREEN_PAD
    unique: bool = False
    skip_pad: bool = False


def df(*, scales: tuple = (1.0,), diagonal: bool = True, lam: float = 1e-8,
       chunk: int = 2048) -> DFSpec:
    """Density-fitted Coulomb on the frozen self-constructing pair-product aux (RI-J)."""
    if not scales:
        raise ValueError("df(scales=...) needs at least one exponent scale.")
    return DFSpec(scales=tuple(float(s) for s in scales), diagonal=bool(diagonal),
                  lam=float(lam), chunk=int(chunk))


def pairlist(eps: float = 1e-7, *, pad: float = SCREEN_PAD, unique: bool = False,
             skip_pad: bool = False) -> Pairlist:
    """Screen the Coulomb work to the significant-overlap pairs (|S_ij| > eps; eps <= 0 keeps
    every ordered pair)."""
    return Pairlist(eps=float(eps), pad=float(pad), unique=bool(unique), skip_pad=bool(skip_pad))


class ScreenedProductDFCoulomb:
    """Frozen pair-product RI-J over the significant pairs only.

    ``energy(basis, C_orth, P, occ, state) -> (E_J, E_K)`` like the reference. Exact exchange
    (RI-K, for hybrids) is not on the B200 path: ``hf_coeff != 0`` raises.
    """

    def __init__(self, hf_coeff: float = 0.0, lam: float = 1e-8, chunk: int = 2048,
                 scales: tuple = (1.0,), diagonal: bool = True, skip_pad: bool = False):
        if hf_coeff != 0.0:
            raise NotImplementedError("screened RI-K (hybrid exchange) is not on the B200 path")
        self.hf_coeff = 0.0
        self.lam, self.chunk = float(lam), int(chunk)
        self.scales, self.diagonal = tuple(scales), bool(diagonal)
        self.skip_pad = bool(skip_pad)

    @classmethod
    def from_spec(cls, spec: DFSpec, skip_pad: bool = False):
        return cls(lam=spec.lam, chunk=spec.chunk, scales=spec.scales, diagonal=spec.diagonal,
                   skip_pad=skip_pad)

    def energy(self, basis, C_orth, P, occ, state):
        from ..coulomb.ri import _ScreenedDFEnergy
        eng = state.engine_for(basis, C_orth)
        e_j = _ScreenedDFEnergy.apply(basis.quat, basis.log_scale, basis.centers, C_orth,
                                      occ, eng)
        return e_j, torch.zeros((), dtype=e_j.dtype, device=e_j.device)
