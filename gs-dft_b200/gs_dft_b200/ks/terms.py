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
    """Frozen pair-product RI-J (+ RI-K for hybrids) over the significant pairs only.

    ``energy(basis, C_orth, P, occ, state) -> (E_J, E_K)`` like the reference
    (gs_dft/ks/terms.py:236-256): E_K from ``df_exchange_energy_screened`` on the same pairs and
    aux (the reference's aux_K is the same product basis, gs_dft/ks/energy.py:468) when
    ``hf_coeff != 0``, else 0. ``energy_lr`` is the unscaled long-range exchange
    E_K[erf(omega r)/r] when ``hf_coeff_lr != 0`` (gs_dft/ks/terms.py:258-265), else 0: the builder
    adds hf_coeff E_K + hf_coeff_lr E_K^lr.
    """

    def __init__(self, hf_coeff: float = 0.0, lam: float = 1e-8, chunk: int = 2048,
                 scales: tuple = (1.0,), diagonal: bool = True, skip_pad: bool = False,
                 hf_coeff_lr: float = 0.0, omega: float = 0.0):
        if hf_coeff_lr != 0.0 and not omega > 0.0:
            raise ValueError("range-separated exchange (hf_coeff_lr != 0) needs omega > 0")
        self.hf_coeff = float(hf_coeff)
        self.hf_coeff_lr, self.omega = float(hf_coeff_lr), float(omega)
        self.lam, self.chunk = float(lam), int(chunk)
        self.scales, self.diagonal = tuple(scales), bool(diagonal)
        self.skip_pad = bool(skip_pad)

    @classmethod
    def from_spec(cls, spec: DFSpec, skip_pad: bool = False, hf_coeff: float = 0.0,
                  hf_coeff_lr: float = 0.0, omega: float = 0.0):
        return cls(hf_coeff=hf_coeff, lam=spec.lam, chunk=spec.chunk, scales=spec.scales,
                   diagonal=spec.diagonal, skip_pad=skip_pad, hf_coeff_lr=hf_coeff_lr,
                   omega=omega)

    def energy_lr(self, basis, C_orth, P, occ, state):
        """Unscaled long-range exchange E_K[erf(omega r)/r] on the same pairs and aux, with the
        attenuated metric's factor (built once per state); 0 without range separation."""
        if self.hf_coeff_lr == 0.0:
            return torch.zeros((), dtype=torch.float64, device=basis.centers.device)
        from ..coulomb.exchange import _ScreenedDFExchange
        keng = state.k_engine_for(basis, C_orth, omega=self.omega, lam=self.lam)
        return _ScreenedDFExchange.apply(basis.quat, basis.log_scale, basis.centers, C_orth, keng)

    def energy(self, basis, C_orth, P, occ, state):
        from ..coulomb.ri import _ScreenedDFEnergy
        eng = state.engine_for(basis, C_orth)
        e_j = _ScreenedDFEnergy.apply(basis.quat, basis.log_scale, basis.centers, C_orth,
                                      occ, eng)
        if self.hf_coeff == 0.0:
            return e_j, torch.zeros((), dtype=e_j.dtype, device=e_j.device)
        from ..coulomb.exchange import _ScreenedDFExchange
        keng = state.k_engine_for(basis, C_orth)
        e_k = _ScreenedDFExchange.apply(basis.quat, basis.log_scale, basis.centers, C_orth, keng)
        return e_j, e_k


class ScreenedExactCoulomb:
    """Exact streamed ERI over the significant pairs (DF-free), PBE-class only: the reference's
    ``ScreenedExactCoulomb`` (gs_dft/ks/terms.py:195-205). ``energy(basis, C_orth, P, occ, state)
    -> (E_J, 0)``, differentiable in the splats and ``C_orth``; hybrids are rejected as in the
    reference (there is no screened exact K)."""

    def __init__(self, chunk: int = 128, hf_coeff: float = 0.0):
        if hf_coeff != 0.0:
            raise ValueError("ScreenedExactCoulomb is PBE-class only (no screened exact K)")
        self.chunk = int(chunk)
        self.hf_coeff = 0.0

    def energy(self, basis, C_orth, P, occ, state):
        from ..coulomb.stream import screened_coulomb_energy
        pi, pj, valid = state.pairs
        e_j = screened_coulomb_energy(basis, C_orth, occ, pi, pj, valid=valid,
                                      bra_chunk=self.chunk)
        return e_j, torch.zeros((), dtype=e_j.dtype, device=e_j.device)
