"""Refresh state and the Coulomb-only builder.

``SplatState`` / ``refresh`` mirror gs_dft/ks/energy.py:121-139 and :421-474 for the fields the
screened DF Coulomb needs (pairs, aux, cholV); the pad rule mirrors gs_dft/ks/train.py:356-359.
``CoulombKS`` carries the ``coulomb`` / ``screen`` / ``mesh`` arguments of ``SplatKS``
(gs_dft/ks/energy.py:166-173) and evaluates the Hartree term E_J of a model; ``ExternalKS`` is the
screened external term of the same ``SplatKS`` branch, E_external on the refresh state's pair list
(gs_dft/ks/energy.py:326-328). The rest of the Kohn-Sham energy (kinetic, XC) is outside this
library.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from ..basis.isotropic import IsotropicSplat, init_product_aux
from ..basis.spectral import Splat
from ..coulomb.engine import RIJEngine
from ..coulomb.ri import aux_cholesky
from ..screening.nuclear import _ScreenedExternalEnergy, atom_records
from ..screening.pairs import count_significant, neighbor_pairs, pair_weight, stripe_pairs
from .terms import DFSpec, Pairlist, ScreenedProductDFCoulomb


def pad_rule(n0: int, pad: float, G: int) -> int:
    """pad_to = ceil(pad * n0 / G) * G (gs_dft/ks/train.py:356-359)."""
    return -(-int(pad * n0) // G) * G


@dataclass
class SplatModel:
    """Trainable model: splats + MO coefficients + occupations (gs_dft/ks/energy.py:109-118)."""

    basis: Splat
    C: torch.Tensor
    occupations: torch.Tensor


@dataclass
class SplatState:
    """Refresh products: pair list, frozen product aux, factor of V + lam I."""

    pairs: tuple | None = None
    aux: IsotropicSplat | None = None
    cholV: torch.Tensor | None = None
    _engine: RIJEngine | None = field(default=None, repr=False)
    _ext_engine: RIJEngine | None = field(default=None, repr=False)
    _k_engine: object | None = field(default=None, repr=False)
    _k_engines_lr: dict = field(default_factory=dict, repr=False)

    def engine_for(self, basis, C_occ) -> RIJEngine:
        """The device engine for this state's pairs/aux/factor (built once, reused per step)."""
        if self._engine is None:
            pi, pj, valid = self.pairs
            beta, R, KN = self.aux.quantities()
            self._engine = RIJEngine(pi.to(torch.int32).contiguous(), pj.to(torch.int32).contiguous(),
                                     pair_weight(valid).contiguous(), basis.n_basis,
                                     int(C_occ.shape[1]), beta, R.contiguous(), KN, self.cholV)
        return self._engine

    def k_engine_for(self, basis, C_occ, omega=None, lam=None):
        """The device engine of the screened RI-K term on this state's pairs/aux/factor; with
        ``omega`` the long-range one, whose attenuated metric is factored here (with ``lam``)
        once per state."""
        from ..coulomb.exchange import RIKEngine
        pi, pj, valid = self.pairs
        beta, R, KN = self.aux.quantities()
        if omega:
            eng = self._k_engines_lr.get(float(omega))
            if eng is None:
                from ..coulomb.ri import aux_cholesky
                L = aux_cholesky(self.aux, 1e-8 if lam is None else lam, omega=omega)
                eng = RIKEngine(pi, pj, valid, basis.n_basis, int(C_occ.shape[1]), beta, R, KN,
                                L, omega=omega)
                self._k_engines_lr[float(omega)] = eng
            return eng
        if self._k_engine is None:
            self._k_engine = RIKEngine(pi, pj, valid, basis.n_basis, int(C_occ.shape[1]), beta,
                                       R, KN, self.cholV)
        return self._k_engine

    def external_engine_for(self, basis, C_occ, atoms) -> RIJEngine:
        """The device engine of the screened external term on this state's pairs (built once)."""
        if self._ext_engine is None:
            pi, pj, valid = self.pairs
            self._ext_engine = RIJEngine(pi.to(torch.int32).contiguous(),
                                         pj.to(torch.int32).contiguous(),
                                         pair_weight(valid).contiguous(), basis.n_basis,
                                         int(C_occ.shape[1]), atoms=atoms)
        return self._ext_engine


def refresh(ks, basis: Splat, *, pad_to: int | None = None,
            like: SplatState | None = None) -> SplatState:
    """Rebuild the refresh products for the current splats (host cadence).

    ``like=previous_state`` inherits the previous pad so shapes stay constant.
    """
    if pad_to is None and like is not None and like.pairs is not None:
        pad_to = int(like.pairs[0].shape[0])
    screen: Pairlist = ks.screen
    pairs = neighbor_pairs(basis, eps=screen.eps, pad_to=pad_to, unique=screen.unique)
    G = int(getattr(ks, "n_devices", 1) or 1)
    if G > 1:
        pairs = stripe_pairs(*pairs, G)
    c: ScreenedProductDFCoulomb = ks.coulomb
    aux = init_product_aux(basis, scales=c.scales, diagonal_only=c.diagonal,
                           pi=pairs[0], pj=pairs[1], valid=pairs[2])
    cholV = aux_cholesky(aux, c.lam)
    return SplatState(pairs=pairs, aux=aux, cholV=cholV)


class CoulombKS:
    """The Hartree term of ``SplatKS(system, xc, grid=..., coulomb=df(), screen=pairlist())``:
    ``ks(model, state) -> E_J`` (differentiable in the model's splats and C)."""

    def __init__(self, *, coulomb: DFSpec | None = None, screen: Pairlist | None = None,
                 n_devices: int = 1, hf_coeff: float = 0.0, hf_coeff_lr: float = 0.0,
                 omega: float = 0.0):
        coulomb = coulomb or DFSpec()
        if not isinstance(coulomb, DFSpec):
            raise TypeError(f"coulomb must come from df(), got {coulomb!r}")
        if screen is None:
            raise ValueError("the B200 RI-J path is the screened path: pass screen=pairlist(...)")
        self.screen = screen
        self.coulomb = ScreenedProductDFCoulomb.from_spec(coulomb, skip_pad=screen.skip_pad,
                                                          hf_coeff=hf_coeff,
                                                          hf_coeff_lr=hf_coeff_lr, omega=omega)
        self.n_devices = int(n_devices)

    def initial_pad(self, basis: Splat) -> int:
        n0 = count_significant(basis, self.screen.eps, self.screen.unique)
        return pad_rule(n0, self.screen.pad, self.n_devices)

    def __call__(self, model: SplatModel, state: SplatState):
        if state is None or state.pairs is None or state.aux is None:
            raise ValueError("coulomb=df() needs the refresh state: see refresh(ks, basis).")
        e_j, _ = self.coulomb.energy(model.basis, model.C, None, model.occupations, state)
        return e_j

    def energy(self, model: SplatModel, state: SplatState):
        """(E_J, E_K) as ``ScreenedProductDFCoulomb.energy`` returns them (E_K = 0 unless the
        builder was given ``hf_coeff != 0``)."""
        if state is None or state.pairs is None or state.aux is None:
            raise ValueError("coulomb=df() needs the refresh state: see refresh(ks, basis).")
        return self.coulomb.energy(model.basis, model.C, None, model.occupations, state)

    def energy_lr(self, model: SplatModel, state: SplatState):
        """The unscaled long-range exchange E_K[erf(omega r)/r] (0 unless the builder was given
        ``hf_coeff_lr != 0``); the total exchange is hf_coeff E_K + hf_coeff_lr E_K^lr."""
        if state is None or state.pairs is None or state.aux is None:
            raise ValueError("coulomb=df() needs the refresh state: see refresh(ks, basis).")
        return self.coulomb.energy_lr(model.basis, model.C, None, model.occupations, state)


class ExternalKS:
    """The screened external term of ``SplatKS(..., screen=pairlist())``:
    ``ext(model, state) -> E_external = sum_ij P_ij V_ij`` over the refresh state's pair list
    (gs_dft/ks/energy.py:326-328 with gs_dft/screening/pairs.py:409-440), differentiable in the
    model's splats and C. The coefficients are used as given: pass orthonormalised orbitals, as the
    reference does (its C_orth)."""

    def __init__(self, atom_coords, atom_charges):
        self.atom_coords = atom_coords
        self.atom_charges = atom_charges

    def __call__(self, model: SplatModel, state: SplatState):
        if state is None or state.pairs is None:
            raise ValueError("the screened external term needs the refresh state's pair list")
        basis = model.basis
        atoms = atom_records(self.atom_coords, self.atom_charges, basis.centers.device)
        eng = state.external_engine_for(basis, model.C, atoms)
        return _ScreenedExternalEnergy.apply(basis.quat, basis.log_scale, basis.centers, model.C,
                                             model.occupations, eng)
