"""Screened nuclear attraction on the significant-pair list, on the GPU.

Mirror of gs_dft/screening/pairs.py:348-370 (``_full_nuclear_pairs``), :378-380
(``screened_nuclear_pairs``), :403-406 (``density_pairs``) and :409-440
(``screened_external_energy``): V_ij = -N_iN_jK sum_A Z_A (2/sqrt(pi)) sum_t w_t pi^1.5
det(A_ij + t^2 I)^-1/2 exp(-t^2 d.A_ij (A_ij + t^2 I)^-1 d), d = P_ij - R_A, and
E_ext = sum_a valid_a P_a V_a. The integrals, their reverse pass and every reduction run in the
library (``gsdft_vne``, ``gsdft_density_pairs`` and the shared pair chain), deterministically.

``chunk`` and ``skip_pad`` are accepted for signature compatibility: the device kernel streams the
whole list in one launch and never evaluates zero-weight entries.
"""
from __future__ import annotations

import torch

from .._lib import lib, ptr, stream_handle
from .pairs import pair_weight

F64 = torch.float64


def atom_records(atom_coords, atom_charges, device=None) -> torch.Tensor:
    """(n_atoms, 4) float64 device tensor (x, y, z, Z): the nuclei as ``gsdft_vne`` reads them."""
    X = torch.as_tensor(atom_coords, dtype=F64, device=device)
    Z = torch.as_tensor(atom_charges, dtype=F64, device=X.device)
    if X.dim() != 2 or X.shape[1] != 3 or Z.shape != (X.shape[0],):
        raise ValueError("atom_coords must be (n_atoms, 3) and atom_charges (n_atoms,)")
    return torch.cat([X, Z[:, None]], dim=1).contiguous()


def _engine(splats, C_occ, pi, pj, valid, atoms, merge_twins=True):
    from ..coulomb.engine import RIJEngine
    n = int(pi.shape[0])
    w = (torch.ones(n, dtype=F64, device=pi.device) if valid is None
         else pair_weight(valid).contiguous())
    n_occ = 0 if C_occ is None else int(C_occ.shape[1])
    return RIJEngine(pi.to(torch.int32).contiguous(), pj.to(torch.int32).contiguous(), w,
                     splats.n_basis, n_occ, atoms=atoms, merge_twins=merge_twins)


def screened_nuclear_pairs(splats, pi, pj, atom_coords, atom_charges) -> torch.Tensor:
    """V_ij for every listed pair (padding entries included, as in the reference)."""
    atoms = atom_records(atom_coords, atom_charges, splats.centers.device)
    eng = _engine(splats, None, pi, pj, None, atoms, merge_twins=False)
    q, ls, c = (splats.quat.detach().contiguous(), splats.log_scale.detach().contiguous(),
                splats.centers.detach().contiguous())
    eng.prepare(q, ls, c, None, None)
    eng.external()
    return eng.V[:eng.plan.n].clone()


def density_pairs(C_orth, occ, pi, pj) -> torch.Tensor:
    """P_ij = sum_o occ_o C_io C_jo on the pair list, without forming the dense P."""
    n = int(pi.shape[0])
    C = C_orth.detach().to(F64).contiguous()
    oc = occ.detach().to(F64).contiguous()
    out = torch.empty(max(n, 1), dtype=F64, device=C.device)
    lib.call("gsdft_density_pairs", ptr(pi.to(torch.int32).contiguous()),
             ptr(pj.to(torch.int32).contiguous()), n, ptr(C), ptr(oc), int(C.shape[1]), ptr(out),
             stream_handle(C.device))
    return out[:n]


class _ScreenedExternalEnergy(torch.autograd.Function):
    """E_ext as a function of (quat, log_scale, centers, C_orth); pair list and nuclei frozen."""

    @staticmethod
    def forward(ctx, quat, log_scale, centers, C_orth, occ, eng):
        q, ls, c = quat.detach().contiguous(), log_scale.detach().contiguous(), centers.detach().contiguous()
        C, oc = C_orth.detach().to(F64).contiguous(), occ.detach().to(F64).contiguous()
        eng.prepare(q, ls, c, C, oc)
        E = eng.external()
        ctx.eng = eng
        ctx.save_for_backward(q, ls, c, C, oc)
        return E[0].clone()

    @staticmethod
    def backward(ctx, gE):
        q, ls, c, C, oc = ctx.saved_tensors
        eng = ctx.eng
        gE = gE.detach().to(F64).reshape(1).contiguous()
        eng.prepare(q, ls, c, C, oc)
        eng.backward_local(c, C, oc, g_E_ne=gE)
        g_quat, g_log = eng.chart(q, ls)
        g_C = eng.g_C[:, :eng.n_occ].clone()
        return g_quat.clone(), g_log.clone(), eng.gmu.clone(), g_C, None, None


def screened_external_energy(splats, C_orth, occ, pi, pj, atom_coords, atom_charges, valid=None,
                             chunk: int = 8192, skip_pad: bool = False):
    """E_external = sum_a valid_a P_a V_a over the listed pairs; differentiable in the splat
    parameters and ``C_orth`` through torch autograd (pairs and nuclei frozen)."""
    atoms = atom_records(atom_coords, atom_charges, splats.centers.device)
    eng = _engine(splats, C_orth, pi, pj, valid, atoms)
    return _ScreenedExternalEnergy.apply(splats.quat, splats.log_scale, splats.centers, C_orth,
                                         occ, eng)
