"""Screened EXACT Hartree energy over the significant pairs, on the GPU.

Mirror of ``screened_coulomb_energy`` (gs_dft/coulomb/stream.py:294-320) with the Schur
(pair|pair) block ``full_eri_block_schur`` (:249-283): E_J = 1/2 sum_{a,b} P_a P_b (a|b) over the
listed pairs, P_a = valid_a sum_o occ_o C_io C_jo, with no density fitting. The O(n_pair^2)
integral sweep and every reduction run in ``gsdft_exact_j`` (one representative per thread per
transposed twin pair, which carries the same integral). This is the audit energy of
``evaluate()`` (gs_dft/ks/train.py:554) and the ``ScreenedExactCoulomb`` backend. Differentiable in
the splat parameters and ``C_orth`` through torch autograd: the backward is ``gsdft_exact_j_vjp``
(a second O(n_pair^2) sweep, the closed-form derivative of the same node sum, where the reference
differentiates its streamed block with a checkpointed custom VJP, stream.py:144-189) followed by the
same chain as the density-fitted energy. ``bra_chunk`` is accepted for signature compatibility.
"""
from __future__ import annotations

import torch

from .engine import RIJEngine

F64 = torch.float64


class _ScreenedExactEnergy(torch.autograd.Function):
    """Exact E_J as a function of (quat, log_scale, centers, C_occ); pairs frozen."""

    @staticmethod
    def forward(ctx, quat, log_scale, centers, C_occ, occ, eng):
        q, ls, c = quat.detach().contiguous(), log_scale.detach().contiguous(), centers.detach().contiguous()
        C, oc = C_occ.detach().to(F64).contiguous(), occ.detach().to(F64).contiguous()
        E = eng.forward_local(q, ls, c, C, oc)
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
            ctx.token = eng.last_forward
        eng.backward_local(c, C, oc, g_E=gE)
        g_quat, g_log = eng.chart(q, ls)
        g_C = eng.g_C[:, :eng.n_occ].clone()
        return g_quat.clone(), g_log.clone(), eng.gmu.clone(), g_C, None, None


def exact_engine(splats, C_orth, pi, pj, valid=None, merge_twins: bool = True,
                 block: str = "schur"):
    """The engine of the exact energy over the listed pairs (plan, records, buffers)."""
    dev = splats.centers.device
    n = int(pi.shape[0])
    w = (torch.ones(n, dtype=F64, device=dev) if valid is None else valid.to(F64).contiguous())
    return RIJEngine(pi.to(torch.int32).contiguous(), pj.to(torch.int32).contiguous(), w,
                     splats.n_basis, int(C_orth.shape[1]), merge_twins=merge_twins, exact=True,
                     exact_rule=block)


def screened_coulomb_energy(splats, C_orth, occ, pi, pj, valid=None, bra_chunk: int = 128,
                            merge_twins: bool = True, return_j: bool = False,
                            block: str = "schur"):
    """Exact E_J over the listed pairs. ``block`` picks the (pair|pair) quadrature: "schur" (the
    reference's default, the 20-node rule of full_eri_block_schur) or "fused" (the 32-node
    Boys-scaled rule of full_eri_block_fused, stream.py:323-458). With ``return_j`` also
    J_a = sum_b (a|b) P_b per representative and the plan (representative -> list position in
    ``plan.rep_pos``)."""
    eng = exact_engine(splats, C_orth, pi, pj, valid, merge_twins, block)
    E = _ScreenedExactEnergy.apply(splats.quat, splats.log_scale, splats.centers, C_orth, occ, eng)
    if return_j:
        return E, eng.Jx[:eng.plan.n_rep].clone(), eng.plan
    return E
