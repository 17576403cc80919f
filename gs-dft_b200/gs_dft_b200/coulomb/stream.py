"""Screened EXACT Hartree energy over the significant pairs, on the GPU.

Mirror of ``screened_coulomb_energy`` (gs_dft/coulomb/stream.py:294-320) with the Schur
(pair|pair) block ``full_eri_block_schur`` (:249-283): E_J = 1/2 sum_{a,b} P_a P_b (a|b) over the
listed pairs, P_a = valid_a sum_o occ_o C_io C_jo, with no density fitting. The O(n_pair^2)
integral sweep and every reduction run in ``gsdft_exact_j`` (one representative per thread per
transposed twin pair, which carries the same integral). This is the audit energy of
``evaluate()`` (gs_dft/ks/train.py:554) and the ``ScreenedExactCoulomb`` backend: the value only;
its gradient is not on the B200 path (the returned tensor does not require grad).
``bra_chunk`` is accepted for signature compatibility.
"""
from __future__ import annotations

import torch

from .._lib import REC_FIELDS, lib, ptr, stream_handle
from .engine import make_plan, splat_quantities

F64 = torch.float64


def screened_coulomb_energy(splats, C_orth, occ, pi, pj, valid=None, bra_chunk: int = 128,
                            merge_twins: bool = True, return_j: bool = False):
    """Exact E_J over the listed pairs (value). With ``return_j`` also J_a = sum_b (a|b) P_b per
    representative and the plan (representative -> list position in ``plan.rep_pos``)."""
    dev = splats.centers.device
    M = splats.n_basis
    n = int(pi.shape[0])
    w = (torch.ones(n, dtype=F64, device=dev) if valid is None else valid.to(F64).contiguous())
    pi32, pj32 = pi.to(torch.int32).contiguous(), pj.to(torch.int32).contiguous()
    plan = make_plan(pi32, pj32, w, M, 0, 1, merge_twins)
    nl = plan.n_rep
    q, ls, c = (splats.quat.detach().contiguous(), splats.log_scale.detach().contiguous(),
                splats.centers.detach().contiguous())
    C = C_orth.detach().to(F64).contiguous()
    oc = occ.detach().to(F64).contiguous()
    A9, N = splat_quantities(q, ls)
    rec = torch.empty((max(nl, 1), REC_FIELDS), dtype=F64, device=dev)
    s = stream_handle(dev)
    lib.call("gsdft_pair_prep", ptr(A9), ptr(c), ptr(N), M, ptr(pi32), ptr(pj32),
             ptr(plan.rep_pos), ptr(plan.rep_w), nl, ptr(C), ptr(oc), int(C.shape[1]), ptr(rec), s)
    ws_bytes = int(lib.gsdft_exact_j_workspace_size(nl))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    J = torch.empty(max(nl, 1), dtype=F64, device=dev)
    E = torch.empty(1, dtype=F64, device=dev)
    lib.call("gsdft_exact_j", ptr(rec), nl, ptr(J), ptr(E), ptr(ws), ws_bytes, s)
    if return_j:
        return E[0], J[:nl], plan
    return E[0]
