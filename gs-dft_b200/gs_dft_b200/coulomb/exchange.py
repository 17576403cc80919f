"""Screened density-fitted exchange (RI-K) over the significant pairs, on the GPU.

Mirror of ``_exchange_M_streamed_screened`` / ``df_exchange_energy_screened``
(gs_dft/coulomb/ri.py:497-544): D[P,o,o'] = sum_{live (i,k)} (P|ik) C_io C_ko',
M = D D^T (over o, o'), E_K = -tr((V + lam I)^-1 M), differentiable in the splat parameters and
the orbitals (aux, pairs and factor frozen, as for E_J). The integral block, the orbital products,
every reduction, the reverse pass and the contractions (the library's DMMA GEMMs, with the packed
inverse factor for L^-1 and L^-T) are the library's kernels (``gsdft_k_forward`` /
``gsdft_k_backward``), then the same pair chain, per-splat reductions and chart reverse as RI-J.

The orbital products are streamed over chunks of ``occ_chunk`` orbitals, as the reference streams
its M-build: only n_rep x occ_chunk x n_occ products are held at a time. Differences from the
reference, by design: the integral block over the whole list is kept resident for the step
(8 n_rep n_aux bytes) instead of being recomputed per orbital chunk, and D's n_aux x n_occ^2 entries
are held (the reference keeps only M); lists whose workspace exceeds ``max_bytes`` raise; the solve
uses the Cholesky factor's inverse, formed once per engine (the reference LU-solves V + lam I).
``chunk`` (the reference's pair-chunk knob) is accepted and unused. ``omega`` gives the long-range
exchange E_K[erf(omega r)/r]: the 12-node segment rule on [0, omega] for the 3-centre integrals and
the attenuated metric's factor (gs_dft/coulomb/ri.py:149,232-235,267-275).
"""
from __future__ import annotations

import torch

from .._lib import (NODE_TABLE_DOUBLES, REC_FIELDS, SIDE_FIELDS, SOLVE_INV_MAX, VJP_FIELDS, lib,
                    ptr, stream_handle)
from .. import _check
from .engine import check_step_inputs, make_plan

F64 = torch.float64
MAX_WORKSPACE_BYTES = 64 << 30
CHUNK_BYTES = 8 << 30        # the orbital-product chunk chosen when occ_chunk is None
LR_NODES = 12                # nodes of the long-range segment rule (gs_dft/coulomb/ri.py:232)


def auto_occ_chunk(n_rep: int, n_occ: int, budget: int = CHUNK_BYTES) -> int:
    """Orbitals per chunk so that the n_rep x chunk x n_occ products fit ``budget`` bytes."""
    per = 8 * max(n_rep, 1) * n_occ
    return int(max(1, min(n_occ, budget // per)))


class RIKEngine:
    """Repeated screened RI-K evaluations on a fixed (ordered 0/1 pair list, aux, factor).

    Args:
        pi, pj: int32 pair indices (device); valid: bool mask or 0/1 weights (0 = padding).
        M: number of splats; n_occ: orbitals (columns of C).
        beta, R, KN: aux quantities; L: lower Cholesky factor of V + lam I (row-major); with
            ``omega`` the factor of the long-range metric (``aux_cholesky(aux, lam, omega)``).
        merge_twins: evaluate each live (i,j)/(j,i) twin once (same integral).
        omega: range separation: the long-range exchange E_K[erf(omega r)/r].
        occ_chunk: orbitals per product chunk (None: as many as fit ``CHUNK_BYTES``).
    """

    def __init__(self, pi, pj, valid, M, n_occ, beta, R, KN, L, merge_twins=True,
                 max_bytes=MAX_WORKSPACE_BYTES, omega=None, occ_chunk=None):
        w = valid.to(F64).contiguous()
        if bool(((w != 0) & (w != 1)).any()):
            raise ValueError("screened RI-K takes an ordered pair list with a 0/1 mask, as the "
                             "reference's valid & occupied mask does (not unique-pair weights)")
        if n_occ < 1:
            raise ValueError("RI-K needs at least one orbital")
        self.device = pi.device
        self.M, self.n_occ = int(M), int(n_occ)
        self.pi, self.pj = pi.to(torch.int32).contiguous(), pj.to(torch.int32).contiguous()
        self.n_aux = int(beta.shape[0])
        self.beta = _check.f64(beta, "beta", (self.n_aux,))
        self.R = _check.f64(R.contiguous(), "R", (self.n_aux, 3))
        self.KN = _check.f64(KN, "KN", (self.n_aux,))
        self.L = _check.f64(L, "L", (self.n_aux, self.n_aux))
        self.plan = make_plan(self.pi, self.pj, w, self.M, 0, 1, merge_twins)
        # packed inverse factor (L^-1 in its lower triangle), formed once: the solves of every step
        # are then two triangular products on the tensor cores
        if self.n_aux > SOLVE_INV_MAX:
            raise ValueError(f"screened RI-K supports n_aux <= {SOLVE_INV_MAX}")
        self.Linv = torch.empty((self.n_aux, self.n_aux), dtype=F64, device=pi.device)
        lib.call("gsdft_j_solve_inverse", ptr(self.L), self.n_aux, ptr(self.Linv),
                 stream_handle(pi.device))
        dev, nl, n = self.device, self.plan.n_rep, self.plan.n
        self.omega = None if not omega else float(omega)
        self.nodes, self.n_nodes = None, 0
        if self.omega is not None:
            if self.omega <= 0.0:
                raise ValueError("omega must be positive")
            self.nodes = torch.empty(NODE_TABLE_DOUBLES, dtype=F64, device=dev)
            self.n_nodes = LR_NODES
            lib.call("gsdft_lr_node_table", self.omega, LR_NODES, ptr(self.nodes),
                     stream_handle(dev))
        self.occ_chunk = (auto_occ_chunk(nl, self.n_occ) if occ_chunk is None
                          else int(max(1, min(int(occ_chunk), self.n_occ))))
        self.ws_bytes = int(lib.gsdft_k_workspace_size(nl, self.n_aux, self.n_occ, self.occ_chunk))
        if self.ws_bytes > max_bytes:
            raise ValueError(f"screened RI-K needs {self.ws_bytes / 2**30:.1f} GiB of workspace for "
                             f"{nl} pairs x {self.n_aux} aux (integral block) with {self.occ_chunk}"
                             f"-orbital chunks of {self.n_occ} orbitals "
                             f"(limit {max_bytes / 2**30:.0f} GiB)")
        e = lambda *s: torch.empty(s, dtype=F64, device=dev)
        self.A9, self.N = e(self.M, 9), e(self.M)
        self.rec, self.rec_K = e(max(nl, 1), REC_FIELDS), e(max(nl, 1), REC_FIELDS)
        self.sums, self.side = e(max(nl, 1), VJP_FIELDS), e(max(nl, 1), SIDE_FIELDS)
        self.J, self.jw = e(max(n, 1)), e(max(nl, 1))
        self.Z, self.E = e(self.n_aux, self.n_occ * self.n_occ), e(1)
        self.gA6, self.gmu, self.gN = e(self.M, 6), e(self.M, 3), e(self.M)
        self.g_quat, self.g_log = e(self.M, 4), e(self.M, 3)
        self.g_C = e(self.M, self.n_occ)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.last_forward = None      # token of the forward whose products the workspace holds

    def forward(self, quat, log_scale, centers, C):
        """E_K (device scalar); keeps what the backward needs in the engine's workspace."""
        check_step_inputs(self.M, self.n_occ, quat, log_scale, centers, C)
        s = stream_handle(self.device)
        nl = self.plan.n_rep
        lib.call("gsdft_splat_quantities", ptr(quat), ptr(log_scale), self.M, ptr(self.A9),
                 ptr(self.N), s)
        lib.call("gsdft_pair_prep", ptr(self.A9), ptr(centers), ptr(self.N), self.M, ptr(self.pi),
                 ptr(self.pj), ptr(self.plan.rep_pos), ptr(self.plan.rep_w), nl, None, None, 0,
                 ptr(self.rec), s)
        lib.call("gsdft_k_forward", ptr(self.rec), ptr(self.pi), ptr(self.pj),
                 ptr(self.plan.rep_pos), ptr(self.plan.rep_twin), nl, ptr(self.beta), ptr(self.R),
                 ptr(self.KN), self.n_aux, ptr(self.nodes), self.n_nodes, ptr(self.Linv), ptr(C),
                 self.n_occ, self.occ_chunk, ptr(self.Z), ptr(self.E), ptr(self.ws), self.ws_bytes,
                 s)
        self.last_forward = object()
        return self.E

    def backward(self, quat, log_scale, centers, C, g_E=None):
        """Gradient of g_E E_K after ``forward`` on the same inputs: (g_quat, g_log_scale,
        g_centers, g_C)."""
        s = stream_handle(self.device)
        nl, p = self.plan.n_rep, self.plan
        lib.call("gsdft_k_backward", ptr(self.rec), ptr(self.pi), ptr(self.pj), ptr(p.rep_pos),
                 ptr(p.rep_twin), nl, ptr(self.beta), ptr(self.R), ptr(self.KN), self.n_aux,
                 ptr(self.nodes), self.n_nodes, ptr(self.Linv), ptr(C), self.n_occ,
                 self.occ_chunk, ptr(self.Z), ptr(g_E), ptr(p.order_i),
                 ptr(p.seg_i), ptr(p.partner_i), ptr(p.order_j), ptr(p.seg_j), ptr(p.partner_j),
                 self.M, ptr(self.sums), ptr(self.g_C), ptr(self.ws), self.ws_bytes, s)
        lib.call("gsdft_k_unit_q", ptr(self.rec), nl, ptr(self.rec_K), s)
        lib.call("gsdft_pair_chain", ptr(self.A9), ptr(centers), ptr(self.N), self.M,
                 ptr(self.pi), ptr(self.pj), ptr(p.rep_pos), ptr(p.rep_twin), ptr(p.rep_w), nl,
                 p.n, ptr(self.rec_K), ptr(self.sums), None, ptr(self.side), ptr(self.J),
                 ptr(self.jw), s)
        lib.call("gsdft_splat_reduce", ptr(self.side), ptr(p.order_i), ptr(p.seg_i),
                 ptr(p.order_j), ptr(p.seg_j), nl, self.M, ptr(self.gA6), ptr(self.gmu),
                 ptr(self.gN), s)
        lib.call("gsdft_chart_vjp", ptr(quat), ptr(log_scale), ptr(self.gA6), ptr(self.gN),
                 self.M, ptr(self.g_quat), ptr(self.g_log), s)
        # gsdft_k_backward overwrote the workspace's integral block with its weights: a further
        # backward must re-run the forward first
        self.last_forward = None
        return self.g_quat, self.g_log, self.gmu, self.g_C

    def step(self, quat, log_scale, centers, C, grad=True, g_E=None):
        out = dict(E_K=self.forward(quat, log_scale, centers, C))
        if grad:
            gq, gl, gc, gC = self.backward(quat, log_scale, centers, C, g_E)
            out.update(g_quat=gq, g_log_scale=gl, g_centers=gc, g_C=gC)
        return out


class _ScreenedDFExchange(torch.autograd.Function):
    """E_K as a function of (quat, log_scale, centers, C_occ); aux, pairs and factor frozen."""

    @staticmethod
    def forward(ctx, quat, log_scale, centers, C_occ, eng):
        q, ls, c = quat.detach().contiguous(), log_scale.detach().contiguous(), centers.detach().contiguous()
        C = C_occ.detach().to(F64).contiguous()
        E = eng.forward(q, ls, c, C)
        ctx.eng, ctx.token = eng, eng.last_forward
        ctx.save_for_backward(q, ls, c, C)
        return E[0].clone()

    @staticmethod
    def backward(ctx, gE):
        q, ls, c, C = ctx.saved_tensors
        eng = ctx.eng
        gE = gE.detach().to(F64).reshape(1).contiguous()
        if eng.last_forward is not ctx.token:   # another forward used the workspace since
            eng.forward(q, ls, c, C)
        g_quat, g_log, g_cen, g_C = eng.backward(q, ls, c, C, gE)
        return g_quat.clone(), g_log.clone(), g_cen.clone(), g_C.clone(), None


def df_exchange_energy_screened(splats, C_occ, aux, pi, pj, lam=1e-8, chunk=2048, valid=None,
                                occ_chunk=16, omega=None):
    """RI-K E_K over the significant bra-pairs (ordered list, 0/1 ``valid``); differentiable in the
    splat parameters and ``C_occ`` through torch autograd. ``omega``: the long-range exchange
    E_K[erf(omega r)/r] (attenuated metric and 3-centre integrals). ``occ_chunk``: orbitals per
    streamed product chunk."""
    from .ri import aux_cholesky
    L = aux_cholesky(aux, lam, omega=omega)
    beta, R, KN = aux.quantities()
    n = int(pi.shape[0])
    v = (torch.ones(n, dtype=torch.bool, device=pi.device) if valid is None else valid)
    eng = RIKEngine(pi, pj, v, splats.n_basis, int(C_occ.shape[1]), beta, R, KN, L, omega=omega,
                    occ_chunk=occ_chunk)
    return _ScreenedDFExchange.apply(splats.quat, splats.log_scale, splats.centers, C_occ, eng)
