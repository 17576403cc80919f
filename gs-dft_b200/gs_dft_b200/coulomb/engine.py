"""Device-resident RI-J engine: one pair list, one frozen aux basis, repeated J-builds.

Holds every buffer the per-step path needs (pair plan, pair records, reverse-pass sums, gradients,
workspace), allocated once per refresh, so a step allocates nothing. A step is

    splat quantities -> pair prep (A_hat, P, KN, eigenframe, q) -> gamma (fused 3-centre contraction)
    -> [allreduce gamma] -> d, E_J (metric solve) -> reverse pass over (pair x aux) -> pair chain
    -> per-splat reductions -> chart reverse -> [allreduce gradients]

which is the single-device screened DF step of the reference (gs_dft/coulomb/ri.py:436-494 under
jax.value_and_grad, gs_dft/ks/train.py:367-382) with the gradient written out.

With ``atoms`` the engine also evaluates the screened nuclear attraction on the same pair list,
E_ne = sum_a q_a V_a (gs_dft/screening/pairs.py:348-370, 409-440, as SplatKS uses it with a
screened pair list, gs_dft/ks/energy.py:326-328): its reverse-pass sums are added to the RI-J ones
before the shared chain, so one backward pass gives the gradient of E_J + E_ne. With ``beta=None``
the engine carries E_ne alone.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from .. import _check
from .._lib import (REC_FIELDS, SIDE_FIELDS, SOLVE_INV_MAX, VJP_FIELDS, XC_FIELDS, lib, ptr,
                    stream_handle)

F64 = torch.float64


def _i64():
    return ctypes.c_int64(0)


@dataclass
class PairPlan:
    """Refresh-time plan of a pair list: the representatives this device evaluates (a contiguous
    slice of all of them) and their groupings by pi and by pj.

    A representative is a live entry (w != 0); with ``merge_twins`` a live (i,j), i < j, whose
    transpose (j,i) is also live stands for both — the two carry the same integral — with the
    summed weight, and J is written to both list positions."""

    n: int              # list length
    n_rep_total: int    # representatives over the whole list
    r0: int             # this slice: representatives [r0, r1)
    r1: int
    rep_pos: torch.Tensor
    rep_w: torch.Tensor
    rep_twin: torch.Tensor
    order_i: torch.Tensor
    seg_i: torch.Tensor
    partner_i: torch.Tensor
    order_j: torch.Tensor
    seg_j: torch.Tensor
    partner_j: torch.Tensor

    @property
    def n_rep(self) -> int:
        return self.r1 - self.r0


def partition_bounds(n_rep: int, world: int, cost=None):
    """Rank boundaries [r_0 = 0, ..., r_world = n_rep] of the representatives: equal counts, or with
    ``cost`` (int64 per representative, on any device) contiguous ranges of equal estimated cost
    (r_k = the number of leading representatives whose cumulative cost is <= k/world of the total).
    Integer arithmetic throughout, so every rank computes the same cut."""
    if cost is None or world <= 1 or n_rep == 0:
        return [n_rep * k // world for k in range(world + 1)]
    cum = torch.cumsum(cost[:n_rep].to(torch.int64), 0)
    total = int(cum[-1])
    targets = torch.tensor([total * k // world for k in range(world + 1)], dtype=torch.int64,
                           device=cum.device)
    b = torch.searchsorted(cum, targets, right=True).tolist()
    b[0], b[-1] = 0, n_rep
    return [int(x) for x in b]


def make_plan(pi, pj, w, M: int, rank: int = 0, world: int = 1, merge_twins: bool = True,
              cost_fn=None):
    """The plan of this rank's slice. ``cost_fn(rep_pos, n_rep)`` (optional) returns the int64
    estimated cost of every representative; the slices then balance cost instead of count."""
    _check.pair_indices(pi, pj, M)
    _check.f64(w, "pair weights", (int(pi.shape[0]),))
    dev = pi.device
    n = int(pi.shape[0])
    pos = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
    rw = torch.empty(max(n, 1), dtype=torch.float64, device=dev)
    tw = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
    ws_bytes = lib.gsdft_pair_plan_workspace_size(n, M)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    nr = _i64()
    lib.call("gsdft_pair_reps", ptr(pi), ptr(pj), ptr(w), n, M, int(bool(merge_twins)), ptr(pos),
             ptr(rw), ptr(tw), ctypes.byref(nr), ptr(ws), ws_bytes, stream_handle(dev))
    n_rep = int(nr.value)
    cost = cost_fn(pos, n_rep) if (cost_fn is not None and world > 1 and n_rep > 0) else None
    bounds = partition_bounds(n_rep, world, cost)
    r0, r1 = bounds[rank], bounds[rank + 1]
    pos, rw, tw = pos[r0:max(r1, r0 + 1)], rw[r0:max(r1, r0 + 1)], tw[r0:max(r1, r0 + 1)]
    k = r1 - r0
    oi = torch.empty(max(k, 1), dtype=torch.int32, device=dev)
    oj = torch.empty(max(k, 1), dtype=torch.int32, device=dev)
    qi = torch.empty(max(k, 1), dtype=torch.int32, device=dev)
    qj = torch.empty(max(k, 1), dtype=torch.int32, device=dev)
    si = torch.empty(M + 1, dtype=torch.int64, device=dev)
    sj = torch.empty(M + 1, dtype=torch.int64, device=dev)
    gb = lib.gsdft_pair_groups_workspace_size(k, M)
    gws = torch.empty(gb, dtype=torch.uint8, device=dev)
    lib.call("gsdft_pair_groups", ptr(pi), ptr(pj), ptr(pos), k, M, ptr(oi), ptr(si), ptr(qi),
             ptr(oj), ptr(sj), ptr(qj), ptr(gws), gb, stream_handle(dev))
    return PairPlan(n=n, n_rep_total=n_rep, r0=r0, r1=r1, rep_pos=pos, rep_w=rw, rep_twin=tw,
                    order_i=oi, seg_i=si, partner_i=qi, order_j=oj, seg_j=sj, partner_j=qj)


# Quadrature rules of the exact (pair|pair) Hartree term (GSDFT_EXACT_SCHUR20 / _FUSED32).
EXACT_RULES = {"schur": 0, "fused": 1}

# Orbital counts from which q and g_C run as dense DMMA tiles over 64-splat row blocks
# (gsdft_block_density / gsdft_block_density_grad); below it, per-pair kernels.
BLOCK_MIN_OCC = 64


@dataclass
class RowBlocks:
    """Row blocks of 64 consecutive splats over this device's representatives: block b's sorted
    partner list J_b (the splats its rows pair with), and each representative's cell in the blocks'
    dense tiles (row = its own splat, column = its partner's place in J_b)."""

    n_blocks: int
    boff: torch.Tensor   # int64 (n_blocks): tile offsets
    nj: torch.Tensor     # int32 (n_blocks)
    joff: torch.Tensor   # int64 (n_blocks)
    jidx: torch.Tensor   # int32: concatenated partner lists
    cell: torch.Tensor   # int64 (n_rep)
    max_nj: int
    buf_len: int


def row_blocks(rows, partners, M: int) -> RowBlocks:
    """The block structure of representatives (rows[a], partners[a]) (int tensors on the device):
    exact integer sorting (torch.unique), identical on every call."""
    dev = rows.device
    nb = (M + 63) // 64
    r = rows.to(torch.int64)
    key = (r // 64) * M + partners.to(torch.int64)
    if key.numel() == 0:
        z64 = torch.zeros(nb, dtype=torch.int64, device=dev)
        return RowBlocks(nb, z64, z64.to(torch.int32), z64, torch.zeros(1, dtype=torch.int32,
                         device=dev), torch.zeros(1, dtype=torch.int64, device=dev), 0, 0)
    uniq, inv = torch.unique(key, sorted=True, return_inverse=True)
    blk_u = uniq // M
    nj = torch.bincount(blk_u, minlength=nb)
    joff = torch.cumsum(nj, 0) - nj
    rows_b = torch.clamp(M - 64 * torch.arange(nb, device=dev, dtype=torch.int64), max=64)
    sizes = rows_b * nj
    boff = torch.cumsum(sizes, 0) - sizes
    b = r // 64
    col = inv - joff[b]
    cell = boff[b] + (r - 64 * b) * nj[b] + col
    return RowBlocks(nb, boff.contiguous(), nj.to(torch.int32).contiguous(), joff.contiguous(),
                     (uniq % M).to(torch.int32).contiguous(), cell.contiguous(),
                     int(nj.max()), int(sizes.sum()))


def check_step_inputs(M, n_occ, quat, log_scale, centers, C_occ=None, occ=None):
    """The per-step parameters as the kernels read them: contiguous float64 CUDA tensors of the
    engine's sizes (metadata only)."""
    args = [(quat, "quat", (M, 4)), (log_scale, "log_scale", (M, 3)), (centers, "centers", (M, 3))]
    if n_occ > 0:
        args.append((C_occ, "C_occ", (M, n_occ)))
        if occ is not None:
            args.append((occ, "occ", (n_occ,)))
    for t, name, shape in args:          # dtype, shape and layout of all first, then the device
        _check.tensor(t, name, torch.float64, shape, cuda=False)
    for t, name, _ in args:
        _check.tensor(t, name, torch.float64, None, contiguous=False)


def splat_quantities(quat, log_scale):
    """(A9 (M,9), N (M)) on the device."""
    M = int(quat.shape[0])
    A9 = torch.empty((M, 9), dtype=F64, device=quat.device)
    N = torch.empty(M, dtype=F64, device=quat.device)
    lib.call("gsdft_splat_quantities", ptr(quat), ptr(log_scale), M, ptr(A9), ptr(N),
             stream_handle(quat.device))
    return A9, N


class RIJEngine:
    """Repeated screened RI-J builds on a fixed (pair list, aux, factor).

    Args:
        pi, pj: int32 pair indices (device); w: float64 weights (0 = padding; 1 ordered; 2 unique).
        M: number of splats; n_occ: occupied orbitals.
        beta, R, KN: the aux quantities; L: lower Cholesky factor of V + lam I (row-major).
            ``beta=None``: no RI-J term (an engine for the nuclear attraction alone).
        rank, world: this device evaluates representatives [n_rep*rank//world, n_rep*(rank+1)//world).
        merge_twins: evaluate each (i,j)/(j,i) pair of a live transposed twin once (same integral).
        inverse_solve: form the packed inverse factor once (O(n_aux^3), n_aux <= 65536) so each
            step's solve is two parallel mat-vecs; for engines that run many steps. Off: per-step
            blocked triangular substitution.
        atoms: optional (n_atoms, 4) float64 device tensor of nuclei (x, y, z, Z) in Bohr: adds the
            screened nuclear attraction E_ne on the same pairs.
        balance: optional (quat, log_scale, centers) of the splats at refresh: with world > 1 the
            ranks' slices then carry equal estimated integral cost (``gsdft_rep_cost``: node
            screening makes distant pairs cheaper), instead of equal representative counts.
        exact: the Hartree term is the exact (pair|pair) E_J over the representatives
            (``gsdft_exact_j`` / ``gsdft_exact_j_vjp``, O(n_rep^2)) instead of the density fit;
            no aux, one device. ``exact_rule``: "schur" (the 20-node rule of
            full_eri_block_schur) or "fused" (the 32-node Boys-scaled rule of
            full_eri_block_fused).
    """

    def __init__(self, pi, pj, w, M, n_occ, beta=None, R=None, KN=None, L=None, rank=0, world=1,
                 merge_twins=True, inverse_solve=True, atoms=None, balance=None, exact=False,
                 exact_rule="schur"):
        self.device = pi.device
        self.M, self.n_occ = int(M), int(n_occ)
        self.pi = pi.to(torch.int32).contiguous()
        self.pj = pj.to(torch.int32).contiguous()
        self.w = w.to(F64).contiguous()
        if beta is not None:
            n_aux = int(beta.shape[0])
            beta, KN = _check.f64(beta, "beta", (n_aux,)), _check.f64(KN, "KN", (n_aux,))
            R = _check.f64(R.contiguous(), "R", (n_aux, 3))
            if L is not None:
                _check.f64(L, "L", (n_aux, n_aux))
        self.beta, self.R, self.KN, self.L = beta, R, KN, L
        self.rij = beta is not None
        self.exact = bool(exact)
        if exact_rule not in EXACT_RULES:
            raise ValueError(f"exact_rule must be one of {sorted(EXACT_RULES)}")
        self.exact_rule = EXACT_RULES[exact_rule]
        self.n_aux = int(beta.shape[0]) if self.rij else 0
        if self.exact and (self.rij or world != 1):
            raise ValueError("the exact Hartree term replaces the density fit (no aux) and runs "
                             "on one device")
        if not self.rij and not self.exact and atoms is None:
            raise ValueError("RIJEngine needs the aux quantities (beta, R, KN), exact=True, "
                             "atoms, or a Hartree term and atoms")
        cost_fn = None
        if balance is not None and world > 1 and self.rij:
            cost_fn = self._cost_fn(*balance)
        self.plan = make_plan(self.pi, self.pj, self.w, self.M, rank, world, merge_twins, cost_fn)
        dev, nl, n = self.device, self.plan.n_rep, self.plan.n
        e = lambda *s: torch.empty(s, dtype=F64, device=dev)
        self.A9, self.N = e(self.M, 9), e(self.M)
        self.rec = e(max(nl, 1), REC_FIELDS)
        self.sums = e(max(nl, 1), VJP_FIELDS)
        self.side = e(max(nl, 1), SIDE_FIELDS)
        self.J = e(max(n, 1))
        self.jw = e(max(nl, 1))
        self.gamma, self.d, self.E = e(self.n_aux), e(self.n_aux), e(1)
        self.gA6, self.gmu, self.gN = e(self.M, 6), e(self.M, 3), e(self.M)
        self.g_quat, self.g_log = e(self.M, 4), e(self.M, 3)
        self.g_C = e(self.M, max(self.n_occ, 1))
        self.atoms, self.n_atoms = None, 0
        if atoms is not None:
            self.atoms = atoms.to(device=dev, dtype=F64).contiguous()
            if self.atoms.dim() != 2 or self.atoms.shape[1] != 4:
                raise ValueError("atoms must be (n_atoms, 4): x, y, z, Z")
            self.n_atoms = int(self.atoms.shape[0])
            self.E_ne, self.V = e(1), e(max(n, 1))
        sizes = [256]
        if self.rij:
            sizes += [lib.gsdft_j_forward_workspace_size(nl, self.n_aux),
                      lib.gsdft_j_vjp_workspace_size(nl, self.n_aux),
                      lib.gsdft_j_solve_workspace_size(self.n_aux),
                      lib.gsdft_j_solve_inv_workspace_size(self.n_aux)]
        if self.atoms is not None:
            sizes.append(lib.gsdft_vne_workspace_size(nl))
        self.xc = self.Jx = None
        if self.exact:
            self.xc, self.Jx = e(max(nl, 1), XC_FIELDS), e(max(nl, 1))
            sizes += [lib.gsdft_exact_j_workspace_size(nl), lib.gsdft_exact_j_vjp_workspace_size(nl)]
        self.ws_bytes = max(sizes)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)
        # many orbitals: q and g_C as dense tiles over row blocks (by pi and by pj)
        self.blocks = None
        if self.n_occ >= BLOCK_MIN_OCC and nl > 0:
            rp = self.plan.rep_pos[:nl].to(torch.int64)
            ri, rj = self.pi[rp], self.pj[rp]
            self.blocks = (row_blocks(ri, rj, self.M), row_blocks(rj, ri, self.M))
            self.block_buf = [e(max(bl.buf_len, 1)) for bl in self.blocks]
        # the packed inverse factor [L^-1 lower | L^-T strict upper] once per refresh: the per-step
        # solve is then two row-parallel mat-vecs over one n_aux^2 matrix
        self.Linv = None
        if inverse_solve and L is not None and self.n_aux <= SOLVE_INV_MAX:
            self.Linv = e(self.n_aux, self.n_aux)
            lib.call("gsdft_j_solve_inverse", ptr(self.L), self.n_aux, ptr(self.Linv),
                     stream_handle(dev))
        # Optional CUDA-event brackets around the two integral kernels (recorded on the current
        # stream, the one the kernels are launched on): {"forward": [(start, end)], "vjp": [...]}.
        self.timing = False
        self.events = {"forward": [], "vjp": [], "vne": []}
        # token of the forward whose pair records, gamma and d the buffers hold (a backward after
        # another forward on this engine must re-run its own forward first)
        self.last_forward = None

    def _cost_fn(self, quat, log_scale, centers, n_sample: int = 256):
        """Estimated cost per representative from the splats' geometry and a sample of the aux."""
        def fn(rep_pos, n_rep):
            check_step_inputs(self.M, 0, quat, log_scale, centers)
            A9, _ = splat_quantities(quat, log_scale)
            cost = torch.empty(n_rep, dtype=torch.int64, device=self.device)
            lib.call("gsdft_rep_cost", ptr(A9), ptr(centers), self.M, ptr(self.pi), ptr(self.pj),
                     ptr(rep_pos), n_rep, ptr(self.beta), ptr(self.R), self.n_aux,
                     min(n_sample, self.n_aux), ptr(cost), stream_handle(self.device))
            return cost
        return fn

    def _bracket(self, name):
        if not self.timing:
            return None
        st = torch.cuda.current_stream(self.device)
        # external: inside a CUDA-graph capture these become event-record nodes that time replays
        a = torch.cuda.Event(enable_timing=True, external=True)
        b = torch.cuda.Event(enable_timing=True, external=True)
        a.record(st)
        self.events[name].append((a, b))
        return b

    def kernel_ms(self, name):
        """Mean event time (ms) of the bracketed launches of ``name`` recorded so far."""
        ev = self.events[name]
        return sum(a.elapsed_time(b) for a, b in ev) / max(len(ev), 1)

    # -- stages -----------------------------------------------------------------------------------
    def prepare(self, quat, log_scale, centers, C_occ, occ):
        """Splat quantities and the pair records (A_hat eigenframe, P, KN, q) of this device's
        representatives."""
        check_step_inputs(self.M, self.n_occ, quat, log_scale, centers, C_occ, occ)
        s = stream_handle(self.device)
        lib.call("gsdft_splat_quantities", ptr(quat), ptr(log_scale), self.M, ptr(self.A9),
                 ptr(self.N), s)
        blocks = self.blocks is not None
        lib.call("gsdft_pair_prep", ptr(self.A9), ptr(centers), ptr(self.N), self.M, ptr(self.pi),
                 ptr(self.pj), ptr(self.plan.rep_pos), ptr(self.plan.rep_w), self.plan.n_rep,
                 None if blocks else ptr(C_occ), None if blocks else ptr(occ),
                 0 if blocks else self.n_occ, ptr(self.rec), s)
        if blocks:
            bl = self.blocks[0]
            lib.call("gsdft_block_density", ptr(C_occ), ptr(occ), self.M, self.n_occ, bl.n_blocks,
                     ptr(bl.boff), ptr(bl.nj), ptr(bl.joff), ptr(bl.jidx), bl.max_nj, ptr(bl.cell),
                     ptr(self.plan.rep_w), self.plan.n_rep, ptr(self.block_buf[0]), ptr(self.rec),
                     s)

    def external(self, sums=False, add=False, g_E=None):
        """This device's E_ne = sum_a q_a V_a and V per list entry (after ``prepare``); with
        ``sums`` also the reverse-pass sums of g_E * E_ne, written or (``add``) added."""
        end = self._bracket("vne")
        lib.call("gsdft_vne", ptr(self.rec), self.plan.n_rep, ptr(self.atoms), self.n_atoms,
                 ptr(g_E), ptr(self.plan.rep_pos), ptr(self.plan.rep_twin), self.plan.n,
                 ptr(self.V), ptr(self.E_ne), ptr(self.sums) if sums else None, int(bool(add)),
                 ptr(self.ws), self.ws_bytes, stream_handle(self.device))
        if end is not None:
            end.record(torch.cuda.current_stream(self.device))
        return self.E_ne

    def forward_local(self, quat, log_scale, centers, C_occ, occ):
        """Splat quantities, pair prep and this device's gamma (before any allreduce)."""
        s = stream_handle(self.device)
        nl = self.plan.n_rep
        self.prepare(quat, log_scale, centers, C_occ, occ)
        self.last_forward = object()
        if self.exact:
            lib.call("gsdft_exact_j", ptr(self.rec), nl, self.exact_rule, ptr(self.Jx),
                     ptr(self.E), ptr(self.ws), self.ws_bytes, s)
            return self.E
        if not self.rij:
            return None
        end = self._bracket("forward")
        lib.call("gsdft_j_forward", ptr(self.rec), nl, ptr(self.beta), ptr(self.R), ptr(self.KN),
                 self.n_aux, ptr(self.gamma), ptr(self.ws), self.ws_bytes, s)
        if end is not None:
            end.record(torch.cuda.current_stream(self.device))
        return self.gamma

    def solve(self):
        """d = (L L^T)^-1 gamma, E = 1/2 gamma.d (replicated tail)."""
        if self.Linv is not None:
            lib.call("gsdft_j_solve_inv", ptr(self.Linv), ptr(self.L), ptr(self.gamma), self.n_aux,
                     ptr(self.d), ptr(self.E), ptr(self.ws), self.ws_bytes,
                     stream_handle(self.device))
        else:
            lib.call("gsdft_j_solve", ptr(self.L), ptr(self.gamma), self.n_aux, ptr(self.d),
                     ptr(self.E), ptr(self.ws), self.ws_bytes, stream_handle(self.device))
        return self.E, self.d

    def backward_local(self, centers, C_occ, occ, g_E=None, g_E_ne=None):
        """This device's pre-chart splat cotangents (gA6, gmu, gN), J = dE/dq per list entry and
        g_C, of g_E E_J + g_E_ne E_ne (the terms the engine carries; device scalars, None = 1).
        With atoms this also evaluates E_ne."""
        s = stream_handle(self.device)
        nl = self.plan.n_rep
        if self.rij:
            end = self._bracket("vjp")
            lib.call("gsdft_j_vjp", ptr(self.rec), nl, ptr(self.beta), ptr(self.R), ptr(self.KN),
                     ptr(self.d), ptr(g_E), self.n_aux, ptr(self.sums), ptr(self.ws),
                     self.ws_bytes, s)
            if end is not None:
                end.record(torch.cuda.current_stream(self.device))
        if self.exact:
            lib.call("gsdft_exact_j_vjp", ptr(self.rec), nl, self.exact_rule, ptr(g_E),
                     ptr(self.xc), ptr(self.ws), self.ws_bytes, s)
        if self.atoms is not None:
            self.external(sums=True, add=self.rij, g_E=g_E_ne)
        has_sums = self.rij or self.atoms is not None
        lib.call("gsdft_pair_chain", ptr(self.A9), ptr(centers), ptr(self.N), self.M,
                 ptr(self.pi), ptr(self.pj), ptr(self.plan.rep_pos), ptr(self.plan.rep_twin),
                 ptr(self.plan.rep_w), nl, self.plan.n, ptr(self.rec),
                 ptr(self.sums) if has_sums else None, ptr(self.xc) if self.exact else None,
                 ptr(self.side), ptr(self.J), ptr(self.jw), s)
        lib.call("gsdft_splat_reduce", ptr(self.side), ptr(self.plan.order_i),
                 ptr(self.plan.seg_i), ptr(self.plan.order_j), ptr(self.plan.seg_j), nl, self.M,
                 ptr(self.gA6), ptr(self.gmu), ptr(self.gN), s)
        if self.blocks is not None:
            # g_C = occ (T_i C_J + T_j C_I): the J w values in each grouping's tiles, two block SpMMs
            for k, bl in enumerate(self.blocks):
                lib.call("gsdft_block_density_grad", ptr(self.jw), ptr(bl.cell), nl, ptr(C_occ),
                         ptr(occ), self.M, self.n_occ, bl.n_blocks, ptr(bl.boff), ptr(bl.nj),
                         ptr(bl.joff), ptr(bl.jidx), bl.buf_len, ptr(self.block_buf[k]),
                         float(k), ptr(self.g_C), s)
        elif self.n_occ > 0:
            lib.call("gsdft_density_grad", ptr(self.plan.order_i), ptr(self.plan.seg_i),
                     ptr(self.plan.partner_i), ptr(self.plan.order_j), ptr(self.plan.seg_j),
                     ptr(self.plan.partner_j), ptr(self.jw), nl, self.M, ptr(C_occ), ptr(occ),
                     self.n_occ, ptr(self.g_C), s)
        return self.gA6, self.gmu, self.gN, self.g_C

    def chart(self, quat, log_scale):
        lib.call("gsdft_chart_vjp", ptr(quat), ptr(log_scale), ptr(self.gA6), ptr(self.gN),
                 self.M, ptr(self.g_quat), ptr(self.g_log), stream_handle(self.device))
        return self.g_quat, self.g_log

    # -- whole step -------------------------------------------------------------------------------
    def step(self, quat, log_scale, centers, C_occ, occ, grad=True, g_E=None, g_E_ne=None):
        """Single-device J-build (and E_ne with atoms) + gradient of their sum. Returns a dict of
        device tensors (views of the engine's buffers: copy them before the next step if they
        must persist)."""
        self.forward_local(quat, log_scale, centers, C_occ, occ)
        out = {}
        if self.rij:
            self.solve()
            out.update(E=self.E, gamma=self.gamma, d=self.d)
        elif self.exact:
            out.update(E=self.E)
        if grad:
            self.backward_local(centers, C_occ, occ, g_E, g_E_ne)
            self.chart(quat, log_scale)
            out.update(J=self.J, g_quat=self.g_quat, g_log_scale=self.g_log, g_centers=self.gmu,
                       g_C=self.g_C[:, :self.n_occ], gA6=self.gA6, gN=self.gN)
        elif self.atoms is not None:
            self.external()
        if self.atoms is not None:
            out.update(E_ne=self.E_ne, V=self.V[:self.plan.n])
        return out


class StepGraph:
    """A whole J-build + gradient step captured once in a CUDA graph and replayed.

    ``step_fn`` launches every kernel (the library's own; never a collective) on the current
    stream and returns its outputs. Its input tensors are
    read at their captured addresses: copy new parameters into them before ``replay()``. The
    outputs are the captured buffers, overwritten by every replay."""

    def __init__(self, step_fn, warmup: int = 2):
        if warmup:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(warmup):
                    step_fn()
            torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        n0 = lib.gsdft_kernel_launches()
        with torch.cuda.graph(self.graph):
            self.out = step_fn()
        # the library's own kernels in the graph (each replay launches exactly these)
        self.launches = int(lib.gsdft_kernel_launches() - n0)

    def replay(self, phases=None):
        self.graph.replay()
        return self.out


def check_device_status(clear=True):
    """Raise if a kernel's bounded wait ran out since the last check."""
    st = ctypes.c_int(0)
    lib.call("gsdft_device_status", ctypes.byref(st), 1 if clear else 0)
    if st.value:
        raise RuntimeError(f"gs_dft_b200 device status {st.value}: a bulk-copy wait timed out")
