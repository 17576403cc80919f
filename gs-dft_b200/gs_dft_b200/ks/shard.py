"""Multi-GPU RI-J: one process per GPU, the pair list partitioned across ranks, NCCL allreduce of
the aux fit vector and of the splat cotangents.

Replaces the DF branch of gs_dft/ks/shard.py:169-245 (``shard_map`` over mesh axis "g" with
``lax.psum`` of gamma, replicated solve, gradient psum through the shard_map transpose) and the
per-step replica ``pmean`` of gs_dft/ks/shard.py:44-65, which is not needed because every rank
computes bit-identical replicated values.

Partition: every rank builds the same refresh-time plan of the whole list (live entries, with each
(i,j)/(j,i) twin merged into one representative) and evaluates a contiguous slice of the
representatives. Every representative has N_aux integrals, but node screening makes distant
(aux, pair) combinations cheaper, so with ``balance`` (the splats at refresh) the slices carry equal
estimated cost (``gsdft_rep_cost``), else equal counts; padding costs nothing, and contiguity keeps
each rank's per-splat scatter local. The reference instead deals the padded list round-robin (``stripe_pairs``) because
its padding is appended; striped lists are accepted too (a stripe only reorders the same pairs).

With ``atoms`` each rank also evaluates the screened nuclear attraction on its slice (the
reference's ``screened_external_energy`` on the local stripe, psum'd: gs_dft/ks/shard.py:223,
267); its partial E_ne travels in one extra slot of the packed gradient allreduce, so the step
keeps two collectives.

Failure detection (the reference configures distributed-init timeouts, gs_dft/ks/shard.py:90-93):
with ``heartbeat`` (seconds), every step starts with a host-side liveness check of all ranks over a
gloo side group (``monitored_barrier``, which names the ranks that did not arrive), so a rank that
failed or left between steps is reported as ``PeerFailure`` before any kernel or collective of the
step is launched; an error raised by a collective itself (the process group's timeout) is reported
as ``PeerFailure`` too. A rank leaves only between steps, never with its kernels or collectives in
flight.
"""
from __future__ import annotations

from datetime import timedelta

import torch

from ..coulomb.engine import RIJEngine
from ..screening.pairs import pair_weight, stripe_pairs

__all__ = ["PeerFailure", "ShardedRIJ", "stripe_pairs"]


class PeerFailure(RuntimeError):
    """Another rank did not take part in a step: it failed, exited, or hung before the step's
    collectives. Raised on the host before this rank launches the step's kernels (liveness check)
    or when a collective ends with an error (the process group's timeout)."""


class ShardedRIJ:
    """This rank's share of a sharded J-build + gradient.

    ``group`` is a torch.distributed process group (NCCL on GPUs; gloo works for CPU-side tests of
    the host logic). All ranks take the same collective steps in the same order.
    """

    def __init__(self, pi, pj, valid, M, n_occ, beta, R, KN, L, rank: int, world: int,
                 group=None, engine_cls=RIJEngine, atoms=None, balance=None, inverse_solve=True,
                 heartbeat: float | None = None):
        self.rank, self.world, self.group = rank, world, group
        self.heartbeat = heartbeat
        self._hb_group = None
        if heartbeat is not None and world > 1:
            import torch.distributed as dist
            # monitored_barrier needs gloo: a side group for the liveness check on any backend
            self._hb_group = dist.new_group(backend="gloo")
        kw = {} if atoms is None else {"atoms": atoms}
        if balance is not None:
            kw["balance"] = balance
        if not inverse_solve:
            kw["inverse_solve"] = False
        self.engine = engine_cls(pi.contiguous(), pj.contiguous(), pair_weight(valid).contiguous(),
                                 M, n_occ, beta, R, KN, L, rank=rank, world=world, **kw)
        self.M, self.n_occ = int(M), int(n_occ)
        self.external = atoms is not None
        # [gA6 (6M) | gmu (3M) | gN (M) | g_C (M n_occ) | E_ne partial (1)]
        self.n_gc = self.M * max(self.n_occ, 1)
        self.packed = torch.empty(10 * self.M + self.n_gc + 1, dtype=torch.float64,
                                  device=pi.device)

    # The step in three parts around its two collectives, so that the compute parts can be
    # captured as CUDA graphs while the NCCL allreduces stay eager.
    def _forward(self, quat, log_scale, centers, C_occ, occ):
        return self.engine.forward_local(quat, log_scale, centers, C_occ, occ)

    def _middle(self, centers, C_occ, occ):
        eng = self.engine
        E, d = eng.solve()
        gA6, gmu, gN, gC = eng.backward_local(centers, C_occ, occ)
        M, p = self.M, self.packed
        p[:6 * M].copy_(gA6.reshape(-1))
        p[6 * M:9 * M].copy_(gmu.reshape(-1))
        p[9 * M:10 * M].copy_(gN)
        if self.n_occ:
            p[10 * M:10 * M + M * self.n_occ].copy_(gC[:, :self.n_occ].reshape(-1))
        if self.external:
            p[-1:].copy_(eng.E_ne)
        return E, d

    def _tail(self, quat, log_scale):
        eng, M, p = self.engine, self.M, self.packed
        eng.gA6.copy_(p[:6 * M].view(M, 6))
        eng.gmu.copy_(p[6 * M:9 * M].view(M, 3))
        eng.gN.copy_(p[9 * M:10 * M])
        return eng.chart(quat, log_scale)

    def _allreduce(self, t):
        if self.world > 1:
            import torch.distributed as dist
            try:
                dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
            except RuntimeError as exc:   # a peer left or hung: the collective timed out or broke
                raise PeerFailure(f"rank {self.rank}: allreduce failed: {exc}") from exc

    def check_peers(self):
        """Host-side liveness check of every rank (no-op without ``heartbeat`` or on one rank):
        returns when all ranks reached it, raises ``PeerFailure`` naming the missing ones after
        ``heartbeat`` seconds."""
        if self._hb_group is None:
            return
        import torch.distributed as dist
        try:
            dist.monitored_barrier(group=self._hb_group, timeout=timedelta(seconds=self.heartbeat),
                                   wait_all_ranks=True)
        except RuntimeError as exc:
            raise PeerFailure(f"rank {self.rank}: liveness check failed: {exc}") from exc

    def _outputs(self, E, d, g_quat, g_log):
        M, eng = self.M, self.engine
        gC = self.packed[10 * M:10 * M + self.n_gc].view(M, -1)[:, :self.n_occ]
        out = dict(E=E, gamma=eng.gamma, d=d, J_local=eng.J, g_quat=g_quat, g_log_scale=g_log,
                   g_centers=eng.gmu, g_C=gC)
        if self.external:
            out["E_ne"] = self.packed[-1:]
        return out

    def step(self, quat, log_scale, centers, C_occ, occ, grad=True):
        self.check_peers()
        gamma = self._forward(quat, log_scale, centers, C_occ, occ)
        self._allreduce(gamma)
        if not grad:
            E, d = self.engine.solve()
            out = dict(E=E, gamma=gamma, d=d)
            if self.external:
                E_ne = self.engine.external().clone()
                self._allreduce(E_ne)
                out["E_ne"] = E_ne
            return out
        E, d = self._middle(centers, C_occ, occ)
        self._allreduce(self.packed)
        g_quat, g_log = self._tail(quat, log_scale)
        return self._outputs(E, d, g_quat, g_log)

    def capture(self, quat, log_scale, centers, C_occ, occ, warmup: int = 2):
        """The step as CUDA graphs: one graph on a single device; on several, three graphs (the
        compute before, between and after the two allreduces) with the NCCL allreduces issued
        eagerly in between — collectives are never captured. ``warmup`` eager steps run first.
        Inputs are read at the given tensors' addresses: copy new parameters into them before
        ``replay()``."""
        from ..coulomb.engine import StepGraph
        if self.world == 1:
            return StepGraph(lambda: self.step(quat, log_scale, centers, C_occ, occ),
                             warmup=warmup)
        return _SegmentedStep(self, quat, log_scale, centers, C_occ, occ, warmup)

    def phase_events(self):
        """Six timing events for ``_SegmentedStep.replay(phases)``: recorded on the current stream
        before the forward, after it, after the gamma allreduce, after the middle segment, after
        the gradient allreduce and after the chart (five phases)."""
        import torch
        return [torch.cuda.Event(enable_timing=True) for _ in range(6)]


class _SegmentedStep:
    """Three captured compute segments with eager NCCL allreduces between them."""

    def __init__(self, sh, quat, log_scale, centers, C_occ, occ, warmup=2):
        import torch
        from ..coulomb.engine import StepGraph
        # eager warm-up of the whole step (collectives included) on the current stream
        for _ in range(max(warmup, 1)):
            sh.step(quat, log_scale, centers, C_occ, occ)
        torch.cuda.synchronize()
        self.sh = sh
        self.gA = StepGraph(lambda: sh._forward(quat, log_scale, centers, C_occ, occ), warmup=0)
        self.gB = StepGraph(lambda: sh._middle(centers, C_occ, occ), warmup=0)
        self.gC = StepGraph(lambda: sh._tail(quat, log_scale), warmup=0)
        self.launches = self.gA.launches + self.gB.launches + self.gC.launches

    def replay(self, phases=None):
        """One step; with ``phases`` (six events from ``phase_events``) each segment and each
        allreduce is bracketed on the current stream."""
        sh = self.sh
        sh.check_peers()
        rec = (lambda k: phases[k].record()) if phases is not None else (lambda k: None)
        rec(0)
        gamma = self.gA.replay()
        rec(1)
        sh._allreduce(gamma)
        rec(2)
        E, d = self.gB.replay()
        rec(3)
        sh._allreduce(sh.packed)
        rec(4)
        g_quat, g_log = self.gC.replay()
        rec(5)
        return sh._outputs(E, d, g_quat, g_log)
