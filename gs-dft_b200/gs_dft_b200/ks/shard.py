"""Multi-GPU RI-J: one process per GPU, the pair list partitioned across ranks, NCCL allreduce of
the aux fit vector and of the splat cotangents.

Replaces the DF branch of gs_dft/ks/shard.py:169-245 (``shard_map`` over mesh axis "g" with
``lax.psum`` of gamma, replicated solve, gradient psum through the shard_map transpose) and the
per-step replica ``pmean`` of gs_dft/ks/shard.py:44-65, which is not needed because every rank
computes bit-identical replicated values.

Partition: every rank builds the same refresh-time plan of the whole list (live entries, with each
(i,j)/(j,i) twin merged into one representative) and evaluates a contiguous slice of the
representatives, equal to within one: every representative costs the same N_aux integrals and
padding costs nothing, so equal counts are equal work, and contiguity keeps each rank's per-splat
scatter local. The reference instead deals the padded list round-robin (``stripe_pairs``) because
its padding is appended; striped lists are accepted too (a stripe only reorders the same pairs).
"""
from __future__ import annotations

import torch

from ..coulomb.engine import RIJEngine
from ..screening.pairs import pair_weight, stripe_pairs

__all__ = ["ShardedRIJ", "stripe_pairs"]


class ShardedRIJ:
    """This rank's share of a sharded J-build + gradient.

    ``group`` is a torch.distributed process group (NCCL on GPUs; gloo works for CPU-side tests of
    the host logic). All ranks take the same collective steps in the same order.
    """

    def __init__(self, pi, pj, valid, M, n_occ, beta, R, KN, L, rank: int, world: int,
                 group=None, engine_cls=RIJEngine):
        self.rank, self.world, self.group = rank, world, group
        self.engine = engine_cls(pi.contiguous(), pj.contiguous(), pair_weight(valid).contiguous(),
                                 M, n_occ, beta, R, KN, L, rank=rank, world=world)
        self.M, self.n_occ = int(M), int(n_occ)
        self.packed = torch.empty(10 * self.M + self.M * max(self.n_occ, 1),
                                  dtype=torch.float64, device=pi.device)

    def step(self, quat, log_scale, centers, C_occ, occ, grad=True):
        import torch.distributed as dist
        eng = self.engine
        gamma = eng.forward_local(quat, log_scale, centers, C_occ, occ)
        if self.world > 1:
            dist.all_reduce(gamma, op=dist.ReduceOp.SUM, group=self.group)
        E, d = eng.solve()
        out = dict(E=E, gamma=gamma, d=d)
        if not grad:
            return out
        gA6, gmu, gN, gC = eng.backward_local(centers, C_occ, occ)
        M = self.M
        p = self.packed
        p[:6 * M].copy_(gA6.reshape(-1))
        p[6 * M:9 * M].copy_(gmu.reshape(-1))
        p[9 * M:10 * M].copy_(gN)
        if self.n_occ:
            p[10 * M:].copy_(gC[:, :self.n_occ].reshape(-1))
        if self.world > 1:
            dist.all_reduce(p, op=dist.ReduceOp.SUM, group=self.group)
        eng.gA6.copy_(p[:6 * M].view(M, 6))
        eng.gmu.copy_(p[6 * M:9 * M].view(M, 3))
        eng.gN.copy_(p[9 * M:10 * M])
        g_quat, g_log = eng.chart(quat, log_scale)
        out.update(J_local=eng.J, g_quat=g_quat, g_log_scale=g_log, g_centers=eng.gmu,
                   g_C=p[10 * M:].view(M, -1)[:, :self.n_occ])
        return out
