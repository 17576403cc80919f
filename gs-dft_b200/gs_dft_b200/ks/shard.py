"""Multi-GPU RI-J: one process per GPU, the pair list partitioned across ranks, NCCL allreduce of
the aux fit vector and of the splat cotangents.

Replaces the DF branch of gs_dft/ks/shard.py:169-245 (``shard_map`` over mesh axis "g" with
``lax.psum`` of gamma, replicated solve, gradient psum through the shard_map transpose) and the
per-step replica ``pmean`` of gs_dft/ks/shard.py:44-65, which is not needed because every rank
computes bit-identical replicated values.

Partition: contiguous ranges of the (lexsorted) list, balanced on LIVE pairs — every live pair
costs the same N_aux integrals, and zero-weight padding costs nothing, so equal live counts are
equal work; contiguity keeps each rank's per-splat scatter local. The reference instead deals the
padded list round-robin (``stripe_pairs``) because its padding is appended; striped lists are
accepted too (a stripe is just a different order of the same pairs).
"""
from __future__ import annotations

import torch

from ..coulomb.engine import RIJEngine
from ..screening.pairs import pair_weight, stripe_pairs

__all__ = ["partition_pairs", "ShardedRIJ", "stripe_pairs"]


def partition_pairs(valid: torch.Tensor, G: int) -> list[tuple[int, int]]:
    """G contiguous [start, end) ranges of the list with live counts equal to within one."""
    w = pair_weight(valid)
    n = int(w.shape[0])
    live = (w != 0).to(torch.int64)
    csum = torch.cumsum(live, 0)
    total = int(csum[-1].item()) if n else 0
    bounds = [0]
    for g in range(1, G):
        target = (total * g) // G
        # first index whose prefix live count exceeds the target
        k = int(torch.searchsorted(csum, torch.tensor([target], device=csum.device),
                                   right=True).item()) if n else 0
        bounds.append(min(max(k, bounds[-1]), n))
    bounds.append(n)
    return [(bounds[g], bounds[g + 1]) for g in range(G)]


class ShardedRIJ:
    """This rank's share of a sharded J-build + gradient.

    ``group`` is a torch.distributed process group (NCCL on GPUs; gloo works for CPU-side tests of
    the host logic). All ranks take the same collective steps in the same order.
    """

    def __init__(self, pi, pj, valid, M, n_occ, beta, R, KN, L, rank: int, world: int,
                 group=None, engine_cls=RIJEngine):
        self.rank, self.world, self.group = rank, world, group
        self.ranges = partition_pairs(valid, world)
        s, e = self.ranges[rank]
        w = pair_weight(valid)
        self.engine = engine_cls(pi[s:e].contiguous(), pj[s:e].contiguous(), w[s:e].contiguous(),
                                 M, n_occ, beta, R, KN, L)
        self.M, self.n_occ = int(M), int(n_occ)
        dev = pi.device
        self.packed = torch.empty(10 * self.M + self.M * max(self.n_occ, 1),
                                  dtype=torch.float64, device=dev)

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
