"""The multi-rank host logic of ``ShardedRIJ`` (contiguous live-balanced partition, allreduce of
gamma, replicated solve, packed allreduce of the splat cotangents, replicated chart reverse) on
world_size 2 over gloo, CPU only. A CPU engine built on the oracle stands in for the CUDA engine
(same stage interface); the 2-rank result must equal the 1-rank result."""
import os
import socket

import numpy as np
import pytest
import torch

import gsdft_oracle as O


def _sym6(gA):
    return np.stack([gA[:, 0, 0], gA[:, 1, 1], gA[:, 2, 2], 0.5 * (gA[:, 0, 1] + gA[:, 1, 0]),
                     0.5 * (gA[:, 0, 2] + gA[:, 2, 0]), 0.5 * (gA[:, 1, 2] + gA[:, 2, 1])], -1)


def _full(g6):
    A = np.empty((g6.shape[0], 3, 3))
    A[:, 0, 0], A[:, 1, 1], A[:, 2, 2] = g6[:, 0], g6[:, 1], g6[:, 2]
    A[:, 0, 1] = A[:, 1, 0] = g6[:, 3]
    A[:, 0, 2] = A[:, 2, 0] = g6[:, 4]
    A[:, 1, 2] = A[:, 2, 1] = g6[:, 5]
    return A


class OracleEngine:
    """CPU stand-in for RIJEngine with the same stage methods, computed by the oracle."""

    def __init__(self, pi, pj, w, M, n_occ, beta, R, KN, L, rank=0, world=1, atoms=None):
        # this rank's contiguous share of the live entries (the sum over pairs is order-free)
        live = np.nonzero(w.numpy() != 0)[0]
        r0, r1 = len(live) * rank // world, len(live) * (rank + 1) // world
        sel = live[r0:r1]
        self.pi, self.pj, self.w = pi.numpy()[sel], pj.numpy()[sel], w.numpy()[sel]
        self.M, self.n_occ = M, n_occ
        self.aq = (beta.numpy(), R.numpy(), KN.numpy())
        self.L = L.numpy()
        self.J = torch.zeros(max(len(self.pi), 1), dtype=torch.float64)
        self.atoms = None if atoms is None else atoms.numpy()

    def forward_local(self, quat, ls, cen, C, occ):
        q = O.full_quantities(quat.numpy(), ls.numpy(), cen.numpy())
        self.qs = q
        g = O.df_coulomb_gamma_screened(q, C.numpy(), occ.numpy(), self.aq, self.pi, self.pj,
                                        self.w, chunk=256)
        self.gamma = torch.from_numpy(g)
        return self.gamma

    def solve(self):
        E, d = O.df_coulomb_solve(self.gamma.numpy(), self.L)
        self.E, self.d = torch.tensor([E], dtype=torch.float64), torch.from_numpy(d)
        return self.E, self.d

    def backward_local(self, cen, C, occ, g_E=None):
        live = self.w != 0
        ci, cj, cw = self.pi[live], self.pj[live], self.w[live]
        Cn, on = C.numpy(), occ.numpy()
        qa = O.pair_density(Cn, on, ci, cj, cw)
        Ah, Pa, KNa = O.full_pair_quantities(self.qs, ci, cj)
        J, Abar, Pbar, KNbar = O._pair_vjp_integral(*self.aq[:2], self.aq[2], self.d.numpy(), Ah,
                                                    Pa, KNa, qa)
        if self.atoms is not None:
            V, Ab2, Pb2, Kb2 = O._pair_vjp_nuclear(self.atoms[:, :3], self.atoms[:, 3], Ah, Pa,
                                                   KNa, qa)
            J, Abar, Pbar, KNbar = J + V, Abar + Ab2, Pbar + Pb2, KNbar + Kb2
            self.E_ne = torch.tensor([float(np.sum(qa * V))], dtype=torch.float64)
        gAi, gAj, gmui, gmuj, gNi, gNj = O._pair_chain(self.qs, ci, cj, Abar, Pbar, KNbar)
        gA, gmu, gN = np.zeros((self.M, 3, 3)), np.zeros((self.M, 3)), np.zeros(self.M)
        np.add.at(gA, ci, gAi)
        np.add.at(gA, cj, gAj)
        np.add.at(gmu, ci, gmui)
        np.add.at(gmu, cj, gmuj)
        np.add.at(gN, ci, gNi)
        np.add.at(gN, cj, gNj)
        s = (J * cw)[:, None] * on[None, :]
        gC = np.zeros_like(Cn)
        np.add.at(gC, ci, s * Cn[cj])
        np.add.at(gC, cj, s * Cn[ci])
        self.gA6 = torch.from_numpy(_sym6(gA))
        self.gmu, self.gN, self.g_C = torch.from_numpy(gmu), torch.from_numpy(gN), torch.from_numpy(gC)
        return self.gA6, self.gmu, self.gN, self.g_C

    def chart(self, quat, ls):
        gq, gl = O.chart_vjp(quat.numpy(), ls.numpy(), _full(self.gA6.numpy()), self.gN.numpy())
        return torch.from_numpy(gq), torch.from_numpy(gl)


def _problem():
    from gs_dft_b200.systems import small_random_system
    s = small_random_system(20, 3, seed=11, spread=3.0, n_atoms=5)
    q = O.full_quantities(s.quat, s.log_scale, s.centers)
    n = O.count_significant(q, s.M, s.eps, False)
    pi, pj, v, _ = O.neighbor_pairs(q, eps=s.eps, pad_to=O.pad_rule(n, 2.0, 2))
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    L = O.aux_cholesky(O.aux_metric(*aq), s.lam)
    return s, pi, pj, v, aq, L


def _run(rank, world, port, out, with_atoms=False):
    import torch.distributed as dist
    from gs_dft_b200.ks.shard import ShardedRIJ
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world)
    s, pi, pj, v, aq, L = _problem()
    T = torch.from_numpy
    atoms = T(np.concatenate([s.atoms, s.charges[:, None]], 1)) if with_atoms else None
    sh = ShardedRIJ(T(pi), T(pj), T(v), s.M, s.n_occ, T(aq[0]), T(aq[1]), T(aq[2]), T(L), rank,
                    world, engine_cls=OracleEngine, atoms=atoms)
    o = sh.step(T(s.quat), T(s.log_scale), T(s.centers), T(s.C_occ), T(s.occ))
    keys = ("E", "gamma", "g_quat", "g_log_scale", "g_centers", "g_C") + (("E_ne",) if with_atoms else ())
    res = {k: o[k].numpy().copy() for k in keys}
    if world > 1:
        dist.destroy_process_group()
    np.savez(out.format(rank=rank, world=world), **res)


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


@pytest.mark.parametrize("with_atoms", [False, True])
def test_two_rank_gloo_equals_single_rank(tmp_path, with_atoms):
    import torch.multiprocessing as mp
    out = str(tmp_path / "r{rank}_w{world}.npz")
    _run(0, 1, _free_port(), out, with_atoms)
    mp.start_processes(_run, args=(2, _free_port(), out, with_atoms), nprocs=2,
                       start_method="spawn")
    one = np.load(out.format(rank=0, world=1))
    keys = ("E", "gamma", "g_quat", "g_log_scale", "g_centers", "g_C") + (("E_ne",) if with_atoms else ())
    for r in range(2):
        two = np.load(out.format(rank=r, world=2))
        for k in keys:
            np.testing.assert_allclose(two[k], one[k], rtol=1e-12, atol=1e-12 * np.abs(one[k]).max())
    if with_atoms:
        # the whole-system E_ne and gradient of E_J + E_ne against the oracle's separate terms
        s, pi, pj, v, aq, L = _problem()
        arr = (s.quat, s.log_scale, s.centers, s.C_occ, s.occ)
        rj = O.energy_and_grad(arr, aq, L, pi, pj, v)
        rn = O.external_energy_and_grad(arr, pi, pj, v, s.atoms, s.charges)
        np.testing.assert_allclose(float(one["E_ne"][0]), rn["E"], rtol=1e-12)
        for k in ("g_quat", "g_log_scale", "g_centers", "g_C"):
            want = rj[k] + rn[k]
            np.testing.assert_allclose(one[k], want, rtol=1e-10, atol=1e-12 * np.abs(want).max())


def _run_leave(rank, world, port, out, mode):
    """Both ranks take one step; then rank 1 leaves (exits, or stalls past the liveness timeout)
    and rank 0 tries the next step. Rank 0 records what happened and how long it took."""
    import time
    from datetime import timedelta
    import torch.distributed as dist
    from gs_dft_b200.ks.shard import PeerFailure, ShardedRIJ
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    s, pi, pj, v, aq, L = _problem()
    T = torch.from_numpy
    sh = ShardedRIJ(T(pi), T(pj), T(v), s.M, s.n_occ, T(aq[0]), T(aq[1]), T(aq[2]), T(L), rank,
                    world, engine_cls=OracleEngine, heartbeat=3.0)
    args = (T(s.quat), T(s.log_scale), T(s.centers), T(s.C_occ), T(s.occ))
    E1 = float(sh.step(*args)["E"][0])
    if rank == 1:
        if mode == "stall":
            time.sleep(10.0)
        os._exit(0)                       # leaves between steps, nothing in flight
    t0 = time.time()
    try:
        sh.step(*args)
        res = "completed"
    except PeerFailure as exc:
        res = f"PeerFailure {exc}"
    with open(out, "w") as f:
        f.write(f"{E1!r}\n{time.time() - t0:.2f}\n{res}\n")
    os._exit(0)                           # the group has a dead member: skip its teardown


@pytest.mark.timeout(180)
@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_peer_that_leaves_is_reported_not_waited_for(tmp_path, mode):
    """A rank that exits, or stalls, between steps: the surviving rank's next step raises
    PeerFailure from the host-side liveness check (3 s limit) before it launches anything, instead
    of waiting in a collective."""
    import torch.multiprocessing as mp
    out = str(tmp_path / "leave.txt")
    mp.start_processes(_run_leave, args=(2, _free_port(), out, mode), nprocs=2,
                       start_method="spawn")
    E1, dt, res = open(out).read().splitlines()
    assert np.isfinite(float(E1))
    assert res.startswith("PeerFailure"), res
    assert float(dt) < 20.0
    if mode == "stall":
        assert "1" in res                  # the liveness check names the missing rank
