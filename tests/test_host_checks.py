"""The host layer refuses arguments the kernels would misread (wrong dtype, shape, layout, device,
or pair indices outside [0, M)) before any launch. CPU only: every check raises before the library
is called."""
import pytest
import torch

from gs_dft_b200 import _check
from gs_dft_b200.basis.spectral import Splat
from gs_dft_b200.coulomb.engine import check_step_inputs, make_plan

F64 = torch.float64


def test_splat_rejects_wrong_dtype_shape_and_host_memory():
    q, l, c = torch.zeros(5, 4, dtype=F64), torch.zeros(5, 3, dtype=F64), torch.zeros(5, 3, dtype=F64)
    with pytest.raises(TypeError, match="float64"):
        Splat(q.float(), l, c)
    with pytest.raises(ValueError, match="shape"):
        Splat(q[:, :3], l, c)
    with pytest.raises(ValueError, match="shape"):
        Splat(q, l, c[:4])
    with pytest.raises(ValueError, match="CUDA"):
        Splat(q, l, c)


def test_step_inputs_checked_against_the_engine_sizes():
    M, n_occ = 6, 2
    q, l, c = torch.zeros(M, 4, dtype=F64), torch.zeros(M, 3, dtype=F64), torch.zeros(M, 3, dtype=F64)
    C, occ = torch.zeros(M, n_occ, dtype=F64), torch.zeros(n_occ, dtype=F64)
    with pytest.raises(TypeError, match="C_occ"):
        check_step_inputs(M, n_occ, q, l, c, C.float(), occ)
    with pytest.raises(ValueError, match="C_occ"):
        check_step_inputs(M, n_occ, q, l, c, C[:, :1], occ)
    with pytest.raises(ValueError, match="contiguous"):
        check_step_inputs(M, n_occ, torch.zeros(4, M, dtype=F64).t(), l, c, C, occ)
    with pytest.raises(ValueError, match="CUDA"):
        check_step_inputs(M, n_occ, q, l, c, C, occ)


def test_pair_indices_dtype_length_and_range():
    pi = torch.tensor([0, 1, 2], dtype=torch.int32)
    pj = torch.tensor([2, 1, 0], dtype=torch.int32)
    _check.pair_indices(pi, pj, 3, cuda=False)
    with pytest.raises(TypeError, match="int32"):
        _check.pair_indices(pi.long(), pj, 3, cuda=False)
    with pytest.raises(ValueError, match="shape"):
        _check.pair_indices(pi, pj[:2], 3, cuda=False)
    with pytest.raises(ValueError, match=r"\[0, 3\)"):
        _check.pair_indices(pi, pj + 1, 3, cuda=False)
    with pytest.raises(ValueError, match=r"\[0, 3\)"):
        _check.pair_indices(pi - 1, pj, 3, cuda=False)
    with pytest.raises(ValueError, match="CUDA"):
        make_plan(pi, pj, torch.ones(3, dtype=F64), 3)


def test_partition_bounds_balance_cost():
    """Rank boundaries: equal counts without costs; with integer costs, contiguous ranges whose
    cumulative cost first passes k/world of the total (exact integer arithmetic)."""
    import torch
    from gs_dft_b200.coulomb.engine import partition_bounds
    assert partition_bounds(10, 3) == [0, 3, 6, 10]
    assert partition_bounds(0, 4) == [0, 0, 0, 0, 0]
    cost = torch.tensor([10, 1, 1, 1, 1, 1, 1, 1, 1, 2], dtype=torch.int64)   # total 20
    b = partition_bounds(10, 2, cost)
    assert b == [0, 1, 10]                     # the first representative alone is half the work
    rng = torch.Generator().manual_seed(0)
    cost = torch.randint(1, 40, (1000,), generator=rng, dtype=torch.int64)
    for world in (2, 3, 8):
        b = partition_bounds(1000, world, cost)
        assert b[0] == 0 and b[-1] == 1000 and all(x <= y for x, y in zip(b, b[1:]))
        sums = [int(cost[b[k]:b[k + 1]].sum()) for k in range(world)]
        assert max(sums) - min(sums) <= 2 * int(cost.max())


def test_row_blocks_structure():
    """The row-block structure of the many-orbital q / g_C tiles (host logic, on CPU tensors):
    every representative gets its own cell inside its row block's tile, at its row (the splat's
    place in its block of 64) and its partner's column; each block's partner list is sorted and
    holds exactly the partners of its rows; tile offsets are the exclusive sums of rows x partners;
    blocks without representatives are empty."""
    import numpy as np
    from gs_dft_b200.coulomb.engine import row_blocks
    rng = np.random.default_rng(4)
    M = 200                                   # blocks of 64, 64, 64, 8 rows; block 1 left empty
    live = np.r_[np.arange(0, 64), np.arange(128, M)]
    pairs = sorted({(int(rng.choice(live)), int(rng.choice(M))) for _ in range(1500)})
    rows = torch.tensor([p[0] for p in pairs], dtype=torch.int32)
    partners = torch.tensor([p[1] for p in pairs], dtype=torch.int32)
    bl = row_blocks(rows, partners, M)
    assert bl.n_blocks == 4
    nj, joff, boff = bl.nj.numpy(), bl.joff.numpy(), bl.boff.numpy()
    jidx, cell = bl.jidx.numpy(), bl.cell.numpy()
    rows_b = np.minimum(64, M - 64 * np.arange(4))
    np.testing.assert_array_equal(boff, np.r_[0, np.cumsum(rows_b * nj)[:-1]])
    assert bl.buf_len == int((rows_b * nj).sum()) and bl.max_nj == int(nj.max()) and nj[1] == 0
    r, p = rows.numpy().astype(np.int64), partners.numpy().astype(np.int64)
    for b in range(4):
        J = jidx[joff[b]:joff[b] + nj[b]]
        assert np.all(np.diff(J) > 0)
        np.testing.assert_array_equal(J, np.unique(p[r // 64 == b]))
    b = r // 64
    col = np.array([np.searchsorted(jidx[joff[k]:joff[k] + nj[k]], q) for k, q in zip(b, p)])
    np.testing.assert_array_equal(cell, boff[b] + (r - 64 * b) * nj[b] + col)
    assert len(np.unique(cell)) == len(cell) and cell.max() < bl.buf_len
    empty = row_blocks(rows[:0], partners[:0], M)
    assert empty.buf_len == 0 and empty.max_nj == 0
