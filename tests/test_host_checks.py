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
