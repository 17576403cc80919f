"""Seeded synthetic splat clouds for the five benchmark configurations.

The reference measures on no public dataset; these clusters stand in for its molecules. Every
array is FP64 numpy, generated from ``numpy.random.default_rng(seed)`` in a fixed draw order, so
the oracle, the GPU path and the CPU baseline all see the same inputs.

Conventions (fixed here, kept everywhere):

* splats per atom follow the reference's divmod rule, the first atoms taking the remainder
  (gs_dft/basis/spectral.py:95-106);
* centres are the atom plus N(0, 0.5 Bohr) jitter;
* per-axis widths sigma are log-uniform in [0.2, 3.0] Bohr, stored as
  ``log_scale = -2 ln(sigma) - ln 2`` (precision eigenvalue 1/(2 sigma^2));
* quaternions are normalised 4-D Gaussians (uniform random rotations);
* ``C_occ`` is the Q factor of an M x n_occ Gaussian, ``occ = 2``;
* nuclear charges are the elements' (H 1, C 6, O 8); the random test clouds cycle through
  (6, 1, 8, 1, 7, 1) with no random draw, so adding them changed no other array.

Geometries: CO2 with O at +-2.196 Bohr (1.1621 A, gs_dft/geometries.py:29-33); ethanol from
gs_dft/geometries.py:68-78; water clusters from the monomer gs_dft/geometries.py:18-22, each
molecule randomly rotated, on a cubic lattice of 3.1 A.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

BOHR_PER_ANGSTROM = 1.0 / 0.529177210903

_ETHANOL_A = np.array([
    [1.1879, -0.3829, 0.0000],   # C
    [0.0000, 0.5526, 0.0000],    # C
    [-1.1867, -0.2472, 0.0000],  # O
    [-1.9237, 0.3850, 0.0000],   # H
    [2.0985, 0.2306, 0.0000],    # H
    [1.1184, -1.0093, 0.8869],   # H
    [1.1184, -1.0093, -0.8869],  # H
    [-0.0227, 1.1812, 0.8852],   # H
    [-0.0227, 1.1812, -0.8852],  # H
])

_ETHANOL_Z = np.array([6.0, 6.0, 8.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0])
_WATER_Z = np.array([8.0, 1.0, 1.0])
_CO2_Z = np.array([6.0, 8.0, 8.0])
_CYCLE_Z = (6.0, 1.0, 8.0, 1.0, 7.0, 1.0)

_WATER_A = np.array([
    [0.0000, 0.0000, 0.1173],    # O
    [0.0000, 0.7572, -0.4692],   # H
    [0.0000, -0.7572, -0.4692],  # H
])


@dataclass
class SplatSystem:
    """One synthetic configuration: the splat chart parameters plus occupied orbitals."""

    name: str
    atoms: np.ndarray        # (n_atoms, 3) Bohr
    quat: np.ndarray         # (M, 4)
    log_scale: np.ndarray    # (M, 3)
    centers: np.ndarray      # (M, 3) Bohr
    C_occ: np.ndarray        # (M, n_occ), orthonormal columns
    occ: np.ndarray          # (n_occ,)
    eps: float = 1e-7
    lam: float = 1e-8
    charges: np.ndarray | None = None   # (n_atoms,) nuclear charges Z_A

    def __post_init__(self):
        if self.charges is None:
            self.charges = np.array([_CYCLE_Z[k % len(_CYCLE_Z)]
                                     for k in range(self.atoms.shape[0])], dtype=np.float64)

    @property
    def M(self) -> int:
        return int(self.centers.shape[0])

    @property
    def n_occ(self) -> int:
        return int(self.C_occ.shape[1])


def _random_rotation(rng) -> np.ndarray:
    q = rng.standard_normal(4)
    q /= np.linalg.norm(q)
    w, x, y, z = q
    return np.array([
        [1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
        [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
        [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)],
    ])


def water_cluster(n_side: int, n_keep: int | None, rng, spacing_A: float = 3.1) -> np.ndarray:
    """Randomly oriented waters on an n_side^3 lattice (first ``n_keep`` sites), in Bohr."""
    sites = np.array([(i, j, k) for i in range(n_side) for j in range(n_side)
                      for k in range(n_side)], dtype=np.float64) * spacing_A
    if n_keep is not None:
        sites = sites[:n_keep]
    atoms = []
    for s in sites:
        R = _random_rotation(rng)
        atoms.append(_WATER_A @ R.T + s)
    return np.concatenate(atoms, axis=0) * BOHR_PER_ANGSTROM


def splat_cloud(name: str, atoms: np.ndarray, M: int, n_occ: int, rng,
                eps: float = 1e-7, charges: np.ndarray | None = None) -> SplatSystem:
    """Draw M splats over ``atoms`` (divmod allocation) and an orthonormal C_occ."""
    n_atoms = atoms.shape[0]
    base, rem = divmod(M, n_atoms)
    counts = [base + (1 if a < rem else 0) for a in range(n_atoms)]
    owner = np.repeat(np.arange(n_atoms), counts)
    centers = atoms[owner] + 0.5 * rng.standard_normal((M, 3))
    log_sigma = rng.uniform(np.log(0.2), np.log(3.0), size=(M, 3))
    log_scale = -2.0 * log_sigma - np.log(2.0)
    quat = rng.standard_normal((M, 4))
    quat /= np.linalg.norm(quat, axis=1, keepdims=True)
    G = rng.standard_normal((M, n_occ))
    C_occ, _ = np.linalg.qr(G)
    occ = np.full(n_occ, 2.0)
    return SplatSystem(name=name, atoms=atoms, quat=quat, log_scale=log_scale,
                       centers=centers, C_occ=np.ascontiguousarray(C_occ), occ=occ, eps=eps,
                       charges=None if charges is None else np.asarray(charges, np.float64))


def make_config(index: int, M: int | None = None) -> SplatSystem:
    """Configuration ``index`` (0-4) of the benchmark ladder; ``M`` overrides the splat count
    (used by tests to shrink a geometry while keeping its layout)."""
    if index == 0:
        rng = np.random.default_rng(0)
        atoms = np.array([[0.0, 0.0, 0.0], [0.0, 0.0, 2.196], [0.0, 0.0, -2.196]])
        return splat_cloud("co2", atoms, M or 126, 11, rng, charges=_CO2_Z)
    if index == 1:
        rng = np.random.default_rng(0)
        atoms = _ETHANOL_A * BOHR_PER_ANGSTROM
        return splat_cloud("ethanol", atoms, M or 600, 13, rng, charges=_ETHANOL_Z)
    if index == 2:
        rng = np.random.default_rng(1)
        atoms = water_cluster(4, None, rng)
        return splat_cloud("h2o_64", atoms, M or 3000, 320, rng,
                           charges=np.tile(_WATER_Z, atoms.shape[0] // 3))
    if index == 3:
        rng = np.random.default_rng(2)
        atoms = water_cluster(7, None, rng)
        return splat_cloud("h2o_343", atoms, M or 20000, 1715, rng,
                           charges=np.tile(_WATER_Z, atoms.shape[0] // 3))
    if index == 4:
        rng = np.random.default_rng(3)
        atoms = water_cluster(10, 914, rng)
        return splat_cloud("h2o_914", atoms, M or 53000, 4570, rng,
                           charges=np.tile(_WATER_Z, atoms.shape[0] // 3))
    raise ValueError(f"unknown config {index}")


def small_random_system(M: int = 24, n_occ: int = 4, seed: int = 0, spread: float = 1.5,
                        n_atoms: int = 4) -> SplatSystem:
    """A tiny random cloud for parity tests (atoms uniform in a box of half-width ``spread``)."""
    rng = np.random.default_rng(seed)
    atoms = rng.uniform(-spread, spread, size=(n_atoms, 3))
    return splat_cloud(f"random_M{M}_s{seed}", atoms, M, n_occ, rng)
