"""The splat chart A = R(q) diag(exp l) R(q)^T on the device.

Mirror of gs_dft/basis/spectral.py:55-82 (``Splat`` with ``.A / .norm / .centers / .n_basis``);
the arithmetic runs in ``gsdft_splat_quantities`` (CUDA). Parameters are float64 CUDA tensors.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _check
from ..coulomb.engine import splat_quantities


@dataclass
class Splat:
    """Full-covariance Gaussian splats: quaternion ``quat`` (M,4), log precision eigenvalues
    ``log_scale`` (M,3), ``centers`` (M,3)."""

    quat: torch.Tensor
    log_scale: torch.Tensor
    centers: torch.Tensor

    def __post_init__(self):
        M = int(self.centers.shape[0]) if isinstance(self.centers, torch.Tensor) else -1
        for t, name, k in ((self.quat, "quat", 4), (self.log_scale, "log_scale", 3),
                           (self.centers, "centers", 3)):
            _check.f64(t, name, (M, k), contiguous=False)

    @property
    def n_basis(self) -> int:
        return int(self.centers.shape[0])

    @property
    def A(self) -> torch.Tensor:
        """Precision matrices (M,3,3)."""
        return splat_quantities(self.quat.detach(), self.log_scale.detach())[0].view(-1, 3, 3)

    @property
    def norm(self) -> torch.Tensor:
        """N = (8 det A / pi^3)^(1/4)."""
        return splat_quantities(self.quat.detach(), self.log_scale.detach())[1]

    @classmethod
    def from_numpy(cls, quat, log_scale, centers, device="cuda"):
        t = lambda a: torch.as_tensor(a, dtype=torch.float64, device=device).contiguous()
        return cls(t(quat), t(log_scale), t(centers))


def full_quantities(splats: Splat):
    """(A9 (M,9) row-major, centers (M,3), N (M)) — gs_dft/coulomb/stream.py:79-81."""
    A9, N = splat_quantities(splats.quat.detach().contiguous(),
                             splats.log_scale.detach().contiguous())
    return A9, splats.centers.detach().contiguous(), N


def quat_to_rotation(q: torch.Tensor) -> torch.Tensor:
    """Unit-quaternion (w,x,y,z) -> rotation (gs_dft/basis/spectral.py:33-40); host-side helper
    for callers that want R itself (the kernels compute it inline)."""
    q = q / (torch.linalg.norm(q, dim=-1, keepdim=True) + 1e-12)
    w, x, y, z = q.unbind(-1)
    r0 = torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1)
    r1 = torch.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1)
    r2 = torch.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1)
    return torch.stack([r0, r1, r2], -2)
