"""Host-side argument checks at the library's boundary.

Every device entry point receives raw pointers, so a tensor of the wrong dtype, shape or layout
would be read as something it is not (and past its end). These checks are metadata only (no device
work, so they are safe inside CUDA-graph capture) and raise before any launch.
"""
from __future__ import annotations

import torch


def tensor(t, name: str, dtype: torch.dtype, shape=None, contiguous: bool = True,
           cuda: bool = True) -> torch.Tensor:
    """Check ``t``'s type, dtype, shape (a tuple; None matches any extent), layout and device."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if shape is not None:
        if t.dim() != len(shape) or any(s is not None and int(t.shape[k]) != int(s)
                                        for k, s in enumerate(shape)):
            want = tuple("*" if s is None else int(s) for s in shape)
            raise ValueError(f"{name} must have shape {want}, got {tuple(t.shape)}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if cuda and not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the library has no CPU path)")
    return t


def f64(t, name: str, shape=None, contiguous: bool = True) -> torch.Tensor:
    return tensor(t, name, torch.float64, shape, contiguous)


def pair_indices(pi, pj, M: int, cuda: bool = True):
    """int32 pair index lists of equal length with every index in [0, M) (one device sync)."""
    tensor(pi, "pi", torch.int32, (None,), cuda=cuda)
    tensor(pj, "pj", torch.int32, (int(pi.shape[0]),), cuda=cuda)
    if int(pi.shape[0]) > 0:
        lo = int(torch.minimum(pi.min(), pj.min()))
        hi = int(torch.maximum(pi.max(), pj.max()))
        if lo < 0 or hi >= M:
            raise ValueError(f"pair indices must lie in [0, {M}), got [{lo}, {hi}]")
