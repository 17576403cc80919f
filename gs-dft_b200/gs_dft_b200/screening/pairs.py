"""Significant-overlap pair list, built on the GPU.

Mirror of gs_dft/screening/pairs.py:225-315 (``neighbor_pairs``), :318-327 (weights) and
gs_dft/ks/shard.py:146-166 (``stripe_pairs``). The overlap test, ordered compaction, tail padding
and overflow ranking run in ``gsdft_pairs_count`` / ``gsdft_pairs_build`` (CUDA).
"""
from __future__ import annotations

import ctypes

import torch

from .._lib import lib, ptr, stream_handle
from ..basis.spectral import full_quantities


def _check_splats(splats):
    if not all(hasattr(splats, a) for a in ("A", "centers", "norm", "n_basis")):
        raise NotImplementedError(
            f"neighbor_pairs: {type(splats).__name__} does not expose the splat interface "
            f"(.A / .centers / .norm / .n_basis)")


def count_significant(splats, eps: float, unique: bool = False) -> int:
    """Number of pairs with |S_ij| > eps (j >= i when unique) — one device pass, one host sync."""
    _check_splats(splats)
    A9, mu, N = full_quantities(splats)
    M = splats.n_basis
    ws_bytes = lib.gsdft_pairs_workspace_size(M, 0)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=mu.device)
    n = ctypes.c_int64(0)
    lib.call("gsdft_pairs_count", ptr(A9), ptr(mu), ptr(N), M, float(eps), int(bool(unique)),
             ctypes.byref(n), ptr(ws), ws_bytes, stream_handle(mu.device))
    return int(n.value)


def neighbor_pairs(splats, eps: float = 1e-5, pad_to: int | None = None, row_chunk: int = 256,
                   unique: bool = False):
    """Significant pairs (i,j) with |S_ij| > eps, lexsorted by i*M+j, as (pi, pj, valid).

    ``valid`` is a bool mask (ordered) or float64 (2 - delta_ij) weights (``unique``), 0 on the
    tail padding. With ``pad_to`` the arrays have exactly that length; if more pairs are
    significant the ``pad_to`` largest |S| are kept (ties by ascending flat index); more than twice
    the pad raises ``ValueError``. ``eps < 0`` keeps every pair. ``row_chunk`` is accepted for
    signature compatibility (the device build needs no strip size).
    """
    _check_splats(splats)
    A9, mu, N = full_quantities(splats)
    M = splats.n_basis
    dev = mu.device
    if pad_to is None:
        pad_to = count_significant(splats, eps, unique)
    pad_to = int(pad_to)
    pi = torch.empty(max(pad_to, 1), dtype=torch.int32, device=dev)
    pj = torch.empty(max(pad_to, 1), dtype=torch.int32, device=dev)
    w = torch.empty(max(pad_to, 1), dtype=torch.float64, device=dev)
    ws_bytes = lib.gsdft_pairs_workspace_size(M, pad_to)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    n_sig = ctypes.c_int64(0)
    try:
        lib.call("gsdft_pairs_build", ptr(A9), ptr(mu), ptr(N), M, float(eps),
                 int(bool(unique)), pad_to, ptr(pi), ptr(pj), ptr(w), ctypes.byref(n_sig),
                 ptr(ws), ws_bytes, stream_handle(dev))
    except RuntimeError as exc:
        if getattr(exc, "code", None) == 3:
            raise ValueError(str(exc)) from exc
        raise
    pi, pj, w = pi[:pad_to], pj[:pad_to], w[:pad_to]
    if int(n_sig.value) > pad_to:
        print(f"  [screening] pair count {int(n_sig.value)} > pad {pad_to}: keeping the {pad_to} "
              f"largest-overlap pairs (dropped {int(n_sig.value) - pad_to})", flush=True)
    valid = w if unique else (w != 0)
    return pi, pj, valid


def pair_weight(valid, dtype=torch.float64):
    """``valid`` as a multiplicative factor: 0/1 from a bool mask, 0/1/2 from unique weights."""
    return valid.to(dtype)


def stripe_pairs(pi, pj, valid, G: int):
    """Round-robin deal so each of the G contiguous device blocks holds the same valid:dummy
    ratio with its valid entries first (gs_dft/ks/shard.py:146-166)."""
    n = int(pi.shape[0])
    if G <= 1 or n % G:
        return pi, pj, valid
    w = pair_weight(valid).contiguous()
    pi, pj = pi.to(torch.int32).contiguous(), pj.to(torch.int32).contiguous()
    pio, pjo, wo = torch.empty_like(pi), torch.empty_like(pj), torch.empty_like(w)
    lib.call("gsdft_stripe_pairs", ptr(pi), ptr(pj), ptr(w), n, int(G),
             ptr(pio), ptr(pjo), ptr(wo), stream_handle(pi.device))
    return pio, pjo, (wo if valid.dtype == torch.float64 else wo != 0)
