"""ctypes binding of ``libgsdft_b200.so`` (the C ABI declared in ``include/gsdft_b200.h``).

The library is built in-tree (``gs_dft_b200/_build.py``). There is no fallback: if the shared
library is missing or cannot be loaded, every GPU entry point raises ``RuntimeError``.
Device memory comes from torch tensors (plumbing); only pointers and sizes cross the ABI.
"""
from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libgsdft_b200.so")

GSDFT_OK = 0
ERR_ARG, ERR_CUDA, ERR_OVERFLOW, ERR_LINALG = 1, 2, 3, 4
REC_FIELDS = 18
VJP_FIELDS = 13
SIDE_FIELDS = 20
XC_FIELDS = 11
NODE_TABLE_DOUBLES = 1320
SOLVE_INV_MAX = 65536   # GSDFT_SOLVE_INV_MAX
ABI_VERSION = 4         # GSDFT_ABI_VERSION

_c_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f64 = ctypes.c_double
_sz = ctypes.c_size_t
_pi64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); mirrors include/gsdft_b200.h
SIGNATURES = {
    "gsdft_last_error_string": (ctypes.c_char_p, []),
    "gsdft_version": (_i32, []),
    "gsdft_device_status": (_i32, [ctypes.POINTER(ctypes.c_int), _i32]),
    "gsdft_kernel_launches": (_i64, []),
    "gsdft_dfma_probe": (_i32, [_c_p, _i64, _i32, _i32, _c_p]),
    "gsdft_set_node_screening": (_i32, [_i32]),
    "gsdft_node_screening": (_i32, []),
    "gsdft_node_evals": (_i32, [ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                _i32]),
    "gsdft_dense_gemm": (_i32, [_i32, _i32, _i64, _i64, _i64, _f64, _c_p, _i64, _c_p, _i64, _f64,
                                _c_p, _i64, _c_p]),
    "gsdft_block_density": (_i32, [_c_p, _c_p, _i64, _i64, _i64, _c_p, _c_p, _c_p, _c_p, _i64, _c_p,
                                   _c_p, _i64, _c_p, _c_p, _c_p]),
    "gsdft_block_density_grad": (_i32, [_c_p, _c_p, _i64, _c_p, _c_p, _i64, _i64, _i64, _c_p, _c_p,
                                        _c_p, _c_p, _i64, _c_p, _f64, _c_p, _c_p]),
    "gsdft_splat_quantities": (_i32, [_c_p, _c_p, _i64, _c_p, _c_p, _c_p]),
    "gsdft_chart_vjp": (_i32, [_c_p, _c_p, _c_p, _c_p, _i64, _c_p, _c_p, _c_p]),
    "gsdft_pairs_workspace_size": (_sz, [_i64, _i64]),
    "gsdft_pairs_count": (_i32, [_c_p, _c_p, _c_p, _i64, _f64, _i32, _pi64, _c_p, _sz, _c_p]),
    "gsdft_pairs_build": (_i32, [_c_p, _c_p, _c_p, _i64, _f64, _i32, _i64, _c_p, _c_p, _c_p,
                                 _pi64, _c_p, _sz, _c_p]),
    "gsdft_stripe_pairs": (_i32, [_c_p, _c_p, _c_p, _i64, _i32, _c_p, _c_p, _c_p, _c_p]),
    "gsdft_pair_plan_workspace_size": (_sz, [_i64, _i64]),
    "gsdft_pair_reps": (_i32, [_c_p, _c_p, _c_p, _i64, _i64, _i32, _c_p, _c_p, _c_p, _pi64, _c_p,
                               _sz, _c_p]),
    "gsdft_rep_cost": (_i32, [_c_p, _c_p, _i64, _c_p, _c_p, _c_p, _i64, _c_p, _c_p, _i64, _i64, _c_p,
                              _c_p]),
    "gsdft_pair_groups_workspace_size": (_sz, [_i64, _i64]),
    "gsdft_pair_groups": (_i32, [_c_p, _c_p, _c_p, _i64, _i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
                                 _c_p, _sz, _c_p]),
    "gsdft_product_aux": (_i32, [_c_p, _c_p, _c_p, _i64, _c_p, _c_p, _c_p, _i64,
                                 ctypes.POINTER(ctypes.c_double), _i32, _c_p, _c_p, _c_p]),
    "gsdft_aux_quantities": (_i32, [_c_p, _i64, _c_p, _c_p, _c_p]),
    "gsdft_aux_metric": (_i32, [_c_p, _c_p, _c_p, _i64, _c_p, _c_p]),
    "gsdft_aux_cholesky_workspace_size": (_sz, [_i64]),
    "gsdft_aux_cholesky": (_i32, [_c_p, _i64, _f64, _c_p, _sz, _c_p]),
    "gsdft_pair_prep": (_i32, [_c_p, _c_p, _c_p, _i64, _c_p, _c_p, _c_p, _c_p, _i64, _c_p, _c_p,
                               _i64, _c_p, _c_p]),
    "gsdft_j_forward_workspace_size": (_sz, [_i64, _i64]),
    "gsdft_j_forward": (_i32, [_c_p, _i64, _c_p, _c_p, _c_p, _i64, _c_p, _c_p, _sz, _c_p]),
    "gsdft_j_forward_noalloc": (_i32, [_c_p, _i64, _c_p, _c_p, _c_p, _i64, _c_p, _c_p]),
    "gsdft_j_solve_workspace_size": (_sz, [_i64]),
    "gsdft_j_solve": (_i32, [_c_p, _c_p, _i64, _c_p, _c_p, _c_p, _sz, _c_p]),
    "gsdft_j_solve_inverse": (_i32, [_c_p, _i64, _c_p, _c_p]),
    "gsdft_j_solve_inv_workspace_size": (_sz, [_i64]),
    "gsdft_j_solve_inv": (_i32, [_c_p, _c_p, _c_p, _i64, _c_p, _c_p, _c_p, _sz, _c_p]),
    "gsdft_j_vjp_workspace_size": (_sz, [_i64, _i64]),
    "gsdft_j_vjp": (_i32, [_c_p, _i64, _c_p, _c_p, _c_p, _c_p, _c_p, _i64, _c_p, _c_p, _sz,
                           _c_p]),
    "gsdft_pair_chain": (_i32, [_c_p, _c_p, _c_p, _i64, _c_p, _c_p, _c_p, _c_p, _c_p, _i64, _i64,
                                _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p]),
    "gsdft_splat_reduce": (_i32, [_c_p, _c_p, _c_p, _c_p, _c_p, _i64, _i64, _c_p, _c_p, _c_p,
                                  _c_p]),
    "gsdft_vne_workspace_size": (_sz, [_i64]),
    "gsdft_vne": (_i32, [_c_p, _i64, _c_p, _i64, _c_p, _c_p, _c_p, _i64, _c_p, _c_p, _c_p, _i32,
                         _c_p, _sz, _c_p]),
    "gsdft_density_pairs": (_i32, [_c_p, _c_p, _i64, _c_p, _c_p, _i64, _c_p, _c_p]),
    "gsdft_j_vjp_weighted_workspace_size": (_sz, [_i64, _i64]),
    "gsdft_j_vjp_weighted": (_i32, [_c_p, _i64, _c_p, _c_p, _c_p, _c_p, _i64, _i64, _c_p, _i32, _c_p,
                                    _c_p, _sz, _c_p]),
    "gsdft_lr_node_table": (_i32, [_f64, _i32, _c_p, _c_p]),
    "gsdft_aux_metric_lr": (_i32, [_c_p, _c_p, _c_p, _i64, _f64, _c_p, _c_p]),
    "gsdft_k_workspace_size": (_sz, [_i64, _i64, _i64, _i64]),
    "gsdft_k_forward": (_i32, [_c_p, _c_p, _c_p, _c_p, _c_p, _i64, _c_p, _c_p, _c_p, _i64, _c_p, _i32,
                               _c_p, _c_p, _i64, _i64, _c_p, _c_p, _c_p, _sz, _c_p]),
    "gsdft_k_backward": (_i32, [_c_p, _c_p, _c_p, _c_p, _c_p, _i64, _c_p, _c_p, _c_p, _i64, _c_p, _i32,
                                _c_p, _c_p, _i64, _i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
                                _c_p, _i64, _c_p, _c_p, _c_p, _sz, _c_p]),
    "gsdft_k_unit_q": (_i32, [_c_p, _i64, _c_p, _c_p]),
    "gsdft_exact_j_workspace_size": (_sz, [_i64]),
    "gsdft_exact_j": (_i32, [_c_p, _i64, _i32, _c_p, _c_p, _c_p, _sz, _c_p]),
    "gsdft_exact_j_vjp_workspace_size": (_sz, [_i64]),
    "gsdft_exact_j_vjp": (_i32, [_c_p, _i64, _i32, _c_p, _c_p, _c_p, _sz, _c_p]),
    "gsdft_density_grad": (_i32, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _i64, _i64, _c_p, _c_p,
                                  _i64, _c_p, _c_p]),
}


class GsdftError(RuntimeError):
    """A C-ABI call returned a nonzero status."""

    def __init__(self, fn, code, msg):
        super().__init__(f"{fn} failed (status {code}): {msg}")
        self.code = code


class _Lib:
    def __init__(self):
        self._h = None

    def load(self):
        if self._h is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m gs_dft_b200._build` "
                    f"(nvcc, sm_100a). There is no CPU fallback.")
            h = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                f = getattr(h, name)
                f.restype = res
                f.argtypes = args
            if h.gsdft_version() != ABI_VERSION:
                raise RuntimeError(
                    f"{LIB_PATH} implements ABI version {h.gsdft_version()}, this package needs "
                    f"{ABI_VERSION}: the library is stale, rebuild it with "
                    f"`python -m gs_dft_b200._build`")
            self._h = h
        return self._h

    def __getattr__(self, name):
        return getattr(self.load(), name)

    def call(self, name, *args):
        fn = getattr(self.load(), name)
        rc = fn(*args)
        if rc != GSDFT_OK:
            msg = self.load().gsdft_last_error_string()
            raise GsdftError(name, rc, msg.decode() if msg else "")
        return rc


lib = _Lib()


def ptr(t):
    """Device pointer of a torch tensor (None -> NULL)."""
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def stream_handle(device=None):
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
