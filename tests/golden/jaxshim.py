"""A NumPy stand-in for the subset of the JAX / equinox / jaxtyping / dftax API that the reference's
RI-J modules touch, so that the reference's OWN source files can be executed in this container
(JAX cannot be installed: no network, and the reference pins Python >= 3.13).

Used only by ``make_golden.py`` to produce golden vectors. Every JAX primitive used on the forward
path maps to the NumPy operation with the same semantics:

* ``jnp.*``                -> ``numpy.*`` (float64 throughout, as under ``jax_enable_x64``), with
                              ``.at[idx].add/set`` on arrays and ``nonzero(size=, fill_value=)``;
* ``jnp.argsort``          -> stable argsort (JAX's default);
* ``lax.scan / fori_loop / cond / map`` -> Python loops;
* ``lax.dynamic_update_slice / dynamic_slice_in_dim`` -> slicing with JAX's start-index clamping;
* ``jax.jit / jax.checkpoint`` -> identity; ``jax.custom_vjp`` -> forward only, with the
  registered ``bwd`` kept on the object so the reference's hand-written reverse can be called;
* ``jax.scipy.linalg.cholesky / cho_solve`` -> numpy / scipy;
* ``dftax.energy.boys.boys(0, T)`` -> the closed form 1/2 sqrt(pi/T) erf(sqrt T) (dftax 0.8.0 is
  third-party and absent; its table is not reproduced).

Gradients (``jax.grad`` / ``jax.vjp``) are not provided: the generator takes them by finite
differences of the executed reference energy.
"""
from __future__ import annotations

import importlib
import os
import math
import sys
import types

import numpy as np
from scipy.special import erf

REFERENCE_ROOT = os.environ.get("GSDFT_REFERENCE_ROOT", "/root/reference")


class JArr(np.ndarray):
    """ndarray with JAX's functional ``.at[...]`` update syntax."""

    @property
    def at(self):
        return _At(self)

    def __getitem__(self, idx):
        # JAX clamps out-of-bounds gather indices (the reference's short tail strip relies on it).
        def clamp(ix, n):
            if isinstance(ix, np.ndarray) and ix.dtype.kind in "iu":
                return np.clip(ix, -n, n - 1)
            return ix
        if isinstance(idx, tuple):
            idx = tuple(clamp(ix, self.shape[d]) if d < self.ndim else ix
                        for d, ix in enumerate(idx))
        else:
            idx = clamp(idx, self.shape[0]) if self.ndim else idx
        return super().__getitem__(idx)


class _At:
    def __init__(self, a):
        self.a = a

    def __getitem__(self, idx):
        return _AtIdx(self.a, idx)


class _AtIdx:
    def __init__(self, a, idx):
        self.a, self.idx = a, idx

    def add(self, v):
        out = np.array(self.a, copy=True)
        np.add.at(out, self.idx, v)
        return _wrap(out)

    def set(self, v):
        out = np.array(self.a, copy=True)
        out[self.idx] = v
        return _wrap(out)


def _wrap(x):
    if isinstance(x, np.ndarray) and not isinstance(x, JArr):
        return x.view(JArr)
    if isinstance(x, tuple):
        return tuple(_wrap(e) for e in x)
    if isinstance(x, list):
        return [_wrap(e) for e in x]
    return x


def _wrapped(fn):
    def g(*args, **kwargs):
        return _wrap(fn(*args, **kwargs))
    g.__name__ = getattr(fn, "__name__", "f")
    return g


class _NumpyModule(types.ModuleType):
    """Forwards attribute access to a numpy namespace, wrapping array outputs as JArr."""

    def __init__(self, name, base, overrides):
        super().__init__(name)
        self._base = base
        self._over = overrides

    def __getattr__(self, item):
        if item in self._over:
            return self._over[item]
        v = getattr(self._base, item)
        if callable(v) and not isinstance(v, type):
            return _wrapped(v)
        return v


def _nonzero(x, size=None, fill_value=None):
    idx = np.nonzero(np.asarray(x))
    if size is None:
        return _wrap(idx)
    out = []
    for a in idx:
        a = a[:size]
        if a.size < size:
            fv = 0 if fill_value is None else fill_value
            a = np.concatenate([a, np.full(size - a.size, fv, a.dtype)])
        out.append(a)
    return _wrap(tuple(out))


def _argsort(x, axis=-1, stable=True, descending=False):
    return _wrap(np.argsort(np.asarray(x), axis=axis, kind="stable"))


def _asarray(x, dtype=None):
    return _wrap(np.asarray(x, dtype=dtype))


def _array(x, dtype=None):
    return _wrap(np.array(x, dtype=dtype))


_linalg = _NumpyModule("jax.numpy.linalg", np.linalg, {})


def _install_jnp():
    over = {
        "nonzero": _nonzero, "argsort": _argsort, "asarray": _asarray, "array": _array,
        "linalg": _linalg, "ndarray": JArr, "pi": math.pi,
        "int32": np.int32, "int64": np.int64, "float64": np.float64, "float32": np.float32,
        "bool_": np.bool_,
    }
    return _NumpyModule("jax.numpy", np, over)


def _scan(f, init, xs, length=None):
    carry = init
    ys = []
    if xs is None:
        n = length
        items = [None] * n
    elif isinstance(xs, (tuple, list)):
        n = len(xs[0])
        items = [tuple(x[i] for x in xs) for i in range(n)]
    else:
        n = len(xs)
        items = [xs[i] for i in range(n)]
    for it in items:
        carry, y = f(carry, it)
        ys.append(y)
    if all(y is None for y in ys):
        return carry, None
    if isinstance(ys[0], tuple):
        return carry, tuple(_wrap(np.stack([y[k] for y in ys])) for k in range(len(ys[0])))
    return carry, _wrap(np.stack(ys))


def _map(f, xs):
    _, ys = _scan(lambda c, x: (c, f(x)), None, xs)
    return ys


def _fori_loop(lo, hi, body, init):
    v = init
    for i in range(int(lo), int(hi)):
        v = body(i, v)
    return v


def _cond(pred, tf, ff, *ops):
    return tf(*ops) if bool(pred) else ff(*ops)


def _dynamic_update_slice(a, upd, starts):
    out = np.array(a, copy=True)
    sl = []
    for dim, s in enumerate(starts):
        s = int(s)
        s = max(0, min(s, out.shape[dim] - upd.shape[dim]))
        sl.append(slice(s, s + upd.shape[dim]))
    out[tuple(sl)] = upd
    return _wrap(out)


def _dynamic_slice_in_dim(a, start, size, axis=0):
    start = int(start)
    start = max(0, min(start, a.shape[axis] - size))
    idx = [slice(None)] * a.ndim
    idx[axis] = slice(start, start + size)
    return _wrap(np.asarray(a)[tuple(idx)])


def _jit(fun=None, **kwargs):
    if fun is None:
        return lambda f: f
    return fun


def _checkpoint(fun=None, **kwargs):
    if fun is None:
        return lambda f: f
    return fun


class _CustomVJP:
    def __init__(self, fun, nondiff_argnums=()):
        self.fun = fun
        self.fwd = None
        self.bwd = None

    def defvjp(self, fwd, bwd):
        self.fwd, self.bwd = fwd, bwd

    def __call__(self, *args, **kwargs):
        return self.fun(*args, **kwargs)


def _custom_vjp(fun=None, nondiff_argnums=()):
    if fun is None:
        return lambda f: _CustomVJP(f, nondiff_argnums)
    return _CustomVJP(fun, nondiff_argnums)


def boys_f0(T):
    """F0(T) = 1/2 sqrt(pi/T) erf(sqrt T); Taylor series below 1e-8."""
    T = np.asarray(T, np.float64)
    small = T < 1e-8
    Ts = np.where(small, 1.0, T)
    big = 0.5 * np.sqrt(np.pi / Ts) * erf(np.sqrt(Ts))
    ser = 1.0 - T / 3.0 + T * T / 10.0 - T * T * T / 42.0
    return np.where(small, ser, big)


def _boys(n, T):
    if n != 0:
        raise NotImplementedError("only F0 is on the RI-J path")
    return _wrap(boys_f0(T))


def _cholesky(a, lower=False):
    L = np.linalg.cholesky(np.asarray(a))
    return _wrap(L if lower else L.T)


def _cho_solve(c_and_lower, b):
    from scipy.linalg import cho_solve
    c, lower = c_and_lower
    return _wrap(cho_solve((np.asarray(c), lower), np.asarray(b)))


class _Subscriptable:
    def __getitem__(self, item):
        return self


def _eqx_field(static=False, default=None, **kw):
    import dataclasses
    if default is None:
        return dataclasses.field(default=None)
    return dataclasses.field(default=default)


class _EqxModule:
    def __init_subclass__(cls, **kw):
        import dataclasses
        super().__init_subclass__(**kw)
        if "__init__" not in cls.__dict__:
            dataclasses.dataclass(cls)


def install():
    """Register the stand-in modules and namespace packages for the reference tree."""
    if "jax" in sys.modules and getattr(sys.modules["jax"], "_IS_NUMPY_SHIM", False):
        return
    jax = types.ModuleType("jax")
    jax._IS_NUMPY_SHIM = True
    jax.numpy = _install_jnp()
    lax = types.ModuleType("jax.lax")
    lax.scan, lax.map, lax.fori_loop, lax.cond = _scan, _map, _fori_loop, _cond
    lax.dynamic_update_slice = _dynamic_update_slice
    lax.dynamic_slice_in_dim = _dynamic_slice_in_dim
    jax.lax = lax
    jax.jit, jax.checkpoint, jax.custom_vjp = _jit, _checkpoint, _custom_vjp
    jax.config = types.SimpleNamespace(update=lambda *a, **k: None)
    jax.random = types.ModuleType("jax.random")
    jax.random.PRNGKey = object          # annotation only on the modules loaded here
    jax.tree = types.ModuleType("jax.tree")
    jsp = types.ModuleType("jax.scipy")
    jspl = types.ModuleType("jax.scipy.linalg")
    jspl.cholesky, jspl.cho_solve = _cholesky, _cho_solve
    jsp.linalg = jspl
    jax.scipy = jsp
    for name, mod in [("jax", jax), ("jax.numpy", jax.numpy), ("jax.lax", lax),
                      ("jax.random", jax.random), ("jax.tree", jax.tree), ("jax.scipy", jsp),
                      ("jax.scipy.linalg", jspl)]:
        sys.modules[name] = mod
    eqx = types.ModuleType("equinox")
    eqx.Module, eqx.field = _EqxModule, _eqx_field
    sys.modules["equinox"] = eqx
    jt = types.ModuleType("jaxtyping")
    for n in ("Float", "Array", "Int", "Bool", "Scalar", "PRNGKeyArray"):
        setattr(jt, n, _Subscriptable())
    sys.modules["jaxtyping"] = jt
    dftax = types.ModuleType("dftax")
    dftax.__path__ = []
    en = types.ModuleType("dftax.energy")
    en.__path__ = []
    bmod = types.ModuleType("dftax.energy.boys")
    bmod.boys = _boys
    sys.modules.update({"dftax": dftax, "dftax.energy": en, "dftax.energy.boys": bmod})
    # Namespace packages for the reference tree: the modules load from their files, but the
    # package __init__ files (which pull in the whole trainer) are not executed.
    for pkg in ("gs_dft", "gs_dft.coulomb", "gs_dft.screening", "gs_dft.basis",
                "gs_dft.integrals", "gs_dft.ks"):
        m = types.ModuleType(pkg)
        m.__path__ = [REFERENCE_ROOT + "/" + pkg.replace(".", "/")]
        sys.modules[pkg] = m


def load(name: str):
    """Import one reference module by dotted name, e.g. ``gs_dft.coulomb.ri``."""
    install()
    return importlib.import_module(name)


def as_jarr(x):
    return _wrap(np.asarray(x))
