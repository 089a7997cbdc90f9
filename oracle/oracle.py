"""CPU ORACLE — test infrastructure only.

numpy wrappers around liboracle.so (C restatement of the reference CPU
path, kmb_oracle.c) and, when present, _ref/libkmamba_ref.so (the
reference's own C sources compiled in place).  Imported only by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg, as the checker.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libkmamba_ref.so")

f32 = np.float32
lg = C.c_long
vp = C.c_void_p


def build() -> None:
    """Builds liboracle.so (and _ref/ when the reference tree exists)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _p(a):
    return None if a is None else a.ctypes.data


def _f(a):
    return np.ascontiguousarray(a, dtype=f32)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = C.CDLL(ORACLE_SO)
        L.or_scan1d_fwd.argtypes = [vp] * 8 + [lg] * 5 + [C.c_int]
        L.or_scan1d_bwd.argtypes = [vp] * 13 + [lg] * 5
        L.or_scan2d_fwd.argtypes = [vp] * 9 + [lg] * 6
        L.or_scannd_fwd.argtypes = [vp, lg] + [vp] * 7 + [lg] * 4
        L.or_scannd_bwd.argtypes = [vp, lg] + [vp] * 12 + [lg] * 4
        L.or_convnd_fwd.argtypes = [vp, lg, lg, lg] + [vp] * 4
        L.or_convnd_bwd.argtypes = [vp, lg, lg, lg] + [vp] * 6
        L.or_wavefront_plan.argtypes = [vp, lg, vp, vp]
        L.or_wavefront_plan.restype = lg
        _lib = L
    return _lib


def has_ref() -> bool:
    return os.path.exists(REF_SO)


_ref = None


def ref_lib():
    """The reference's own C path (None when it was never built)."""
    global _ref
    if _ref is None and has_ref():
        _ref = C.CDLL(REF_SO)
    return _ref


# --------------------------------------------------------------------------
# 1D
# --------------------------------------------------------------------------

def scan1d_fwd(x, dt, A, B, C_, h0=None, clamp=True, shared=False, want_h_all=False):
    """One batch item.  x, dt [L,D]; A [D,M]; B, C [L,M] if shared else
    [L,D,M].  Returns (y [L,D], h_last [D,M], h_all [L,D,M] or None)."""
    x, dt, A, B, C_ = map(_f, (x, dt, A, B, C_))
    L, D = x.shape
    M = A.shape[1]
    h = np.zeros((D, M), f32) if h0 is None else _f(h0).copy()
    y = np.empty((L, D), f32)
    h_all = np.empty((L, D, M), f32) if want_h_all else None
    sBt, sBd = (M, 0) if shared else (D * M, M)
    lib().or_scan1d_fwd(_p(x), _p(dt), _p(A), _p(B), _p(C_), _p(h), _p(y), _p(h_all),
                        L, D, M, sBt, sBd, 1 if clamp else 0)
    return y, h, h_all


def scan1d_bwd(x, dt, A, B, C_, h_all, dy, h0=None, shared=False):
    """Reverse adjoint of the reference (cpu/scan1d_backward.c).  Returns
    dx, ddt [L,D]; dA [D,M]; dB, dC shaped like B."""
    x, dt, A, B, C_, h_all, dy = map(_f, (x, dt, A, B, C_, h_all, dy))
    L, D = x.shape
    M = A.shape[1]
    sBt, sBd = (M, 0) if shared else (D * M, M)
    dx = np.empty((L, D), f32)
    ddt = np.empty((L, D), f32)
    dA = np.empty((D, M), f32)
    dB = np.empty(B.shape, f32)
    dC = np.empty(B.shape, f32)
    h0 = None if h0 is None else _f(h0)
    lib().or_scan1d_bwd(_p(x), _p(dt), _p(A), _p(B), _p(C_), _p(h0), _p(h_all), _p(dy),
                        _p(dx), _p(ddt), _p(dA), _p(dB), _p(dC), L, D, M, sBt, sBd)
    return dx, ddt, dA, dB, dC


# --------------------------------------------------------------------------
# 2D / ND
# --------------------------------------------------------------------------

def scan2d_fwd(x, A1, A2, B, C_, dt1, dt2, d1, d2, shared=False):
    """scan2d asm order.  x, dt [P,D]; A [D,M]; B, C [P,M] or [P,D,M]."""
    x, A1, A2, B, C_, dt1, dt2 = map(_f, (x, A1, A2, B, C_, dt1, dt2))
    P, D = x.shape
    M = A1.shape[1]
    h = np.zeros((P, D, M), f32)
    y = np.empty((P, D), f32)
    sBp, sBd = (M, 0) if shared else (D * M, M)
    lib().or_scan2d_fwd(_p(x), _p(A1), _p(A2), _p(B), _p(C_), _p(dt1), _p(dt2), _p(h),
                        _p(y), d1, d2, D, M, sBp, sBd)
    return y, h


def scannd_fwd(dims, x, A, B, C_, delta, shared=False):
    """scannd_ref order.  x [P,D]; A [nd,D,M]; delta [nd,P,D]."""
    dims = np.ascontiguousarray(dims, dtype=np.int64)
    x, A, B, C_, delta = map(_f, (x, A, B, C_, delta))
    P, D = x.shape
    M = A.shape[2]
    h = np.zeros((P, D, M), f32)
    y = np.empty((P, D), f32)
    sBp, sBd = (M, 0) if shared else (D * M, M)
    lib().or_scannd_fwd(_p(dims), len(dims), _p(x), _p(A), _p(B), _p(C_), _p(delta), _p(h),
                        _p(y), D, M, sBp, sBd)
    return y, h


def scannd_bwd(dims, x, A, B, C_, delta, h, dy, shared=False):
    """Adjoint of scannd_fwd.  Returns dx, dA, dB, dC, ddelta."""
    dims = np.ascontiguousarray(dims, dtype=np.int64)
    x, A, B, C_, delta, h, dy = map(_f, (x, A, B, C_, delta, h, dy))
    P, D = x.shape
    nd, _, M = A.shape
    sBp, sBd = (M, 0) if shared else (D * M, M)
    dx = np.empty((P, D), f32)
    dA = np.empty(A.shape, f32)
    dB = np.empty(B.shape, f32)
    dC = np.empty(B.shape, f32)
    ddelta = np.empty(delta.shape, f32)
    lib().or_scannd_bwd(_p(dims), nd, _p(x), _p(A), _p(B), _p(C_), _p(delta), _p(h), _p(dy),
                        _p(dx), _p(dA), _p(dB), _p(dC), _p(ddelta), D, M, sBp, sBd)
    return dx, dA, dB, dC, ddelta


# --------------------------------------------------------------------------
# ConvND and plans
# --------------------------------------------------------------------------

def convnd_fwd(dims, K, inp, kernel, bias=None):
    dims = np.ascontiguousarray(dims, dtype=np.int64)
    inp, kernel = _f(inp), _f(kernel)
    bias = None if bias is None else _f(bias)
    P, D = inp.shape
    out = np.empty((P, D), f32)
    lib().or_convnd_fwd(_p(dims), len(dims), D, K, _p(inp), _p(kernel), _p(bias), _p(out))
    return out


def convnd_bwd(dims, K, inp, kernel, dy, with_bias=True):
    dims = np.ascontiguousarray(dims, dtype=np.int64)
    inp, kernel, dy = _f(inp), _f(kernel), _f(dy)
    P, D = inp.shape
    din = np.empty((P, D), f32)
    dk = np.empty(kernel.shape, f32)
    db = np.empty((D,), f32) if with_bias else None
    lib().or_convnd_bwd(_p(dims), len(dims), D, K, _p(inp), _p(kernel), _p(dy), _p(din),
                        _p(dk), _p(db))
    return din, dk, db


def wavefront_plan(dims):
    """(level_starts [max_level+2], level_offsets [P]) as int64 arrays."""
    dims = np.ascontiguousarray(dims, dtype=np.int64)
    P = int(np.prod(dims))
    maxl = int(np.sum(dims - 1))
    ls = np.empty(maxl + 2, np.int64)
    lo = np.empty(P, np.int64)
    lib().or_wavefront_plan(_p(dims), len(dims), _p(ls), _p(lo))
    return ls, lo
