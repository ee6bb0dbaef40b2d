"""ctypes wrapper of the C oracle ``libmrorc.so`` (test infrastructure only).

Arrays are converted to contiguous float32 numpy; outputs are allocated
here. Used by the tests at sizes beyond the float64 numpy oracle and as the
timed CPU baseline of bench.py.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

import build_oracle

_lib = None


def lib():
    global _lib
    if _lib is None:
        build_oracle.build()
        _lib = ctypes.CDLL(build_oracle.OUT)
    return _lib


def _f(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def _p(x):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def _i(*v):
    return [ctypes.c_int64(int(x)) for x in v]


def ssd(u, delta, B, C, A, seg, gy=None, g_final=None):
    u, delta, B, C = map(_f, (u, delta, B, C))
    Bt, L, H, Dh = u.shape
    N = B.shape[-1]
    A = _f(np.broadcast_to(A, (H, N)))
    y = np.empty_like(u)
    ck = np.empty((Bt, L // seg, H, N, Dh), np.float32)
    lib().orc_ssd_fwd(*map(_p, (u, delta, B, C, A)), *_i(Bt, L, H, Dh, N, seg), _p(y), _p(ck))
    out = {"y": y, "final": ck[:, -1].transpose(0, 1, 3, 2).copy()}
    if gy is not None:
        gy = _f(gy)
        gf = None if g_final is None else _f(g_final)
        gu, gd, gB, gC = (np.empty_like(x) for x in (u, delta, B, C))
        gAp = np.empty((Bt, H, N), np.float32)
        lib().orc_ssd_bwd(_p(gy), _p(gf), _p(ck), *map(_p, (u, delta, B, C, A)),
                          *_i(Bt, L, H, Dh, N, seg), *map(_p, (gu, gd, gB, gC, gAp)))
        out["grads"] = [gu, gd, gB, gC, gAp.sum(0)]
    return out


def gla(q, k, v, g, seg, gy=None, g_final=None):
    q, k, v, g = map(_f, (q, k, v, g))
    Bt, L, H, Dh = q.shape
    y = np.empty_like(q)
    ck = np.empty((Bt, L // seg, H, Dh, Dh), np.float32)
    lib().orc_gla_fwd(*map(_p, (q, k, v, g)), *_i(Bt, L, H, Dh, seg), _p(y), _p(ck))
    out = {"y": y, "final": ck[:, -1].copy()}
    if gy is not None:
        gy = _f(gy)
        gf = None if g_final is None else _f(g_final)
        gq, gk, gv, gg = (np.empty_like(x) for x in (q, k, v, g))
        lib().orc_gla_bwd(_p(gy), _p(gf), _p(ck), *map(_p, (q, k, v, g)), *_i(Bt, L, H, Dh, seg),
                          *map(_p, (gq, gk, gv, gg)))
        out["grads"] = [gq, gk, gv, gg]
    return out


def rglru(a, x, seg, gy=None, g_final=None):
    a, x = map(_f, (a, x))
    Bt, L, D = a.shape
    y = np.empty_like(a)
    ck = np.empty((Bt, L // seg, D), np.float32)
    lib().orc_rglru_fwd(_p(a), _p(x), *_i(Bt, L, D, seg), _p(y), _p(ck))
    out = {"y": y, "final": ck[:, -1].copy()}
    if gy is not None:
        gy = _f(gy)
        gf = None if g_final is None else _f(g_final)
        ga, gx = np.empty_like(a), np.empty_like(x)
        lib().orc_rglru_bwd(_p(gy), _p(gf), _p(ck), _p(a), _p(x), *_i(Bt, L, D, seg), _p(ga), _p(gx))
        out["grads"] = [ga, gx]
    return out


def rotlru(a, cs, sn, x, seg, gy=None, g_final=None):
    a, cs, sn, x = map(_f, (a, cs, sn, x))
    Bt, L, Dp = a.shape
    y = np.empty_like(x)
    ck = np.empty((Bt, L // seg, 2 * Dp), np.float32)
    lib().orc_rotlru_fwd(*map(_p, (a, cs, sn, x)), *_i(Bt, L, Dp, seg), _p(y), _p(ck))
    out = {"y": y, "final": ck[:, -1].copy()}
    if gy is not None:
        gy = _f(gy)
        gf = None if g_final is None else _f(g_final)
        grads = [np.empty_like(t) for t in (a, cs, sn, x)]
        lib().orc_rotlru_bwd(_p(gy), _p(gf), _p(ck), *map(_p, (a, cs, sn, x)), *_i(Bt, L, Dp, seg),
                             *map(_p, grads))
        out["grads"] = grads
    return out


def gdn(q, k, v, alpha, beta, seg, gy=None, g_final=None):
    q, k, v, alpha, beta = map(_f, (q, k, v, alpha, beta))
    Bt, L, H, Dh = q.shape
    y = np.empty_like(q)
    ck = np.empty((Bt, L // seg, H, Dh, Dh), np.float32)
    lib().orc_gdn_fwd(*map(_p, (q, k, v, alpha, beta)), *_i(Bt, L, H, Dh, seg), _p(y), _p(ck))
    out = {"y": y, "final": ck[:, -1].copy()}
    if gy is not None:
        gy = _f(gy)
        gf = None if g_final is None else _f(g_final)
        grads = [np.empty_like(t) for t in (q, k, v, alpha, beta)]
        lib().orc_gdn_bwd(_p(gy), _p(gf), _p(ck), *map(_p, (q, k, v, alpha, beta)), *_i(Bt, L, H, Dh, seg),
                          *map(_p, grads))
        out["grads"] = grads
    return out


def run(kind, ins, seg, gy=None, g_final=None):
    fns = {"ssd": ssd, "gla": gla, "rglru": rglru, "rotlru": rotlru, "gdn": gdn}
    return fns[kind](*ins, seg, gy=gy, g_final=g_final)
