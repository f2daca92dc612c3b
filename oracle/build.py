"""Build the C oracle (oracle/c/hxm_oracle.c -> oracle/lib/libhxm_oracle.so)
and expose it through ctypes.  TEST INFRASTRUCTURE ONLY (see __init__.py).

The reference is pure Python (torch loops + Triton), so there is no
compiled reference to build into oracle/_ref; the oracle is this C
restatement plus the numpy one, pinned by the golden vectors.
"""
from __future__ import annotations

import ctypes as ct
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "c", "hxm_oracle.c")
LIB = os.path.join(HERE, "lib", "libhxm_oracle.so")


def build(force: bool = False) -> str:
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    if force or not os.path.exists(LIB) or os.path.getmtime(SRC) > os.path.getmtime(LIB):
        cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-o", LIB, SRC, "-lm"]
        subprocess.run(cmd, check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        l = ct.CDLL(LIB)
        fp = ct.POINTER(ct.c_float)
        l.hxm_oracle_scan.argtypes = [ct.c_int] * 4 + [fp] * 8 + [ct.c_int] * 3 + [fp, fp, fp]
        l.hxm_oracle_mlstm.argtypes = [ct.c_int] * 4 + [fp] * 5 + [ct.c_int, fp, fp, fp]
        l.hxm_oracle_slstm.argtypes = [ct.c_int] * 4 + [fp] * 3 + [ct.c_float, ct.c_int, fp, fp, fp]
        l.hxm_oracle_max_threads.restype = ct.c_int
        l.hxm_oracle_set_threads.argtypes = [ct.c_int]
        # all host threads (a launcher may have pinned OMP_NUM_THREADS to 1)
        l.hxm_oracle_set_threads(len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count())
        _lib = l
    return _lib


def _p(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ct.POINTER(ct.c_float))


def f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def scan(u, dt, A, B, C, D=None, z=None, bias=None, softplus=False, z_mode=0, disc=0, h0=None):
    """Time-major scan: u, dt, z (b, d, L); B, C (b, n, L); returns y (b,d,L), hT (b,d,n)."""
    u, dt, A, B, C, D, z, bias, h0 = map(f32, (u, dt, A, B, C, D, z, bias, h0))
    b, d, L = u.shape
    n = A.shape[1]
    y = np.empty_like(u)
    hT = np.empty((b, d, n), np.float32)
    lib().hxm_oracle_scan(b, L, d, n, _p(u), _p(dt), _p(A), _p(B), _p(C), _p(D), _p(z), _p(bias),
                          int(softplus), z_mode, disc, _p(h0), _p(y), _p(hT))
    return y, hT


def mlstm(q, k, v, ig, fg, C0=None, n0=None):
    """q, k (b, h, L, dk), v (b, h, L, dv); ig, fg activated gates (b,h,L) or (b,h,L,dk)."""
    q, k, v, ig, fg = map(f32, (q, k, v, ig, fg))
    b, nh, L, dk = q.shape
    dv = v.shape[-1]
    C = np.zeros((b, nh, dk, dv), np.float32) if C0 is None else f32(C0).copy()
    n = np.zeros((b, nh, dk), np.float32) if n0 is None else f32(n0).copy()
    h = np.empty((b, nh, L, dv), np.float32)
    lib().hxm_oracle_mlstm(b * nh, L, dk, dv, _p(q), _p(k), _p(v), _p(ig), _p(fg), int(ig.ndim == 4), _p(h),
                           _p(C), _p(n))
    return h, C, n


def slstm(g, w, R=None, eps=1e-6, exp_gate=True, h0=None, c0=None):
    g, w, R = f32(g), f32(w), f32(R)
    b, L, nh, _, hd = g.shape
    h = np.zeros((b, nh, hd), np.float32) if h0 is None else f32(h0).copy()
    c = np.zeros((b, nh, hd), np.float32) if c0 is None else f32(c0).copy()
    out = np.empty((b, L, nh, hd), np.float32)
    lib().hxm_oracle_slstm(b, L, nh, hd, _p(g), _p(R), _p(w), float(eps), int(exp_gate), _p(out), _p(h), _p(c))
    return out, h, c


if __name__ == "__main__":
    print(build(force=True))
