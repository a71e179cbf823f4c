"""TEST INFRASTRUCTURE ONLY -- ctypes binding of oracle/_ref/libvkbref.so, the reference's own host model compiled
from its source by oracle/Makefile (see oracle/ref_shim.cu). Used to generate the golden fixtures, to pin the numpy
oracle, and as the timed CPU baseline ("kind": "reference"). Returns None from load() when the library is absent
(e.g. a checkout where the reference source was not available to build it)."""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libvkbref.so")
_lib = None


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            return None
        L = ctypes.CDLL(LIB_PATH)
        vp, i, u = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint
        L.ref_rng_new.restype = vp
        L.ref_rng_new.argtypes = [u]
        L.ref_rng_free.argtypes = [vp]
        L.ref_rng_next.restype = u
        L.ref_rng_next.argtypes = [vp]
        L.ref_make_weights.argtypes = [vp, i, i, i, vp, vp]
        L.ref_make_q2.argtypes = [vp, i, i, vp, vp]
        L.ref_uniform_x.argtypes = [vp, ctypes.c_size_t, ctypes.c_float, vp]
        L.ref_bigx.argtypes = [vp, i, i, vp]
        L.ref_pack_q4.argtypes = [i, i, vp, vp, i, vp]
        L.ref_pack_q2_rowmajor.argtypes = [i, i, vp, vp, i, vp]
        L.ref_values.argtypes = [i, i, i, vp, vp, vp, vp, vp]
        L.ref_q2_values.argtypes = [i, i, vp, vp, vp, vp, vp]
        L.ref_gemv_mt.restype = ctypes.c_double
        L.ref_gemv_mt.argtypes = [i, i, i, vp, vp, vp, i, i, i, vp]
        L.oracle_synth_normal.argtypes = [u, ctypes.c_size_t, ctypes.c_float, vp]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


class Rng:
    """The reference's std::mt19937, advanced by its own generators."""

    def __init__(self, seed: int):
        self.L = load()
        self.h = ctypes.c_void_p(self.L.ref_rng_new(seed))

    def __del__(self):
        if getattr(self, "h", None) is not None and self.L is not None:
            self.L.ref_rng_free(self.h)
            self.h = None

    def make_weights(self, N: int, K: int, bits: int):
        codes = np.empty((N, K), np.int8)
        scales = np.empty((N, K // 32), np.uint16)
        self.L.ref_make_weights(self.h, N, K, bits, _p(codes), _p(scales))
        return codes, scales

    def make_q2(self, N: int, K: int):
        codes = np.empty((N, K), np.int8)
        scales = np.empty((N, K // 32), np.uint16)
        self.L.ref_make_q2(self.h, N, K, _p(codes), _p(scales))
        return codes, scales

    def uniform_x(self, M: int, K: int, mul: float = 1.0):
        x = np.empty((M, K), np.uint16)
        self.L.ref_uniform_x(self.h, M * K, mul, _p(x))
        return x

    def bigx(self, x: np.ndarray):
        self.L.ref_bigx(self.h, x.shape[0], x.shape[1], _p(x))
        return x


def pack_q4(codes, scales, sabotage=False):
    L = load()
    N, K = codes.shape
    out = np.empty((N, K // 8), np.uint32)
    L.ref_pack_q4(N, K, _p(np.ascontiguousarray(codes)), _p(np.ascontiguousarray(scales)), int(sabotage), _p(out))
    return out


def pack_q2(codes, scales, sabotage=False):
    L = load()
    N, K = codes.shape
    out = np.empty((N, K // 16), np.uint32)
    L.ref_pack_q2_rowmajor(N, K, _p(np.ascontiguousarray(codes)), _p(np.ascontiguousarray(scales)), int(sabotage),
                           _p(out))
    return out


def values(codes, scales, x):
    L = load()
    N, K = codes.shape
    M = x.shape[0]
    val = np.empty((M, N))
    mag = np.empty((M, N))
    L.ref_values(N, K, M, _p(np.ascontiguousarray(codes)), _p(np.ascontiguousarray(scales)),
                 _p(np.ascontiguousarray(x)), _p(val), _p(mag))
    return val, mag


def q2_values(codes, scales, x):
    L = load()
    N, K = codes.shape
    val = np.empty(N)
    mag = np.empty(N)
    L.ref_q2_values(N, K, _p(np.ascontiguousarray(codes)), _p(np.ascontiguousarray(scales)),
                    _p(np.ascontiguousarray(x)), _p(val), _p(mag))
    return val, mag


def synth_normal(seed: int, shape, std: float) -> np.ndarray:
    """The benchmark's seeded normal draws (mt19937 + Box-Muller), float32, without libvkb.so."""
    out = np.empty(int(np.prod(shape)), np.float32)
    load().oracle_synth_normal(seed, out.size, std, _p(out))
    return out.reshape(shape)


def gemv_mt(codes, scales, x, row0: int, nrows: int, threads: int, out=None) -> float:
    """The reference's ref_value over rows [row0, row0+nrows) x all tokens on `threads` host threads."""
    L = load()
    N, K = codes.shape
    M = x.shape[0]
    return L.ref_gemv_mt(N, K, M, _p(codes), _p(scales), _p(x), row0, nrows, threads,
                         _p(out) if out is not None else None)
