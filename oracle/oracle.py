"""ctypes wrapper of liboracle.so — TEST INFRASTRUCTURE ONLY.

The oracle is a CPU restatement of the reference forward pass (oracle.cpp). It is the checker for the CUDA path
and the timed CPU baseline; the product never calls it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            subprocess.check_call(["make", "-s", "-C", HERE])
        L = ctypes.CDLL(path)
        L.orc_load.restype = ctypes.c_void_p
        L.orc_load.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_int]
        L.orc_free.argtypes = [ctypes.c_void_p]
        L.orc_dims.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
        fp = ctypes.POINTER(ctypes.c_float)
        L.orc_forward.argtypes = [ctypes.c_void_p, ctypes.c_int, fp, fp, fp, ctypes.c_int, ctypes.c_int,
                                  fp, fp, fp, fp, ctypes.c_char_p, ctypes.c_int]
        L.orc_forward.restype = ctypes.c_int
        _LIB = L
    return _LIB


def _fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class OracleNet:
    """A parsed model; `forward` returns the raw outputs (policy [N,P,362], value [N,3], scorevalue [N,Sv],
    ownership [N,1,19,19]) exactly as the reference graph names them."""

    def __init__(self, data: bytes):
        err = ctypes.create_string_buffer(512)
        self.h = lib().orc_load(data, len(data), err, 512)
        if not self.h:
            raise ValueError(err.value.decode())
        d = (ctypes.c_int * 9)()
        lib().orc_dims(self.h, d)
        (self.version, self.n_in, self.n_glob, self.n_meta, self.P, self.n_value, self.n_score, self.n_own,
         self.trunk_c) = list(d)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_free(self.h)
            self.h = None

    def forward(self, spatial, glob, meta=None, double=False, threads=0):
        n = spatial.shape[0]
        spatial = np.ascontiguousarray(spatial, np.float32)
        glob = np.ascontiguousarray(glob, np.float32)
        meta = np.ascontiguousarray(meta if meta is not None and meta.size else np.zeros((n, max(1, self.n_meta))),
                                    np.float32)
        pol = np.zeros((n, self.P, 362), np.float32)
        val = np.zeros((n, self.n_value), np.float32)
        sc = np.zeros((n, self.n_score), np.float32)
        own = np.zeros((n, self.n_own, 19, 19), np.float32)
        err = ctypes.create_string_buffer(512)
        rc = lib().orc_forward(self.h, n, _fp(spatial), _fp(glob), _fp(meta), int(double), int(threads),
                               _fp(pol), _fp(val), _fp(sc), _fp(own), err, 512)
        if rc != 0:
            raise RuntimeError(err.value.decode())
        return {"policy": pol, "value": val, "scorevalue": sc, "ownership": own}
