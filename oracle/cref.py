"""ctypes wrapper of the oracle's C port (oracle/cheby_ref.c) — test / CPU
baseline infrastructure only."""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libossm_oracle.so")
_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        l = C.CDLL(LIB)
        l.ossm_ref_fwd.restype = C.c_int
        l.ossm_ref_fwd.argtypes = [C.c_int] * 5 + [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_float,
                                                    C.c_void_p, C.c_void_p, C.c_float, C.c_float, C.c_float,
                                                    C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int]
        l.ossm_ref_max_threads.restype = C.c_int
        _lib = l
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def max_threads():
    return lib().ossm_ref_max_threads()


def forward(x, coeffs, *, lam=None, momentum=0.9, gate=None, init=None, out_bf16=False, nthreads=0,
            x_is_bf16_bits=False, out=None, fin=None):
    """x: float32 [B,S,D] or uint16 bf16 bits (x_is_bf16_bits).  Returns (out, fin);
    bf16 output is returned as uint16 bits."""
    B, S, D = x.shape
    c = np.ascontiguousarray(coeffs, np.float32)
    H, K, HD = c.shape[1], c.shape[2], c.shape[3]
    x = np.ascontiguousarray(x)
    lam_a = None if lam is None else np.ascontiguousarray(lam, np.float32)
    gw = gb = None
    gs, glo, ghi = 0.008, 0.0, 1.0
    if gate is not None:
        gw = np.ascontiguousarray(gate["W"], np.float32)
        gb = np.ascontiguousarray(gate["b"], np.float32)
        gs, glo, ghi = gate.get("scale", 0.008), gate.get("lo", 0.0), gate.get("hi", 1.0)
    ini = None if init is None else np.ascontiguousarray(init, np.float32)
    if out is None:
        out = np.empty((B, S, D), np.uint16 if out_bf16 else np.float32)
    if fin is None:
        fin = np.empty((B, D), np.float32)
    rc = lib().ossm_ref_fwd(B, S, H, HD, K, _p(x), int(x_is_bf16_bits), _p(c), _p(lam_a), float(momentum),
                            _p(gw), _p(gb), gs, glo, ghi, _p(ini), _p(out), int(out_bf16), _p(fin),
                            int(nthreads))
    if rc != 0:
        raise ValueError("ossm_ref_fwd: bad arguments")
    return out, fin


def bf16_bits_to_f32(u):
    return (np.asarray(u, np.uint32) << 16).view(np.float32)
