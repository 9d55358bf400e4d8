"""Deterministic, platform-independent synthetic inputs for fixtures and tests.

A counter-based hash (splitmix64 finaliser) gives uniform bits for element
index i of stream ``seed``; Box-Muller turns pairs into normals.  The same
seed and shape give the same values on any machine and numpy version, so
golden fixtures store only the reference's outputs, not the inputs.
"""
from __future__ import annotations

import numpy as np

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_G = np.uint64(0x9E3779B97F4A7C15)


def _mix(z):
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def det_uniform(n, seed):
    """n uniforms in (0, 1) as float64 from stream ``seed``."""
    i = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = _mix((i + np.uint64(1)) * _G + np.uint64(seed) * np.uint64(0xD1B54A32D192ED03))
    return ((z >> np.uint64(11)).astype(np.float64) + 0.5) / float(1 << 53)


def det_normal(shape, seed, std=1.0, dtype=np.float32):
    """Normal(0, std^2) array of ``shape`` from stream ``seed``."""
    n = int(np.prod(shape))
    m = (n + 1) // 2
    u = det_uniform(2 * m, seed)
    r = np.sqrt(-2.0 * np.log(u[:m]))
    th = 2.0 * np.pi * u[m:]
    z = np.concatenate([r * np.cos(th), r * np.sin(th)])[:n]
    return (z * std).reshape(shape).astype(dtype)


def spectral_coeffs(B, H, K, hd, seed, scale=1.0):
    """c[b,h,k,j] ~ N(0, (scale/(k+1))^2) — BASELINE.json configs[0]."""
    c = det_normal((B, H, K, hd), seed, 1.0, np.float64)
    c = c * (scale / (np.arange(K) + 1.0))[None, None, :, None]
    return c.astype(np.float32)


def linear_init(out_f, in_f, seed):
    """nn.Linear-style init U(-1/sqrt(in), 1/sqrt(in)) for W [out,in] and b [out]."""
    bound = 1.0 / np.sqrt(in_f)
    W = (det_uniform(out_f * in_f, seed) * 2.0 - 1.0) * bound
    b = (det_uniform(out_f, seed + 7919) * 2.0 - 1.0) * bound
    return W.reshape(out_f, in_f).astype(np.float32), b.astype(np.float32)
