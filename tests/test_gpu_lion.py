"""GPU parity of the reference op apply_cheby_rkv_v10 (full path: chunked
forward + local TTT gradient + Lion, one launch) and of its fast path, against
the reference's golden outputs and the oracle.

Outputs are bf16-rounded by the reference (sdpc_kernel.py:2422, 2433), so
they are compared at bf16 resolution.  Coefficients after Lion match except
where sign(b1*m + (1-b1)*g) sits at rounding level; such flips move one
coefficient by at most 2*lr*(k+1)^-1.5 and are counted, not hidden.
"""
import numpy as np
import pytest
import torch

from oracle import cheby_ref as R
from tests.golden.inputs import det_normal, spectral_coeffs
from tests.test_oracle_golden import load, relerr

pytestmark = pytest.mark.gpu
dev = "cuda"


def T(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)


def N(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def apply(x, c, m, **kw):
    import orthossm_b200 as O
    with torch.no_grad():
        return O.apply_cheby_rkv_v10(T(x), T(c), T(m), **kw)


def check_lion(c_new, m_new, c_ref, m_ref, lr_max, max_flip_frac=0.01):
    diff = np.abs(N(c_new) - c_ref)
    flips = diff > 1e-5
    assert flips.mean() <= max_flip_frac, flips.mean()
    assert np.all(diff[flips] <= 2.0 * lr_max * 1.01)
    assert np.abs(N(c_new) - c_ref)[~flips].max(initial=0) < 1e-5
    assert relerr(N(m_new), m_ref) < 1e-3


def check_out(out, ref):
    o = N(out)
    assert out.dtype == torch.float32
    assert np.array_equal(o, R.bf16_round(o))  # bf16-rounded values, as the reference returns
    assert np.abs(o - ref).max() <= 2 ** -7
    assert relerr(o, ref) < 2e-3


def test_golden_lut_deg8_with_gates_multi_chunk():
    g = load("mega_lut_deg8_gates")
    x = det_normal((2, 600, 64), 151)
    c = spectral_coeffs(2, 8, 8, 8, 152, scale=0.5)
    m = det_normal((2, 8, 8, 8), 153, 0.01)
    out, cn, mn = apply(x, c, m, n_heads=8, seq_threshold=0, chunk_size=256, use_lut=True,
                        gate_global=T(g["gate_global"]), dynamic_lambda=T(g["dynamic_lambda"]))
    check_out(out, g["out"])
    check_lion(cn, mn, g["c_new"], g["m_new"], 0.005 * 1.25)


def test_golden_clenshaw_deg8_truncation():
    g = load("mega_clenshaw_deg8")
    x = det_normal((2, 256, 64), 161)
    c = spectral_coeffs(2, 8, 8, 8, 162, scale=0.5)
    m = np.zeros((2, 8, 8, 8), np.float32)
    out, cn, mn = apply(x, c, m, n_heads=8, seq_threshold=0, chunk_size=256, use_lut=False)
    check_out(out, g["out"])
    check_lion(cn, mn, g["c_new"], g["m_new"], 0.005 * 1.25)


def test_golden_deg4_four_chunks():
    g = load("mega_deg4_chunks")
    x = det_normal((1, 512, 128), 171)
    c = spectral_coeffs(1, 8, 4, 16, 172, scale=0.5)
    m = np.zeros((1, 8, 4, 16), np.float32)
    out, cn, mn = apply(x, c, m, n_heads=8, seq_threshold=0, chunk_size=128, use_lut=True,
                        ema_momentum=0.85, base_lr=0.01)
    check_out(out, g["out"])
    check_lion(cn, mn, g["c_new"], g["m_new"], 0.01 * 1.25)


def test_golden_fast_path_routing():
    g = load("fast_path")
    x = det_normal((2, 100, 64), 181)
    c = spectral_coeffs(2, 8, 4, 8, 182)
    m = np.zeros((2, 8, 4, 8), np.float32)
    out, cn, mn = apply(x, c, m, n_heads=8, ema_momentum=0.9)
    assert relerr(N(out), g["out"]) < 1e-5
    assert np.array_equal(N(cn), c.astype(np.float64))  # fast path: no TTT


@pytest.mark.parametrize("B,S,D,H,K,chunk", [(2, 1024, 128, 8, 8, 256), (1, 2048, 512, 8, 8, 256),
                                             (3, 1000, 64, 4, 4, 300), (1, 257, 64, 8, 8, 256),
                                             (2, 700, 256, 8, 6, 2048),
                                             (3, 600, 512, 8, 8, 256)])  # 192 CTAs: one warp per channel
def test_oracle_shapes(B, S, D, H, K, chunk):
    x = det_normal((B, S, D), 200 + S)
    c = spectral_coeffs(B, H, K, D // H, 201, scale=0.5)
    m = det_normal((B, H, K, D // H), 202, 0.005)
    out, cn, mn = apply(x, c, m, n_heads=H, seq_threshold=0, chunk_size=chunk)
    ro, rc, rm = R.apply_cheby_rkv_v10(x, c, m, n_heads=H, seq_threshold=0, chunk_size=chunk)
    check_out(out, ro)
    check_lion(cn, mn, rc, rm, 0.005 * 1.25)


def test_one_token_last_chunk_stays_finite():
    """S = chunk + 1: the reference divides by zero in the 1-token chunk and
    writes NaN momentum; here that chunk contributes no gradient."""
    x = det_normal((1, 257, 64), 210)
    c = spectral_coeffs(1, 8, 8, 8, 211, scale=0.5)
    m = np.zeros((1, 8, 8, 8), np.float32)
    out, cn, mn = apply(x, c, m, n_heads=8, seq_threshold=0, chunk_size=256)
    assert np.isfinite(N(mn)).all() and np.isfinite(N(cn)).all()
    ro, rc, rm = R.apply_cheby_rkv_v10(x, c, m, n_heads=8, seq_threshold=0, chunk_size=256)
    check_lion(cn, mn, rc, rm, 0.005 * 1.25)


def test_inputs_not_mutated_and_bf16_input():
    x = det_normal((2, 512, 64), 220)
    c = spectral_coeffs(2, 8, 8, 8, 221, scale=0.5)
    m = np.zeros((2, 8, 8, 8), np.float32)
    xt, ct, mt = T(x), T(c), T(m)
    c0, m0 = ct.clone(), mt.clone()
    import orthossm_b200 as O
    with torch.no_grad():
        o1, c1, m1 = O.apply_cheby_rkv_v10(xt, ct, mt, n_heads=8, seq_threshold=0)
        o2, c2, m2 = O.apply_cheby_rkv_v10(xt.to(torch.bfloat16), ct, mt, n_heads=8, seq_threshold=0)
    assert torch.equal(ct, c0) and torch.equal(mt, m0)
    # the reference casts x to bf16 first: bf16 input gives the same result
    assert torch.equal(o1, o2) and torch.equal(c1, c2) and torch.equal(m1, m2)


def test_deterministic():
    x = det_normal((2, 1500, 128), 230)
    c = spectral_coeffs(2, 8, 8, 16, 231, scale=0.5)
    m = np.zeros((2, 8, 8, 16), np.float32)
    a = apply(x, c, m, n_heads=8, seq_threshold=0)
    b = apply(x, c, m, n_heads=8, seq_threshold=0)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
