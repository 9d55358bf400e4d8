"""The oracle's W_pred MSE TTT gradient (no reference
code: parity unpinned) against central finite differences of its own loss, on
CPU.  Pins the hand-written reverse EMA adjoint, the tanh/clamp chain rule and
the Chebyshev basis in float64."""
import numpy as np
import pytest

from oracle import cheby_ref as R


def _loss(x, c, W, lam, gate):
    _, _, loss = R.wpred_chunk_grad(x, c, W, lam, gate=gate, spectral_pow=0.0)
    return loss.sum()


@pytest.mark.parametrize("gated", [False, True])
def test_wpred_gradient_matches_finite_differences(gated):
    rng = np.random.default_rng(7)
    B, L, H, hd, K = 2, 9, 2, 4, 8
    D = H * hd
    x = rng.normal(size=(B, L, D))
    c = rng.normal(size=(B, H, K, hd)) / (np.arange(K) + 1.0)[None, None, :, None]
    W = rng.normal(size=(D, D)) * 0.3
    lam = np.array([0.9, 0.6])
    gate = dict(W=rng.normal(size=(H, D)) * 0.1, b=np.zeros(H)) if gated else None
    _, g, _ = R.wpred_chunk_grad(x, c, W, lam, gate=gate, spectral_pow=0.0)
    eps = 1e-6
    for idx in [(0, 0, 0, 0), (1, 1, 3, 2), (0, 1, 7, 3), (1, 0, 5, 1)]:
        cp, cm = c.copy(), c.copy()
        cp[idx] += eps
        cm[idx] -= eps
        fd = (_loss(x, cp, W, lam, gate) - _loss(x, cm, W, lam, gate)) / (2 * eps)
        assert abs(fd - g[idx]) <= 1e-6 + 1e-5 * abs(fd), (idx, fd, g[idx])


def test_wpred_spectral_scaling():
    rng = np.random.default_rng(8)
    B, L, H, hd, K = 1, 6, 2, 4, 8
    D = H * hd
    x = rng.normal(size=(B, L, D))
    c = rng.normal(size=(B, H, K, hd)) * 0.3
    W = rng.normal(size=(D, D)) * 0.3
    lam = np.array([0.9, 0.8])
    _, g0, _ = R.wpred_chunk_grad(x, c, W, lam, spectral_pow=0.0)
    _, g2, _ = R.wpred_chunk_grad(x, c, W, lam, spectral_pow=2.0)
    k = np.arange(K) + 1.0
    np.testing.assert_allclose(g2, g0 / (k ** 2)[None, None, :, None], rtol=1e-12)
