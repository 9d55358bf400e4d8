"""The coefficient-state initialiser init_chebyshev_coefficients
(sdpc_kernel.py:1833-1867): c ~ N(0, (0.1/(k+1))^2) per degree k, then the
heads of each sequence made orthogonal by QR with their norms kept (or, when
degree*head_dim < n_heads, a Parseval tight frame by SVD).

Pinned to the reference's own outputs under the same torch seeds
(tests/golden/init_coeffs.npz, made by make_init_golden.py), and checked for
the properties callers rely on.  CPU only."""
import os

import numpy as np
import pytest
import torch

from orthossm_b200.sdpc_kernel import init_chebyshev_coefficients

GOLD = os.path.join(os.path.dirname(__file__), "golden", "init_coeffs.npz")


def _cases():
    g = np.load(GOLD)
    return [(k, g[k], g[k + "__meta"]) for k in g.files if not k.endswith("__meta")]


@pytest.mark.parametrize("name,ref,meta", _cases(), ids=lambda v: v if isinstance(v, str) else "")
def test_matches_reference_under_the_same_seed(name, ref, meta):
    seed, B, H, deg, hd = (int(v) for v in meta)
    torch.manual_seed(seed)
    c = init_chebyshev_coefficients(B, H, deg, hd, "cpu").numpy()
    assert c.shape == ref.shape == (B, H, deg, hd)
    np.testing.assert_allclose(c, ref, rtol=1e-5, atol=1e-7)


def test_heads_orthogonal_with_spectral_scale():
    """At the BASELINE state shape [B, 8, 8, 64]: every sequence's 8 heads are
    orthogonal as 512-vectors, and the per-degree spread stays
    0.1/(k+1) (the QR changes directions by about 1/sqrt(512) only)."""
    torch.manual_seed(5)
    B, H, K, hd = 64, 8, 8, 64
    c = init_chebyshev_coefficients(B, H, K, hd, "cpu")
    flat = c.reshape(B, H, K * hd).double()
    gram = flat @ flat.transpose(1, 2)
    diag = torch.diagonal(gram, dim1=1, dim2=2)
    off = gram - torch.diag_embed(diag)
    assert float(off.abs().max() / diag.min()) < 1e-5
    std = c.permute(2, 0, 1, 3).reshape(K, -1).std(dim=1)
    want = 0.1 / torch.arange(1, K + 1, dtype=torch.float32)
    assert torch.allclose(std, want, rtol=0.05), (std, want)


def test_single_head_is_plain_spectral_draw():
    torch.manual_seed(3)
    c = init_chebyshev_coefficients(2, 1, 8, 64, "cpu")
    torch.manual_seed(3)
    sigma = (0.1 / (torch.arange(8, dtype=torch.float32) + 1.0)).view(1, 1, 8, 1)
    assert torch.equal(c, torch.randn(2, 1, 8, 64) * sigma)
