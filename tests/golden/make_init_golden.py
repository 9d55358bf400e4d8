"""Golden fixture for the coefficient-state initialiser.

Runs the reference's own ``sdpc_kernel.init_chebyshev_coefficients``
(``sdpc_kernel.py:1833-1867``: per-degree sigma 0.1/(k+1), heads made
orthogonal by QR, or a Parseval tight frame by SVD when degree*head_dim <
n_heads) on CPU under fixed torch seeds, and stores its outputs with the seeds
in ``tests/golden/init_coeffs.npz``.  Needs the reference checkout (``--ref``
or the ``OSSM_REFERENCE`` environment variable); it is run once, offline, and
its output is committed.  Tests never import the reference.

    python tests/golden/make_init_golden.py --ref <path-to-OrthoSSM>
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, seed, batch, n_heads, degree, head_dim): the QR branch at the
# BASELINE state shape and a small one, the tight-frame branch, one head
CASES = (
    ("qr_b2_h8_k8_d64", 11, 2, 8, 8, 64),
    ("qr_b3_h4_k4_d16", 12, 3, 4, 4, 16),
    ("frame_b2_h8_k2_d2", 13, 2, 8, 2, 2),
    ("one_head_b2_h1_k8_d8", 14, 2, 1, 8, 8),
)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("OSSM_REFERENCE"))
    args = ap.parse_args()
    if not args.ref:
        raise SystemExit("--ref (or OSSM_REFERENCE) must point at the OrthoSSM checkout")
    sys.path.insert(0, args.ref)
    import torch
    import sdpc_kernel as K
    out = {}
    for name, seed, B, H, deg, hd in CASES:
        torch.manual_seed(seed)
        c = K.init_chebyshev_coefficients(B, H, deg, hd, "cpu")
        out[name] = c.numpy().astype(np.float32)
        out[name + "__meta"] = np.asarray([seed, B, H, deg, hd], np.int64)
    path = os.path.join(HERE, "init_coeffs.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


if __name__ == "__main__":
    main()
