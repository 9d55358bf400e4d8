"""The oracle's C port (oracle/cheby_ref.c, the timed CPU baseline of bench.py)
against the float64 numpy restatement, on CPU.  The port computes in fp32,
so the bar is fp32 accumulation error over the EMA chain."""
import numpy as np
import pytest

from oracle import cheby_ref as R
from oracle import cref
from tests.golden.inputs import det_normal, linear_init, spectral_coeffs
from tests.test_oracle_golden import relerr


def f32(v):
    return np.asarray(v, np.float32).astype(np.float64)


@pytest.mark.parametrize("gate,init,lam_kind", [(False, False, "head"), (True, True, "head"),
                                                 (False, True, "scalar"), (True, False, "head")])
def test_cport_matches_numpy_oracle(gate, init, lam_kind):
    B, S, H, hd = 2, 300, 8, 64
    D = H * hd
    x = R.bf16_round(det_normal((B, S, D), 41)).astype(np.float32)
    c = spectral_coeffs(B, H, 8, hd, 42).astype(np.float32)
    W, b = linear_init(H, D, 43)
    ini = det_normal((B, D), 44, 0.1).astype(np.float32) if init else None
    lam = f32(R.BASELINE_LAMBDA) if lam_kind == "head" else None
    g = dict(W=f32(W), b=f32(b)) if gate else None
    out, fin = cref.forward(x, c, lam=lam, momentum=0.9, gate=g, init=ini, nthreads=2)
    ref = R.cheby_ema_forward(x.astype(np.float64), c.astype(np.float64), lam=lam, momentum=f32(0.9)[()],
                              gate=g, init=None if ini is None else ini.astype(np.float64))
    assert relerr(out, ref["out"]) < 1e-4
    assert relerr(fin, ref["final"]) < 1e-4


def test_cport_bf16_io_matches_f32_io():
    B, S, H, hd = 1, 200, 8, 64
    D = H * hd
    x = R.bf16_round(det_normal((B, S, D), 51)).astype(np.float32)
    bits = (x.view(np.uint32) >> 16).astype(np.uint16)
    c = spectral_coeffs(B, H, 8, hd, 52).astype(np.float32)
    o32, f1 = cref.forward(x, c, lam=f32(R.BASELINE_LAMBDA), nthreads=1)
    o16, f2 = cref.forward(bits, c, lam=f32(R.BASELINE_LAMBDA), x_is_bf16_bits=True, out_bf16=True, nthreads=1)
    assert np.abs(cref.bf16_bits_to_f32(o16) - o32).max() <= 2 ** -8
    assert np.array_equal(f1, f2)
