"""cheby_ema_forward_host: a pinned host batch streamed through the GPU in
parts with copies overlapped, against the one-call device forward."""
import numpy as np
import pytest
import torch

from oracle import cheby_ref as R
from tests.golden.inputs import det_normal, linear_init, spectral_coeffs

pytestmark = pytest.mark.gpu


def _inputs(B, S, seed):
    D, H = 512, 8
    x = torch.from_numpy(R.bf16_round(det_normal((B, S, D), seed)).astype(np.float32)).to(torch.bfloat16)
    c = torch.from_numpy(spectral_coeffs(B, H, 8, 64, seed + 1).astype(np.float32))
    W, b = linear_init(H, D, seed + 2)
    init = torch.from_numpy(det_normal((B, D), seed + 3, 0.1).astype(np.float32))
    return x, c, torch.from_numpy(W), torch.from_numpy(b), init


@pytest.mark.parametrize("B,S,pieces", [(8, 3000, 8), (5, 1000, 3), (1, 20000, 6), (1, 777, 4)])
def test_host_stream_matches_device_call(B, S, pieces):
    import orthossm_b200 as O
    x, c, W, b, init = _inputs(B, S, 3000 + B * S)
    lam = list(R.BASELINE_LAMBDA)
    kw = dict(lambda_per_head=lam, gate_weight=W.cuda(), gate_bias=b.cuda())
    ref, fin = O.cheby_ema_forward(x.cuda(), c.cuda(), init_state=init.cuda(), **kw)
    out_h, fin_h = O.cheby_ema_forward_host(x.pin_memory(), c.cuda(), init_state=init.cuda(), pieces=pieces, **kw)
    torch.cuda.synchronize()
    assert out_h.is_pinned() and out_h.dtype == torch.bfloat16
    if B >= 2:  # whole sequences per part: the same kernels on the same rows, bit for bit
        assert torch.equal(out_h, ref.cpu()) and torch.equal(fin_h, fin.cpu())
    else:  # token ranges with the state carried across parts: fp32 rounding of the carries only
        assert (out_h.float() - ref.cpu().float()).abs().max().item() <= 2 ** -7
        assert torch.allclose(fin_h, fin.cpu(), rtol=1e-5, atol=1e-6)


def test_host_stream_rejects_device_input():
    import orthossm_b200 as O
    x, c, W, b, init = _inputs(2, 64, 1)
    with pytest.raises(ValueError):
        O.cheby_ema_forward_host(x.cuda(), c.cuda())
