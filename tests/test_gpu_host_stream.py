"""cheby_ema_forward_host: a pinned host batch streamed through the GPU in
parts with copies overlapped, against the one-call device forward."""
import numpy as np
import pytest
import torch

from oracle import cheby_ref as R
from tests.golden.inputs import det_normal, linear_init, spectral_coeffs

pytestmark = pytest.mark.gpu


def _device_ref(x, c, **kw):
    """The one-call device forward (the three-pass kernels, which the
    host-buffer call runs its parts on)."""
    import orthossm_b200 as O
    return O.cheby_ema_forward(x, c, **kw)


def _inputs(B, S, seed):
    D, H = 512, 8
    x = torch.from_numpy(R.bf16_round(det_normal((B, S, D), seed)).astype(np.float32)).to(torch.bfloat16)
    c = torch.from_numpy(spectral_coeffs(B, H, 8, 64, seed + 1).astype(np.float32))
    W, b = linear_init(H, D, seed + 2)
    init = torch.from_numpy(det_normal((B, D), seed + 3, 0.1).astype(np.float32))
    return x, c, torch.from_numpy(W), torch.from_numpy(b), init


@pytest.mark.parametrize("B,S,pieces", [(8, 3000, 8), (5, 1000, 3), (1, 20000, 6), (1, 777, 4), (4, 3000, 16),
                                         (3, 1001, 8), (8, 2048, 16)])
def test_host_stream_matches_device_call(B, S, pieces):
    import orthossm_b200 as O
    x, c, W, b, init = _inputs(B, S, 3000 + B * S)
    lam = list(R.BASELINE_LAMBDA)
    kw = dict(lambda_per_head=lam, gate_weight=W.cuda(), gate_bias=b.cuda())
    ref, fin = _device_ref(x.cuda(), c.cuda(), init_state=init.cuda(), **kw)
    out_h, fin_h = O.cheby_ema_forward_host(x.pin_memory(), c.cuda(), init_state=init.cuda(), pieces=pieces, **kw)
    torch.cuda.synchronize()
    assert out_h.is_pinned() and out_h.dtype == torch.bfloat16
    _check(out_h, fin_h, ref, fin, whole=B >= pieces)


def _check(out_h, fin_h, ref, fin, whole):
    if whole:  # whole sequences per part: the same kernels on the same rows, bit for bit
        assert torch.equal(out_h, ref.cpu()) and torch.equal(fin_h, fin.cpu())
    else:  # token ranges with the state carried across parts: fp32 rounding of the carries only
        assert (out_h.float() - ref.cpu().float()).abs().max().item() <= 2 ** -7
        assert torch.allclose(fin_h, fin.cpu(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("B,pieces", [(4, 2), (2, 8)])
def test_host_stream_per_token_decay_is_cut_with_the_parts(B, pieces):
    import orthossm_b200 as O
    S = 2500
    x, c, W, b, init = _inputs(B, S, 77 + B)
    g = torch.Generator().manual_seed(5)
    lt = (0.9 + 0.1 * torch.rand(B, S, 8, generator=g)).cuda()
    kw = dict(lambda_per_head=list(R.BASELINE_LAMBDA), lam_tok=lt)
    ref, fin = _device_ref(x.cuda(), c.cuda(), init_state=init.cuda(), **kw)
    out_h, fin_h = O.cheby_ema_forward_host(x.pin_memory(), c.cuda(), init_state=init.cuda(), pieces=pieces, **kw)
    torch.cuda.synchronize()
    _check(out_h, fin_h, ref, fin, whole=B >= pieces)


def test_c_abi_host_call_with_pageable_buffers():
    """ossm_cheby_ema_fwd_host called directly, as a foreign-function caller
    would, on plain (pageable) host buffers: the copies serialise, the result
    is bitwise the device forward's (three parts of one sequence each)."""
    import ctypes as C
    import orthossm_b200 as O
    from orthossm_b200 import _lib as L
    from orthossm_b200.sdpc_kernel import _fwd_args
    B, S = 3, 1500
    x, c, W, b, init = _inputs(B, S, 11)
    kw = dict(lambda_per_head=list(R.BASELINE_LAMBDA), gate_weight=W.cuda(), gate_bias=b.cuda())
    ref, fin = _device_ref(x.cuda(), c.cuda(), init_state=init.cuda(), **kw)
    out_h, fin_h = torch.empty_like(x), torch.empty(B, 512)
    a, keep, _, _ = _fwd_args(x.contiguous(), c.cuda(), init_state=init.contiguous(), out=out_h, final_state=fin_h,
                              host=True, device="cuda", **kw)
    lib = L.lib()
    nb = lib.ossm_fwd_host_workspace_bytes(C.byref(a), 3)
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    assert lib.ossm_cheby_ema_fwd_host(C.byref(a), 3, ws.data_ptr(), nb, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(out_h, ref.cpu()) and torch.equal(fin_h, fin.cpu())


def test_device_forward_after_host_call_on_the_same_stream():
    """The host call's staging buffers live in a workspace of their own: a
    generic-kernel forward (fp32 x) on the same stream afterwards still
    finds its launch counters intact."""
    import orthossm_b200 as O
    x, c, W, b, init = _inputs(4, 1024, 21)
    O.cheby_ema_forward_host(x.pin_memory(), c.cuda(), init_state=init, pieces=8,
                             lambda_per_head=list(R.BASELINE_LAMBDA))
    x32 = x.float()
    out, fin = O.cheby_ema_forward(x32.cuda(), c.cuda(), lambda_per_head=list(R.BASELINE_LAMBDA),
                                   init_state=init.cuda(), out_dtype=torch.float32)
    ref = R.cheby_ema_forward(x32.numpy(), c.numpy(), lam=np.asarray(R.BASELINE_LAMBDA, np.float32),
                              init=init.numpy())
    torch.cuda.synchronize()
    assert np.abs(out.cpu().numpy() - ref["out"]).max() < 1e-4
    assert O.workspace_status() == 0


def test_host_stream_rejects_device_input():
    import orthossm_b200 as O
    x, c, W, b, init = _inputs(2, 64, 1)
    with pytest.raises(ValueError):
        O.cheby_ema_forward_host(x.cuda(), c.cuda())
