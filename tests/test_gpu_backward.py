"""Backward of the forward (``ossm_cheby_ema_bwd`` through ``cheby_ema_forward``'s
autograd node) against torch autograd of a float64 restatement of the same
forward on CPU: gradients for x, the coefficients and the carried-in state,
with the decays held constant (as the reference's backward does,
FusedChebyRKVv10.backward, sdpc_kernel.py:2435-2515)."""
import numpy as np
import pytest
import torch

from oracle import cheby_ref as R
from tests.golden.inputs import det_normal, linear_init, spectral_coeffs
from tests.test_oracle_golden import relerr

pytestmark = pytest.mark.gpu


def torch_forward(x, c, a, init):
    """float64 forward: x [B,S,D], c [B,H,K,hd], a [B,S,D] decays, init [B,D] or None."""
    B, S, D = x.shape
    H, K, hd = c.shape[1], c.shape[2], c.shape[3]
    m = x.abs().clamp(min=1e-7)
    sgn = torch.where(x >= 0, torch.ones_like(x), -torch.ones_like(x))
    xn = sgn * (1.0 - 1.0 / (1.0 + m))
    T = [torch.ones_like(xn), xn]
    for _ in range(2, K):
        T.append(2.0 * xn * T[-1] - T[-2])
    cc = c.permute(0, 2, 1, 3).reshape(B, K, D)
    y = sum(cc[:, k][:, None, :] * T[k] for k in range(K))
    gam = torch.tensor(np.repeat(R.gamma_h(H), hd), dtype=torch.float64)
    u = torch.tanh(torch.clamp(gam * y, -4.0, 4.0))
    s = torch.zeros(B, D, dtype=torch.float64) if init is None else init
    outs = []
    for t in range(S):
        s = torch.clamp(a[:, t] * s + (1.0 - a[:, t]) * u[:, t], -1.0, 1.0)
        outs.append(s)
    return torch.stack(outs, 1), s


@pytest.mark.parametrize("x_bf16,gate,init", [(False, False, True), (True, True, True), (False, True, False)])
def test_backward_matches_float64_autograd(x_bf16, gate, init):
    import orthossm_b200 as O
    B, S, H, hd = 2, 200, 8, 64
    D = H * hd
    x = R.bf16_round(det_normal((B, S, D), 1500)).astype(np.float32)
    c = spectral_coeffs(B, H, 8, hd, 1501).astype(np.float32)
    W, b = linear_init(H, D, 1502)
    ini = det_normal((B, D), 1503, 0.3).astype(np.float32)
    lam = np.asarray(R.BASELINE_LAMBDA, np.float32)
    w_out = det_normal((B, S, D), 1504).astype(np.float32)
    w_fin = det_normal((B, D), 1505).astype(np.float32)

    dev = "cuda"
    xg = torch.tensor(x, device=dev, dtype=torch.bfloat16 if x_bf16 else torch.float32, requires_grad=True)
    cg = torch.tensor(c, device=dev, requires_grad=True)
    ig = torch.tensor(ini, device=dev, requires_grad=True) if init else None
    kw = dict(lambda_per_head=lam.tolist(), out_dtype=torch.float32)
    if gate:
        kw.update(gate_weight=torch.tensor(W, device=dev), gate_bias=torch.tensor(b, device=dev))
    out, fin = O.cheby_ema_forward(xg, cg, init_state=ig, **kw)
    loss = (out * torch.tensor(w_out, device=dev)).sum() + (fin * torch.tensor(w_fin, device=dev)).sum()
    loss.backward()

    # the same decays, as constants
    if gate:
        lt = O.gate_decay(xg.detach(), kw["gate_weight"], kw["gate_bias"], lam.tolist()).cpu().double()
        a = lt.repeat_interleave(hd, dim=2)
    else:
        a = torch.tensor(np.repeat(lam.astype(np.float64), hd))[None, None, :].expand(B, S, D)
    xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    ct = torch.tensor(c, dtype=torch.float64, requires_grad=True)
    it = torch.tensor(ini, dtype=torch.float64, requires_grad=True) if init else None
    o_t, f_t = torch_forward(xt, ct, a, it)
    (o_t * torch.tensor(w_out, dtype=torch.float64)).sum().add((f_t * torch.tensor(w_fin, dtype=torch.float64)).sum()).backward()

    assert relerr(out.detach().cpu().numpy(), o_t.detach().numpy()) < 1e-4
    assert relerr(cg.grad.cpu().numpy(), ct.grad.numpy()) < 1e-4
    gx = xg.grad.float().cpu().numpy()
    tol = 1e-2 if x_bf16 else 1e-4  # a bf16 x gets a bf16 gradient
    assert relerr(gx, xt.grad.numpy()) < tol
    if init:
        assert relerr(ig.grad.cpu().numpy(), it.grad.numpy()) < 1e-4


def test_backward_clamped_carried_state():
    """A carried-in state outside [-1, 1]: the token-0 clamp passes no gradient
    there (to the state or to u_0), elsewhere it does."""
    import orthossm_b200 as O
    B, S, H, hd = 1, 64, 8, 64
    D = H * hd
    x = R.bf16_round(det_normal((B, S, D), 1600)).astype(np.float32)
    c = spectral_coeffs(B, H, 8, hd, 1601).astype(np.float32)
    ini = (det_normal((B, D), 1602, 1.0) * 3).astype(np.float32)  # many |init| > 1
    lam = np.asarray(R.BASELINE_LAMBDA, np.float32)
    xg = torch.tensor(x, device="cuda", requires_grad=True)
    cg = torch.tensor(c, device="cuda", requires_grad=True)
    ig = torch.tensor(ini, device="cuda", requires_grad=True)
    out, fin = O.cheby_ema_forward(xg, cg, init_state=ig, lambda_per_head=lam.tolist())
    out.sum().backward()
    a = torch.tensor(np.repeat(lam.astype(np.float64), hd))[None, None, :].expand(B, S, D)
    xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    ct = torch.tensor(c, dtype=torch.float64, requires_grad=True)
    it = torch.tensor(ini, dtype=torch.float64, requires_grad=True)
    o_t, _ = torch_forward(xt, ct, a, it)
    o_t.sum().backward()
    assert relerr(ig.grad.cpu().numpy(), it.grad.numpy()) < 1e-4
    assert relerr(xg.grad.cpu().numpy(), xt.grad.numpy()) < 1e-4
    assert (ig.grad.cpu().numpy()[np.abs(ini) > 1.5] == 0).all()


def torch_rkv_chunks(x, trace, mu, n_heads, chunk, fast=False):
    """float64 forward of the reference's chunk loop with each chunk's own
    coefficients (EMA from zero per chunk); fast: the fast path (x.sign(),
    unclamped tanh)."""
    B, S, D = x.shape
    hd = D // n_heads
    outs = []
    for ci, t0 in enumerate(range(0, S, chunk)):
        xc = x[:, t0:t0 + chunk]
        c = trace[ci]
        K = c.shape[2]
        m = xc.abs().clamp(min=1e-7)
        sgn = torch.sign(xc) if fast else torch.where(xc >= 0, torch.ones_like(xc), -torch.ones_like(xc))
        xn = sgn * (1.0 - 1.0 / (1.0 + m))
        T = [torch.ones_like(xn), xn]
        for _ in range(2, K):
            T.append(2.0 * xn * T[-1] - T[-2])
        cc = c.permute(0, 2, 1, 3).reshape(B, K, D)
        y = sum(cc[:, k][:, None, :] * T[k] for k in range(K))
        gam = torch.tensor(np.repeat(R.gamma_h(n_heads), hd), dtype=torch.float64)
        z = gam * y
        u = torch.tanh(z) if fast else torch.tanh(torch.clamp(z, -4.0, 4.0))
        s = torch.zeros(B, D, dtype=torch.float64)
        for t in range(xc.shape[1]):
            s = mu * s + (1.0 - mu) * u[:, t]
            outs.append(s)
    return torch.stack(outs, 1)


@pytest.mark.parametrize("S,chunk,n_heads", [(600, 256, 4), (200, 256, 8)])
def test_apply_cheby_rkv_v10_backward_matches_reference_semantics(S, chunk, n_heads):
    """The full (Lion TTT) path: x always gets a gradient; coeffs only when the
    sequence is one chunk (the reference detaches them between chunks)."""
    import orthossm_b200 as O
    from orthossm_b200.sdpc_kernel import _lion_full_path
    B, D = 2, 512
    hd = D // n_heads
    x = det_normal((B, S, D), 1700).astype(np.float32)
    c = spectral_coeffs(B, n_heads, 8, hd, 1701).astype(np.float32)
    w = det_normal((B, S, D), 1702).astype(np.float32)
    xg = torch.tensor(x, device="cuda", requires_grad=True)
    cg = torch.tensor(c, device="cuda", requires_grad=True)
    mom = torch.zeros_like(cg)
    out, c_new, m_new = O.apply_cheby_rkv_v10(xg, cg, mom, n_heads=n_heads, chunk_size=chunk, seq_threshold=128)
    (out * torch.tensor(w, device="cuda")).sum().backward()
    n_chunks = (S + chunk - 1) // chunk
    trace = torch.empty((n_chunks, B, n_heads, 8, hd), device="cuda")
    with torch.no_grad():
        _lion_full_path(torch.tensor(x, device="cuda"), torch.tensor(c, device="cuda"), torch.zeros_like(cg),
                        n_heads, 0.005, 0.9, 0.9, 0.99, 0.01, min(chunk, S), None, None, True, trace=trace)
    xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    tr = trace.cpu().double()
    if n_chunks == 1:
        tr = tr.clone().requires_grad_(True)
    o = torch_rkv_chunks(xt, tr, 0.9, n_heads, min(chunk, S))
    (o * torch.tensor(w, dtype=torch.float64)).sum().backward()
    assert relerr(xg.grad.cpu().numpy(), xt.grad.numpy()) < 1e-4
    if n_chunks == 1:
        assert relerr(cg.grad.cpu().numpy(), tr.grad[0].numpy()) < 1e-4
    else:
        assert cg.grad is None


def test_fast_path_backward():
    """Below seq_threshold: the fast path (x.sign(), unclamped tanh); x and
    coeffs get gradients."""
    import orthossm_b200 as O
    B, S, D, n_heads = 2, 100, 512, 8
    hd = D // n_heads
    x = det_normal((B, S, D), 1800).astype(np.float32)
    x[0, 3, :5] = 0.0
    c = spectral_coeffs(B, n_heads, 8, hd, 1801).astype(np.float32)
    w = det_normal((B, S, D), 1802).astype(np.float32)
    xg = torch.tensor(x, device="cuda", requires_grad=True)
    cg = torch.tensor(c, device="cuda", requires_grad=True)
    out, _, _ = O.apply_cheby_rkv_v10(xg, cg, torch.zeros_like(cg), n_heads=n_heads)
    (out * torch.tensor(w, device="cuda")).sum().backward()
    xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    ct = torch.tensor(c, dtype=torch.float64, requires_grad=True)
    o = torch_rkv_chunks(xt, ct[None], 0.9, n_heads, S, fast=True)
    (o * torch.tensor(w, dtype=torch.float64)).sum().backward()
    assert relerr(out.detach().cpu().numpy(), o.detach().numpy()) < 1e-4
    assert relerr(xg.grad.cpu().numpy(), xt.grad.numpy()) < 1e-4
    assert relerr(cg.grad.cpu().numpy(), ct.grad.numpy()) < 1e-4
