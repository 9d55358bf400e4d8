"""GPU parity of the single-evaluation grouped forward (ossm_forward_grp.cu,
OSSM_F_SINGLE_EVAL: one CTA per SM, each sequence owned by a group of CTAs
exchanging tile aggregates through the workspace; bf16 x and output with 8 or
more sequences) against the float64 oracle and the default three-pass
kernels.

Tolerances: bf16 I/O with fp32 state 2e-2
relative.  Against the three-pass kernels (the default), which compute
the same function with the carries composed in another order: one bf16 step
per output and fp32 rounding (1e-5) on the final state."""
import numpy as np
import pytest
import torch

from oracle import cheby_ref as R
from tests.golden.inputs import det_normal, linear_init, spectral_coeffs
from tests.test_oracle_golden import relerr

pytestmark = pytest.mark.gpu
dev = "cuda"
BF16_TOL = 2e-2


def T(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)


def N(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def _problem(B, S, seed, K=8):
    D, H = 512, 8
    x = R.bf16_round(det_normal((B, S, D), seed)).astype(np.float32)
    c = spectral_coeffs(B, H, K, 64, seed + 1)
    W, b = linear_init(H, D, seed + 2)
    init = det_normal((B, D), seed + 3, 0.1)
    lam = np.asarray(R.BASELINE_LAMBDA, np.float32).astype(np.float64)
    return x, c, W, b, init, lam


def _fwd(x, c, three_pass=False, **kw):
    from orthossm_b200 import _lib as L
    from orthossm_b200.sdpc_kernel import _cheby_ema_forward
    return _cheby_ema_forward(x, c, extra_flags=0 if three_pass else L.OSSM_F_SINGLE_EVAL, **kw)


def _kw(mode, W, b, lam, B, S):
    kw = dict(lambda_per_head=lam.tolist())
    lt = None
    if mode == "gate":
        kw.update(gate_weight=T(W), gate_bias=T(b))
    elif mode == "lamtok":
        lt = 0.95 + 0.0499 * torch.rand(B, S, 8, generator=torch.Generator().manual_seed(S))
        kw.update(lam_tok=lt.to(dev))
    return kw, lt


# (B, S): one tile (one member busy); a ragged tile; several rounds with a
# partial last round; groups of 10 and 7 members; the config-2 batch at a
# shorter length
@pytest.mark.parametrize("B,S,mode,init", [
    (8, 31, "gate", True), (8, 1000, "gate", True), (9, 17 * 32 * 3 + 5, "const", False),
    (12, 512, "gate", False), (8, 3000, "gate", True), (10, 4097, "lamtok", True), (20, 2500, "const", True)])
def test_grouped_vs_oracle(B, S, mode, init):
    import orthossm_b200 as O
    x, c, W, b, ini, lam = _problem(B, S, 500 + S + B)
    kw, lt = _kw(mode, W, b, lam, B, S)
    from orthossm_b200 import _lib as L
    assert O.forward_path(T(x, torch.bfloat16), T(c), extra_flags=L.OSSM_F_SINGLE_EVAL, **kw) == "grouped"
    assert O.forward_path(T(x, torch.bfloat16), T(c), **kw) == "parked"
    out, fin = _fwd(T(x, torch.bfloat16), T(c), init_state=T(ini) if init else None, **kw)
    torch.cuda.synchronize()
    assert O.workspace_status() == 0
    gate = dict(W=W, b=b) if mode == "gate" else None
    # the per-token decays as the kernel receives them (fp32)
    lam_ref = lam if lt is None else lt.numpy().astype(np.float64)
    ref = R.cheby_ema_forward(x, c, lam=lam_ref, gate=gate, init=ini if init else None)
    assert relerr(N(out), ref["out"]) < BF16_TOL
    assert relerr(N(fin), ref["final"]) < 1e-3


@pytest.mark.parametrize("B,S,mode", [(8, 8192, "gate"), (12, 5000, "const"), (8, 3333, "lamtok")])
def test_grouped_vs_three_pass(B, S, mode):
    x, c, W, b, ini, lam = _problem(B, S, 700 + S)
    kw, _ = _kw(mode, W, b, lam, B, S)
    xb, cb, ib = T(x, torch.bfloat16), T(c), T(ini)
    o1, f1 = _fwd(xb, cb, init_state=ib, **kw)
    o3, f3 = _fwd(xb, cb, init_state=ib, three_pass=True, **kw)
    assert (o1.float() - o3.float()).abs().max().item() <= 2 ** -7
    assert relerr(N(f1), N(f3)) < 1e-5


def test_grouped_rows_are_independent_and_reproducible():
    """Each sequence is one group's work, folded in a fixed order: repeat
    calls agree bit for bit, and with groups of equal size (37 sequences: 4
    members each on 148 SMs) a row's output does not depend on the other rows
    or on its place in the batch."""
    import orthossm_b200 as O
    B, S = 37, 700
    x, c, W, b, ini, lam = _problem(B, S, 910)
    kw = dict(lambda_per_head=lam.tolist(), gate_weight=T(W), gate_bias=T(b))
    xb, cb, ib = T(x, torch.bfloat16), T(c), T(ini)
    o, f = _fwd(xb, cb, init_state=ib, **kw)
    o2, f2 = _fwd(xb, cb, init_state=ib, **kw)
    assert torch.equal(o, o2) and torch.equal(f, f2)
    if torch.cuda.get_device_properties(0).multi_processor_count % B:
        pytest.skip("groups of unequal size on this GPU")
    perm = torch.randperm(B, generator=torch.Generator().manual_seed(1)).tolist()
    op, fp = _fwd(xb[perm].contiguous(), cb[perm].contiguous(), init_state=ib[perm].contiguous(), **kw)
    for i, r in enumerate(perm):
        assert torch.equal(op[i], o[r]) and torch.equal(fp[i], f[r]), r
    assert O.workspace_status() == 0


def test_grouped_nan_inf_and_huge_inputs():
    """The reference's fused semantics (sdpc_kernel.py:1078-1085, :1160-1164)
    at non-finite and huge inputs, on the grouped kernel: NaN x contributes
    u = 0, +-inf and near-maximum inputs give xn = +-1."""
    B, S, D = 8, 700, 512
    x = R.bf16_round(det_normal((B, S, D), 931)).astype(np.float32)
    x[0, 5, 3] = np.nan
    x[1, 17, 100] = np.inf
    x[2, 650, 511] = -np.inf
    x[3, 0, :7] = np.nan
    x[3, 699, 64] = 3.0e38
    x[2, 0, 8] = -np.inf
    c = spectral_coeffs(B, 8, 8, 64, 932)
    init = det_normal((B, D), 933, 0.1)
    lam = np.asarray(R.BASELINE_LAMBDA, np.float32).astype(np.float64)
    out, fin = _fwd(T(x, torch.bfloat16), T(c), lambda_per_head=lam.tolist(), init_state=T(init))
    ref = R.cheby_ema_forward(x, c, lam=lam, init=init)
    o = N(out)
    assert np.isfinite(o).all() and np.isfinite(N(fin)).all()
    assert relerr(o, ref["out"]) < BF16_TOL
    assert relerr(N(fin), ref["final"]) < BF16_TOL


@pytest.mark.parametrize("three_pass", [False, True])
def test_strided_batch_and_deg4_mode(three_pass):
    """Strided rows (a view of a wider batch) and the degree-4 truncation
    mode (degree-8 coefficients of which c_0..c_3 are used) on both bf16
    paths."""
    B, S = 8, 1500
    x, c, W, b, ini, lam = _problem(B, S, 950)
    big = torch.zeros(B, S + 40, 512, dtype=torch.bfloat16, device=dev)
    big[:, :S] = T(x, torch.bfloat16)
    xv = big[:, :S]  # batch stride (S + 40) * 512
    out, fin = _fwd(xv, T(c), three_pass=three_pass, lambda_per_head=lam.tolist(), init_state=T(ini),
                    eval_mode="clenshaw_deg4")
    ref = R.cheby_ema_forward(x, c, lam=lam, init=ini, eval_mode="clenshaw_deg4")
    assert relerr(N(out), ref["out"]) < BF16_TOL
    assert relerr(N(fin), ref["final"]) < 1e-3
