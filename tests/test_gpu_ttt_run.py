"""The native BASELINE-mode TTT run (``ossm_ttt_wpred_run``: gate, forward,
the tcgen05 W_pred gradient kernel, reverse adjoint and Adam per chunk, in one
call) against the same chunk loop driven from Python with both W_pred
products on cuBLAS in full fp32, and against the float64 oracle.

The tensor-core kernel forms dL/ds = (2/N)(G s - W_pred^T x_{t+1}) with s . G
as a TF32 product and x . W_pred split into two bf16 terms, so a single
chunk's gradient (the Adam first moment after one step from zero) must agree
with the fp32 loop to TF32 accuracy; over several chunks Adam's near-sign
early steps let a few coefficients with a gradient at rounding level move the
other way, which the bar allows for a small fraction."""
import numpy as np
import pytest
import torch

from oracle import cheby_ref as R
from tests.golden.inputs import det_normal, linear_init, spectral_coeffs
from tests.test_oracle_golden import relerr

pytestmark = pytest.mark.gpu


def T(a, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dt)


def _inputs(B, S, H, hd, seed, gated, init):
    D = H * hd
    x = R.bf16_round(det_normal((B, S, D), seed)).astype(np.float32)
    c = spectral_coeffs(B, H, 8, hd, seed + 1).astype(np.float32)
    Wp = det_normal((D, D), seed + 2, 0.02).astype(np.float32)
    W, b = linear_init(H, D, seed + 3)
    ini = det_normal((B, D), seed + 4, 0.1).astype(np.float32) if init else None
    lam = np.asarray(R.BASELINE_LAMBDA[:H] if H <= 8 else [0.9] * H, np.float32)
    return x, c, Wp, W, b, ini, lam


def _run(x, c, Wp, W, b, ini, lam, chunk, gemm, x_dt=torch.bfloat16):
    import orthossm_b200 as O
    z = np.zeros_like(c)
    kw = dict(lambda_per_head=lam.tolist(), chunk=chunk, gemm=gemm)
    if W is not None:
        kw.update(gate_weight=T(W), gate_bias=T(b))
    if ini is not None:
        kw.update(init_state=T(ini))
    r = O.ttt_wpred_adam(T(x, x_dt), T(c), T(z), T(z), 0, T(Wp), **kw)
    torch.cuda.synchronize()
    return {k: (v.cpu().numpy() if torch.is_tensor(v) else v) for k, v in r.items()}


@pytest.mark.parametrize("B,S,H,chunk,gated,init,x_dt", [
    (2, 128, 8, 128, False, False, torch.bfloat16),
    (3, 300, 8, 300, True, True, torch.bfloat16),     # 3 token tiles, the last one ragged
    (1, 257, 4, 257, False, True, torch.float32),     # D = 256, fp32 x (TF32 x-side product)
])
def test_first_chunk_gradient_matches_fp32_loop(B, S, H, chunk, gated, init, x_dt):
    x, c, Wp, W, b, ini, lam = _inputs(B, S, H, 64, 2100 + S, gated, init)
    if not gated:
        W = b = None
    nat = _run(x, c, Wp, W, b, ini, lam, chunk, "tf32", x_dt)
    ref = _run(x, c, Wp, W, b, ini, lam, chunk, "fp32", x_dt)
    assert nat["step"] == ref["step"] == 1
    np.testing.assert_array_equal(nat["out"], ref["out"])  # the same forward kernels
    np.testing.assert_array_equal(nat["final"], ref["final"])
    assert relerr(nat["m"], ref["m"]) < 1e-3  # m = (1 - beta1) g after one step
    assert relerr(nat["v"], ref["v"]) < 2e-3


@pytest.mark.parametrize("gated", [False, True])
def test_multi_chunk_run_matches_oracle(gated):
    B, S, H, hd, chunk = 2, 700, 8, 64, 200  # four chunks, the last one 100 tokens
    x, c, Wp, W, b, ini, lam = _inputs(B, S, H, hd, 2200, gated, True)
    if not gated:
        W = b = None
    nat = _run(x, c, Wp, W, b, ini, lam, chunk, "tf32")
    z = np.zeros_like(c)
    ref = R.ttt_wpred_adam(x.astype(np.float64), c.astype(np.float64), z, z, 0, Wp.astype(np.float64),
                           lam.astype(np.float64), gate=dict(W=W, b=b) if gated else None,
                           init=ini.astype(np.float64), chunk=chunk)
    assert nat["step"] == ref["step"] == 4
    moved = np.abs(nat["coeffs"] - ref["c"]) > 1e-5
    assert moved.mean() < 0.01, moved.mean()
    assert relerr(nat["out"], ref["out"]) < 5e-3
    assert relerr(nat["final"], ref["final"]) < 5e-3
    assert relerr(nat["m"], ref["m"]) < 2e-2
    assert relerr(nat["v"], ref["v"]) < 2e-2


def test_run_single_token_chunks_and_inputs_untouched():
    """chunk = 1 (no loss term: gs is never formed) and a last chunk of one
    token; the caller's tensors are not modified."""
    import orthossm_b200 as O
    B, S, H, hd = 1, 5, 4, 64
    x, c, Wp, W, b, ini, lam = _inputs(B, S, H, hd, 2300, False, False)
    cT, mT, vT = T(c), T(np.zeros_like(c)), T(np.zeros_like(c))
    for chunk in (1, 4):
        r = O.ttt_wpred_adam(T(x, torch.bfloat16), cT, mT, vT, 0, T(Wp), lambda_per_head=lam.tolist(), chunk=chunk)
        f = O.ttt_wpred_adam(T(x, torch.bfloat16), cT, mT, vT, 0, T(Wp), lambda_per_head=lam.tolist(), chunk=chunk,
                             gemm="fp32")
        torch.cuda.synchronize()
        assert r["step"] == f["step"] == -(-S // chunk)
        if chunk == 1:  # no gradient at all: Adam with g = 0 leaves m, v at zero; only the forget gate acts
            np.testing.assert_array_equal(r["out"].cpu().numpy(), f["out"].cpu().numpy())
            np.testing.assert_array_equal(r["coeffs"].cpu().numpy(), f["coeffs"].cpu().numpy())
        else:
            assert relerr(r["out"].cpu().numpy(), f["out"].cpu().numpy()) < 1e-3
    assert np.array_equal(cT.cpu().numpy(), c) and not mT.abs().sum().item()


def test_run_c_abi_rejects_unsupported_shapes_and_small_workspaces():
    """Through the C ABI: H*head_dim not a multiple of 256 is rejected (size
    query 0, OSSM_EINVAL), a workspace one byte short gives OSSM_EWORKSPACE,
    and neither launches anything (the coefficients are unchanged)."""
    from orthossm_b200 import _lib as L
    lib = L.lib()
    st = torch.cuda.current_stream().cuda_stream

    def case(H, hd, seed):
        B, S = 1, 256
        x, c, Wp, _, _, _, lam = _inputs(B, S, H, hd, seed, False, False)
        t = dict(x=T(x, torch.bfloat16), c=T(c), w=T(Wp), lam=T(lam), out=torch.empty(B, S, H * hd, device="cuda"))
        t["m"], t["v"] = torch.zeros_like(t["c"]), torch.zeros_like(t["c"])
        a = L.TttRunArgs(B=B, S=S, H=H, head_dim=hd, degree=8, chunk=128, x=t["x"].data_ptr(), x_dtype=L.OSSM_BF16,
                         x_stride_b=t["x"].stride(0), x_stride_s=t["x"].stride(1), coeffs=t["c"].data_ptr(),
                         m=t["m"].data_ptr(), v=t["v"].data_ptr(), lam_h=t["lam"].data_ptr(), momentum=0.9,
                         w_pred=t["w"].data_ptr(), out=t["out"].data_ptr(), lr=1e-3, beta1=0.9, beta2=0.999,
                         eps=1e-8, spectral_pow=2.0, step0=0, forget=1, flags=0)
        return a, t, c

    a, t, c = case(8, 16, 2400)  # D = 128
    assert lib.ossm_ttt_run_workspace_bytes(L.C.byref(a)) == 0
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    assert lib.ossm_ttt_wpred_run(L.C.byref(a), ws.data_ptr(), ws.numel(), st) == L.OSSM_EINVAL
    a5, t5, c5 = case(8, 64, 2401)  # D = 512: taken, but one byte short of the workspace is refused
    need = lib.ossm_ttt_run_workspace_bytes(L.C.byref(a5))
    assert need > 0
    ws5 = torch.zeros(need, dtype=torch.uint8, device="cuda")
    assert lib.ossm_ttt_wpred_run(L.C.byref(a5), ws5.data_ptr(), need - 1, st) == L.OSSM_EWORKSPACE
    torch.cuda.synchronize()
    assert np.array_equal(t["c"].cpu().numpy(), c) and np.array_equal(t5["c"].cpu().numpy(), c5)


def test_unsupported_width_takes_the_library_gemm_loop():
    """H*head_dim = 128 (not a multiple of 256): ttt_wpred_adam runs the
    chunk loop with the W_pred products on cuBLAS and still matches the oracle."""
    B, S, H, hd, chunk = 2, 256, 8, 16, 128
    x, c, Wp, W, b, ini, lam = _inputs(B, S, H, hd, 2500, False, True)
    nat = _run(x, c, Wp, None, None, ini, lam, chunk, "tf32")
    z = np.zeros_like(c)
    ref = R.ttt_wpred_adam(x.astype(np.float64), c.astype(np.float64), z, z, 0, Wp.astype(np.float64),
                           lam.astype(np.float64), gate=None, init=ini.astype(np.float64), chunk=chunk)
    assert nat["step"] == ref["step"] == 2
    assert relerr(nat["out"], ref["out"]) < 5e-3
    moved = np.abs(nat["coeffs"] - ref["c"]) > 1e-5
    assert moved.mean() < 0.01, moved.mean()
