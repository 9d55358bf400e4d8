"""Generate golden fixtures by running the reference's own kernels on CPU.

Runs Eddym06/OrthoSSM ``sdpc_kernel.py`` (Triton) under ``TRITON_INTERPRET=1``
on deterministic inputs (``inputs.py``) and stores the reference's outputs in
``tests/golden/*.npz``.  Needs the reference checkout (``--ref``, default the
``OSSM_REFERENCE`` environment variable); it is run once, offline, and its
outputs are committed.  Tests never import the reference.

    python tests/golden/make_golden.py --ref <path-to-OrthoSSM> [--only NAME]
"""
from __future__ import annotations

import argparse
import multiprocessing as mp
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from inputs import det_normal, det_uniform, spectral_coeffs  # noqa: E402

CFG1_LAMBDA = (0.9995, 0.9995, 0.997, 0.997, 0.995, 0.995, 0.95, 0.95)


def _import_ref(ref):
    os.environ["TRITON_INTERPRET"] = "1"
    if ref not in sys.path:
        sys.path.insert(0, ref)
    import torch  # noqa: F401
    import sdpc_kernel as K
    return K


def run_fused(ref, x, c, momentum, use_lut, init=None):
    """One ``_fused_clenshaw_ema_kernel`` launch, call pattern of
    precision_tests.py:48-73."""
    K = _import_ref(ref)
    import torch
    import triton
    x = torch.from_numpy(np.ascontiguousarray(x))
    c = torch.from_numpy(np.ascontiguousarray(c))
    B, S, D = x.shape
    nH, deg, hd = c.shape[1], c.shape[2], c.shape[3]
    lut = K.get_chebyshev_lut(x.device).contiguous()
    xn = torch.empty(B, S, D)
    ty = torch.empty(B, S, D)
    out = torch.empty(B, S, D)
    ei = torch.zeros(B, D) if init is None else torch.from_numpy(np.ascontiguousarray(init))
    ef = torch.empty(B, D)
    BLOCK_HD = min(32, triton.next_power_of_2(hd))
    grid = (B * nH * triton.cdiv(hd, BLOCK_HD),)
    K._fused_clenshaw_ema_kernel[grid](
        x, c, lut, xn, ty, out, ei, ef,
        S, D, hd, nH, deg, K.LUT_TABLE_SIZE, momentum,
        x.stride(0), x.stride(1), x.stride(2),
        c.stride(0), c.stride(1), c.stride(2), c.stride(3),
        lut.stride(0), lut.stride(1),
        xn.stride(0), xn.stride(1), xn.stride(2),
        ty.stride(0), ty.stride(1), ty.stride(2),
        out.stride(0), out.stride(1), out.stride(2),
        ei.stride(0), ei.stride(1),
        BLOCK_HD=BLOCK_HD, BLOCK_S=128, USE_LUT=use_lut)
    return dict(xnorm=xn.numpy(), tanh=ty.numpy(), out=out.numpy(), final=ef.numpy())


def run_parallel_ema(ref, y, momentum, init=None):
    """``_parallel_ema_forward_kernel`` (sdpc_kernel.py:440) as launched by
    ``_EMAFastPathFn.forward`` (:1651)."""
    K = _import_ref(ref)
    import torch
    import triton
    y = torch.from_numpy(np.ascontiguousarray(y))
    B, S, D = y.shape
    out = torch.empty(B, S, D)
    ei = torch.zeros(B, D) if init is None else torch.from_numpy(np.ascontiguousarray(init))
    ef = torch.empty(B, D)
    BLOCK_HD = min(32, triton.next_power_of_2(D))
    grid = (B * triton.cdiv(D, BLOCK_HD),)
    K._parallel_ema_forward_kernel[grid](
        y, out, ei, ef, S, D, momentum,
        y.stride(0), y.stride(1), y.stride(2),
        out.stride(0), out.stride(1), out.stride(2),
        ei.stride(0), ei.stride(1), BLOCK_HD=BLOCK_HD, BLOCK_S=128)
    return dict(out=out.numpy(), final=ef.numpy())


def run_apply(ref, x, c, m, **kw):
    """Public op ``apply_cheby_rkv_v10`` (sdpc_kernel.py:2522)."""
    K = _import_ref(ref)
    import torch
    args = {}
    for k, v in kw.items():
        args[k] = torch.from_numpy(np.ascontiguousarray(v)) if isinstance(v, np.ndarray) else v
    out, cn, mn = K.apply_cheby_rkv_v10(torch.from_numpy(x), torch.from_numpy(c),
                                       torch.from_numpy(m), **args)
    return dict(out=out.float().numpy(), c_new=cn.float().numpy(), m_new=mn.float().numpy())


# ----------------------------------------------------------------------------

def case_fused_f32_deg8(ref):
    x = det_normal((2, 300, 64), 101)
    c = spectral_coeffs(2, 8, 8, 8, 102, scale=1.0)
    r = run_fused(ref, x, c, 0.9, use_lut=False)
    return dict(seed_x=101, seed_c=102, shape=(2, 300, 64), H=8, K=8, momentum=0.9, **r)


def case_fused_f32_deg4_init(ref):
    x = det_normal((2, 257, 128), 111)
    c = spectral_coeffs(2, 8, 4, 16, 112, scale=1.5)
    init = np.clip(det_normal((2, 128), 113, 0.3), -0.95, 0.95)
    r = run_fused(ref, x, c, 0.95, use_lut=False, init=init)
    return dict(seed_x=111, seed_c=112, seed_init=113, shape=(2, 257, 128), H=8, K=4,
                momentum=0.95, init=init, **r)


def case_fused_lut_deg8(ref):
    x = det_normal((1, 200, 64), 121)
    c = spectral_coeffs(1, 4, 8, 16, 122, scale=1.0)
    r = run_fused(ref, x, c, 0.9, use_lut=True)
    return dict(seed_x=121, seed_c=122, shape=(1, 200, 64), H=4, K=8, momentum=0.9, **r)


def case_fused_nan(ref):
    x = det_normal((1, 130, 64), 131)
    x[0, 3, 5] = np.nan
    x[0, 40, 0:8] = np.nan
    x[0, 7, :] = 0.0
    x[0, 8, 9] = -0.0
    x[0, 9, 10] = 1e-9
    c = spectral_coeffs(1, 8, 8, 8, 132, scale=2.0)
    r = run_fused(ref, x, c, 0.9, use_lut=False)
    return dict(x=x, c=c, H=8, K=8, momentum=0.9, **r)


def _cfg1_head(args):
    ref, h = args
    x = det_normal((1, 2048, 512), 1)
    c = spectral_coeffs(1, 8, 8, 64, 2, scale=1.0)
    r = run_fused(ref, x, c, CFG1_LAMBDA[h], use_lut=False)
    sl = slice(h * 64, (h + 1) * 64)
    return h, r["out"][:, :, sl], r["final"][:, sl], r["tanh"][:, :, sl]


CFG1_ROWS = np.unique(np.concatenate([np.arange(16), np.arange(0, 2048, 64),
                                      np.arange(2032, 2048)]))


def case_cfg1(ref):
    """fp32, B=1, S=2048, D=512, deg 8, per-head lambda,
    zero init.  The reference kernel takes one scalar decay, so it is run once
    per head with that head's lambda and the head's channels are kept."""
    ctx = mp.get_context("spawn")
    with ctx.Pool(8) as pool:
        res = pool.map(_cfg1_head, [(ref, h) for h in range(8)])
    out = np.zeros((1, 2048, 512), np.float32)
    fin = np.zeros((1, 512), np.float32)
    tanh = np.zeros((1, 2048, 512), np.float32)
    for h, o, f, t in res:
        out[:, :, h * 64:(h + 1) * 64] = o
        fin[:, h * 64:(h + 1) * 64] = f
        tanh[:, :, h * 64:(h + 1) * 64] = t
    return dict(seed_x=1, seed_c=2, shape=(1, 2048, 512), H=8, K=8, lam=np.array(CFG1_LAMBDA),
                rows=CFG1_ROWS, out_rows=out[:, CFG1_ROWS], tanh_rows=tanh[:, CFG1_ROWS],
                final=fin, out_sum=np.float64(out.astype(np.float64).sum()),
                out_sumsq=np.float64((out.astype(np.float64) ** 2).sum()),
                out_abssum=np.float64(np.abs(out.astype(np.float64)).sum()))


def case_ema_per_head(ref):
    """Per-head-lambda EMA (chimera_v2_ssm.py:75-98 semantics, with the
    reference's clamp) pinned through ``_parallel_ema_forward_kernel`` run
    once per head."""
    B, S, H, hd = 2, 300, 8, 8
    y = (det_uniform(B * S * H * hd, 141).reshape(B, S, H * hd) * 2 - 1).astype(np.float32)
    init = np.clip(det_normal((B, H * hd), 142, 0.4), -0.99, 0.99)
    out = np.zeros_like(y)
    fin = np.zeros((B, H * hd), np.float32)
    for h in range(H):
        sl = slice(h * hd, (h + 1) * hd)
        r = run_parallel_ema(ref, np.ascontiguousarray(y[:, :, sl]), CFG1_LAMBDA[h],
                             np.ascontiguousarray(init[:, sl]))
        out[:, :, sl] = r["out"]
        fin[:, sl] = r["final"]
    return dict(y=y, init=init, lam=np.array(CFG1_LAMBDA), out=out, final=fin)


def case_mega_lut_deg8_gates(ref):
    x = det_normal((2, 600, 64), 151)
    c = spectral_coeffs(2, 8, 8, 8, 152, scale=0.5)
    m = det_normal((2, 8, 8, 8), 153, 0.01)
    gate = np.array([[0.7], [0.3]], np.float32)
    dyn = np.array([[0.9], [0.2]], np.float32)
    r = run_apply(ref, x, c, m, n_heads=8, seq_threshold=0, chunk_size=256, use_lut=True,
                  gate_global=gate, dynamic_lambda=dyn)
    return dict(seed_x=151, seed_c=152, seed_m=153, shape=(2, 600, 64), H=8, K=8,
                gate_global=gate, dynamic_lambda=dyn, chunk_size=256, **r)


def case_mega_clenshaw_deg8(ref):
    x = det_normal((2, 256, 64), 161)
    c = spectral_coeffs(2, 8, 8, 8, 162, scale=0.5)
    m = np.zeros((2, 8, 8, 8), np.float32)
    r = run_apply(ref, x, c, m, n_heads=8, seq_threshold=0, chunk_size=256, use_lut=False)
    return dict(seed_x=161, seed_c=162, shape=(2, 256, 64), H=8, K=8, chunk_size=256, **r)


def case_mega_deg4_chunks(ref):
    x = det_normal((1, 512, 128), 171)
    c = spectral_coeffs(1, 8, 4, 16, 172, scale=0.5)
    m = np.zeros((1, 8, 4, 16), np.float32)
    r = run_apply(ref, x, c, m, n_heads=8, seq_threshold=0, chunk_size=128, use_lut=True,
                  ema_momentum=0.85, base_lr=0.01)
    return dict(seed_x=171, seed_c=172, shape=(1, 512, 128), H=8, K=4, chunk_size=128,
                ema_momentum=0.85, base_lr=0.01, **r)


def case_fast_path(ref):
    x = det_normal((2, 100, 64), 181)
    c = spectral_coeffs(2, 8, 4, 8, 182, scale=1.0)
    m = np.zeros((2, 8, 4, 8), np.float32)
    r = run_apply(ref, x, c, m, n_heads=8, ema_momentum=0.9)
    return dict(seed_x=181, seed_c=182, shape=(2, 100, 64), H=8, K=4, **r)


CASES = {
    "fused_f32_deg8": case_fused_f32_deg8,
    "fused_f32_deg4_init": case_fused_f32_deg4_init,
    "fused_lut_deg8": case_fused_lut_deg8,
    "fused_nan": case_fused_nan,
    "ema_per_head": case_ema_per_head,
    "mega_lut_deg8_gates": case_mega_lut_deg8_gates,
    "mega_clenshaw_deg8": case_mega_clenshaw_deg8,
    "mega_deg4_chunks": case_mega_deg4_chunks,
    "fast_path": case_fast_path,
    "cfg1": case_cfg1,
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("OSSM_REFERENCE", ""))
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    if not a.ref or not os.path.isdir(a.ref):
        sys.exit("reference checkout not found: pass --ref")
    names = [n for n in CASES if not a.only or n in a.only.split(",")]
    for n in names:
        t = time.time()
        d = CASES[n](a.ref)
        d["generator"] = "tests/golden/make_golden.py (TRITON_INTERPRET=1)"
        np.savez_compressed(os.path.join(HERE, f"{n}.npz"), **d)
        print(f"{n}: {time.time() - t:.1f}s", flush=True)


if __name__ == "__main__":
    main()
