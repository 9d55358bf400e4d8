"""ossm_cheby_ema_fwd_noalloc, the forward for callers that cannot allocate
device memory (hosts whose allocator owns all of it, plugins that are only
handed their input and output buffers).  It takes its scratch from a fixed
array inside the library instead of a caller workspace, so it must give the
same outputs as ossm_cheby_ema_fwd with a workspace, call after call.

The tests pass whether they run alone in a fresh process (where their first
call sets the array up) or after the rest of the suite.  The file is named to
be collected last, so that a run which stops at its first failure has run
every other test before it."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import cheby_ref as R
from orthossm_b200 import _lib as L
from tests.golden.inputs import det_normal, linear_init, spectral_coeffs
from tests.test_oracle_golden import relerr

pytestmark = pytest.mark.gpu


def _t(a, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dt)


def _inputs(B, S, x_dtype, seed):
    H, hd = 8, 64
    D = H * hd
    x = R.bf16_round(det_normal((B, S, D), seed)).astype(np.float32)
    c = spectral_coeffs(B, H, 8, hd, seed + 1).astype(np.float32)
    W, b = linear_init(H, D, seed + 2)
    init = det_normal((B, D), seed + 3, 0.1).astype(np.float32)
    lam = np.asarray(R.BASELINE_LAMBDA, np.float32)
    return dict(x=_t(x, x_dtype), c=_t(c), W=_t(W), b=_t(b), init=_t(init), lam=_t(lam))


def _args(d, out, fin):
    x = d["x"]
    B, S, D = x.shape
    return L.FwdArgs(B=B, S=S, H=8, head_dim=64, degree=8, x=x.data_ptr(),
                     x_dtype=L.OSSM_BF16 if x.dtype == torch.bfloat16 else L.OSSM_F32,
                     x_stride_b=S * D, x_stride_s=D, coeffs=d["c"].data_ptr(), lam_h=d["lam"].data_ptr(),
                     momentum=0.9, gate_w=d["W"].data_ptr(), gate_b=d["b"].data_ptr(), gate_scale=0.008,
                     gate_lo=0.0, gate_hi=1.0, init_state=d["init"].data_ptr(), final_state=fin.data_ptr(),
                     out=out.data_ptr(), out_dtype=L.OSSM_BF16 if out.dtype == torch.bfloat16 else L.OSSM_F32,
                     out_stride_b=S * D, out_stride_s=D)


@pytest.mark.parametrize("x_dtype,out_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32)])
def test_noalloc_matches_workspace_entry_point(x_dtype, out_dtype):
    """Two calls in a row through the fixed scratch against one call with a
    caller workspace: bf16 (the fast path; the bar is one bf16 step and fp32
    rounding of the final state)
    and fp32 (generic kernel, bitwise reproducible)."""
    lib = L.lib()
    torch.cuda.set_device(0)
    B, S, D = 2, 3000, 512
    d = _inputs(B, S, x_dtype, 1100)
    stream = torch.cuda.current_stream().cuda_stream

    out_ref = torch.empty(B, S, D, device="cuda", dtype=out_dtype)
    fin_ref = torch.empty(B, D, device="cuda")
    a = _args(d, out_ref, fin_ref)
    nb = lib.ossm_fwd_workspace_bytes(C.byref(a))
    assert 0 < nb <= L.OSSM_NOALLOC_SCRATCH_BYTES
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    assert lib.ossm_cheby_ema_fwd(C.byref(a), ws.data_ptr(), nb, stream) == L.OSSM_OK

    for call in range(2):
        out = torch.full((B, S, D), float("nan"), device="cuda", dtype=out_dtype)
        fin = torch.full((B, D), float("nan"), device="cuda")
        scratch = L._vp()
        rc = lib.ossm_cheby_ema_fwd_noalloc(C.byref(_args(d, out, fin)), stream, C.byref(scratch))
        assert rc == L.OSSM_OK, (call, lib.ossm_status_string(rc))
        torch.cuda.synchronize()
        assert scratch.value and scratch.value % 256 == 0
        st = L._i32(-1)
        assert lib.ossm_workspace_status(scratch, 1, stream, C.byref(st)) == L.OSSM_OK
        assert st.value == L.OSSM_OK, call
        o, r = out.float().cpu().numpy(), out_ref.float().cpu().numpy()
        assert np.isfinite(o).all()
        if out_dtype == torch.bfloat16:
            assert np.abs(o - r).max() <= 2 ** -7, call
            assert relerr(fin.cpu().numpy(), fin_ref.cpu().numpy()) < 1e-5, call
        else:
            assert relerr(o, r) < 1e-6, call
            assert relerr(fin.cpu().numpy(), fin_ref.cpu().numpy()) < 1e-6, call


def test_noalloc_rejects_sizes_over_the_fixed_scratch():
    """A call whose workspace would not fit is refused before any launch and
    leaves its outputs untouched."""
    lib = L.lib()
    torch.cuda.set_device(0)
    B, D = 1, 512

    def args(S, x=0, c=0, out=0):
        return L.FwdArgs(B=B, S=S, H=8, head_dim=64, degree=8, x=x or 1 << 20, x_dtype=L.OSSM_BF16,
                         x_stride_b=S * D, x_stride_s=D, coeffs=c or 1 << 20, momentum=0.9, out=out or 1 << 20,
                         out_dtype=L.OSSM_BF16, out_stride_b=S * D, out_stride_s=D)
    S = 1 << 16  # the smallest power of two whose workspace exceeds the scratch (size query only)
    while lib.ossm_fwd_workspace_bytes(C.byref(args(S))) <= L.OSSM_NOALLOC_SCRATCH_BYTES:
        S *= 2
    x = torch.zeros(B, S, D, device="cuda", dtype=torch.bfloat16)
    c = torch.zeros(B, 8, 8, 64, device="cuda")
    out = torch.full((B, S, D), 7.0, device="cuda", dtype=torch.bfloat16)
    a = args(S, x.data_ptr(), c.data_ptr(), out.data_ptr())
    assert lib.ossm_fwd_workspace_bytes(C.byref(a)) > L.OSSM_NOALLOC_SCRATCH_BYTES
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.ossm_cheby_ema_fwd_noalloc(C.byref(a), stream, None) == L.OSSM_EWORKSPACE
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())


def test_noalloc_sizes_its_scratch_with_its_own_flags():
    """The entry point keeps all work on the caller's stream (OSSM_F_ONE_STREAM),
    which changes how the bf16 path lays out its scratch for one long
    sequence.  Its size limit must be checked on those flags: for B = 1 and a
    long S the one-stream layout is never larger than the default one."""
    lib = L.lib()
    torch.cuda.set_device(0)
    D = 512
    for S in (4095 * 32, 4096 * 32, 4096 * 32 + 777, 1 << 18):
        a = L.FwdArgs(B=1, S=S, H=8, head_dim=64, degree=8, x=1 << 20, x_dtype=L.OSSM_BF16,
                      x_stride_b=S * D, x_stride_s=D, coeffs=1 << 20, momentum=0.9, out=1 << 20,
                      out_dtype=L.OSSM_BF16, out_stride_b=S * D, out_stride_s=D)
        default = lib.ossm_fwd_workspace_bytes(C.byref(a))
        a.flags = L.OSSM_F_ONE_STREAM
        one = lib.ossm_fwd_workspace_bytes(C.byref(a))
        assert 0 < one <= default, S


def test_noalloc_generic_kernel_across_shapes():
    """fp32 calls (the generic kernel, whose look-back flags live in the
    shared array) of two different shapes back to back, each against the
    workspace entry point: the flags of one shape must not be read as
    published records by the next."""
    lib = L.lib()
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream().cuda_stream
    for B, S, seed in ((2, 3000, 1200), (3, 1111, 1300), (1, 5000, 1400), (2, 3000, 1200)):
        d = _inputs(B, S, torch.float32, seed)
        D = 512
        out_ref = torch.empty(B, S, D, device="cuda")
        fin_ref = torch.empty(B, D, device="cuda")
        a = _args(d, out_ref, fin_ref)
        nb = lib.ossm_fwd_workspace_bytes(C.byref(a))
        ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
        assert lib.ossm_cheby_ema_fwd(C.byref(a), ws.data_ptr(), nb, stream) == L.OSSM_OK
        out = torch.full((B, S, D), float("nan"), device="cuda")
        fin = torch.full((B, D), float("nan"), device="cuda")
        scratch = L._vp()
        rc = lib.ossm_cheby_ema_fwd_noalloc(C.byref(_args(d, out, fin)), stream, C.byref(scratch))
        assert rc == L.OSSM_OK, (B, S, lib.ossm_status_string(rc))
        st = L._i32(-1)
        assert lib.ossm_workspace_status(scratch, 1, stream, C.byref(st)) == L.OSSM_OK
        assert st.value == L.OSSM_OK, (B, S)
        assert relerr(out.cpu().numpy(), out_ref.cpu().numpy()) < 1e-6, (B, S)
        assert relerr(fin.cpu().numpy(), fin_ref.cpu().numpy()) < 1e-6, (B, S)
