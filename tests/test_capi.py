"""C-ABI library: loads, exports every symbol include/orthossm_b200.h declares,
struct layouts agree with the ctypes binding, argument checks reject bad input
without touching a GPU."""
import ctypes as C
import os
import re

import pytest

from orthossm_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "orthossm_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ossm_[a-z0-9_]+)\s*\(", src)))


def test_header_matches_binding_list():
    assert declared_symbols() == sorted(L.EXPORTED)


def test_library_loads_and_exports_all():
    lib = L.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert b"sm_100a" in lib.ossm_version()


def test_struct_layouts():
    lib = L.lib()
    assert lib.ossm_sizeof_fwd_args() == C.sizeof(L.FwdArgs)
    assert lib.ossm_sizeof_lion_args() == C.sizeof(L.LionArgs)


def test_status_strings():
    lib = L.lib()
    for s in range(6):
        assert lib.ossm_status_string(s)


def _args(**kw):
    a = dict(B=1, S=16, H=8, head_dim=64, degree=8, x=4096, x_dtype=L.OSSM_BF16, x_stride_b=16 * 512,
             x_stride_s=512, coeffs=8192, out=16384, out_dtype=L.OSSM_BF16, out_stride_b=16 * 512,
             out_stride_s=512, momentum=0.9)
    a.update(kw)
    return L.FwdArgs(**a)


def test_workspace_size_and_validation():
    lib = L.lib()
    ok = _args()
    n = lib.ossm_fwd_workspace_bytes(C.byref(ok))
    assert n > 256 and n % 256 == 0
    bad = [_args(head_dim=48), _args(head_dim=4), _args(degree=9), _args(degree=0), _args(S=0),
           _args(x=4098), _args(x_stride_s=100), _args(flags=3), _args(flags=L.OSSM_EVAL_LUT),
           _args(out_dtype=7), _args(gate_w=4096)]
    for a in bad:
        assert lib.ossm_fwd_workspace_bytes(C.byref(a)) == 0
        # rejected before any CUDA call
        assert lib.ossm_cheby_ema_fwd(C.byref(a), None, 0, None) == L.OSSM_EINVAL
    assert lib.ossm_cheby_ema_fwd(C.byref(ok), None, 0, None) == L.OSSM_EWORKSPACE


def test_gate_workspace_grows_with_tokens():
    lib = L.lib()
    a = _args(gate_w=4096, gate_b=4096, lam_h=4096)
    b = _args(S=32, x_stride_b=32 * 512, out_stride_b=32 * 512, gate_w=4096, gate_b=4096, lam_h=4096)
    assert lib.ossm_fwd_workspace_bytes(C.byref(b)) > lib.ossm_fwd_workspace_bytes(C.byref(a))


def test_lion_validation():
    lib = L.lib()
    a = L.LionArgs(B=1, S=16, H=8, head_dim=8, degree=4, chunk=0, x=4096, x_dtype=L.OSSM_F32,
                   x_stride_b=16 * 64, x_stride_s=64, coeffs=8192, momentum=8192, out=4096,
                   out_dtype=L.OSSM_F32, out_stride_b=16 * 64, out_stride_s=64)
    assert lib.ossm_cheby_rkv_lion(C.byref(a), None) == L.OSSM_EINVAL
    a.chunk = 8
    a.flags = L.OSSM_EVAL_LUT  # LUT mode without a table
    assert lib.ossm_cheby_rkv_lion(C.byref(a), None) == L.OSSM_EINVAL


def test_ops_refuse_cpu_tensors():
    import torch
    from orthossm_b200 import cheby_ema_forward
    with pytest.raises(RuntimeError, match="CUDA"):
        cheby_ema_forward(torch.zeros(1, 8, 64), torch.zeros(1, 8, 8, 8))


def test_host_workspace_size_and_validation():
    """ossm_fwd_host_workspace_bytes: the device forward's workspace for the
    largest part plus the part plan's staging buffers; no GPU needed."""
    lib = L.lib()
    B, S = 8, 4096
    base = dict(B=B, S=S, x_stride_b=S * 512, out_stride_b=S * 512)
    n8 = lib.ossm_fwd_host_workspace_bytes(C.byref(_args(**base)), 8)
    n16 = lib.ossm_fwd_host_workspace_bytes(C.byref(_args(**base)), 16)
    one_part = S * 512 * 2  # one sequence of bf16 activations
    assert n8 % 256 == 0 and n8 >= 2 * 2 * one_part  # two x and two out buffers of one sequence each
    assert n16 < n8  # 16 parts: half sequences
    assert lib.ossm_fwd_host_workspace_bytes(C.byref(_args(**base)), 1) >= 2 * 2 * B * one_part
    bad = [(_args(**base), 0), (_args(**dict(base, x_stride_b=S * 512 + 512)), 8),
           (_args(**dict(base, out_stride_s=1024)), 8), (_args(**dict(base, tanh_out=4096)), 8),
           (_args(**dict(base, degree=9)), 8)]
    for a, pieces in bad:
        assert lib.ossm_fwd_host_workspace_bytes(C.byref(a), pieces) == 0
    assert lib.ossm_cheby_ema_fwd_host(C.byref(_args(**base)), 8, None, 0, None) == L.OSSM_EWORKSPACE
    assert lib.ossm_cheby_ema_fwd_host(C.byref(_args(**dict(base, tanh_out=4096))), 8, None, 0, None) == L.OSSM_EINVAL
