"""ctypes binding of the orthossm_b200 C ABI (include/orthossm_b200.h).

The shared library is built in-tree by ``orthossm_b200.build``.  There is no
fallback: if the library cannot be loaded, every op raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from . import build as _build

OSSM_OK, OSSM_EINVAL, OSSM_ELAUNCH, OSSM_ETIMEOUT, OSSM_ECOMM, OSSM_EWORKSPACE = range(6)
OSSM_F32, OSSM_BF16 = 0, 1
OSSM_EVAL_CLENSHAW, OSSM_EVAL_LUT, OSSM_EVAL_CLENSHAW_DEG4 = 0, 1, 2
OSSM_F_FASTPATH = 1 << 2
OSSM_F_PRECISE = 1 << 3
OSSM_F_GENERIC = 1 << 4
OSSM_F_SINGLE_EVAL = 1 << 5
OSSM_F_ONE_STREAM = 1 << 7
OSSM_NOALLOC_SCRATCH_BYTES = 16 << 20
OSSM_PATH_GENERIC, OSSM_PATH_THREE_PASS, OSSM_PATH_GROUPED, OSSM_PATH_PARKED = 0, 1, 2, 3

EXPORTED = (
    "ossm_fwd_workspace_bytes", "ossm_fwd_path", "ossm_cheby_ema_fwd", "ossm_cheby_ema_fwd_noalloc", "ossm_gate_decay",
    "ossm_fwd_host_workspace_bytes", "ossm_cheby_ema_fwd_host",
    "ossm_workspace_status", "ossm_fwd_shard_aggregate", "ossm_fwd_shard_output", "ossm_fwd_shard_fold",
    "ossm_cheby_rkv_lion", "ossm_version", "ossm_status_string",
    "ossm_sizeof_fwd_args", "ossm_sizeof_lion_args", "ossm_sizeof_ttt_args",
    "ossm_ttt_workspace_bytes", "ossm_ttt_wpred_step", "ossm_sizeof_bwd_args", "ossm_bwd_workspace_bytes",
    "ossm_cheby_ema_bwd", "ossm_ttt_run_workspace_bytes", "ossm_ttt_wpred_run", "ossm_sizeof_ttt_run_args",
)

_vp = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64
_f32 = C.c_float


class FwdArgs(C.Structure):
    _fields_ = [
        ("B", _i32), ("S", _i32), ("H", _i32), ("head_dim", _i32), ("degree", _i32),
        ("x", _vp), ("x_dtype", _i32), ("x_stride_b", _i64), ("x_stride_s", _i64),
        ("coeffs", _vp), ("lam_h", _vp), ("momentum", _f32),
        ("gate_w", _vp), ("gate_b", _vp), ("gate_scale", _f32), ("gate_lo", _f32), ("gate_hi", _f32),
        ("lut", _vp), ("init_state", _vp), ("final_state", _vp),
        ("out", _vp), ("out_dtype", _i32), ("out_stride_b", _i64), ("out_stride_s", _i64),
        ("tanh_out", _vp), ("lam_tok", _vp), ("flags", C.c_uint32),
    ]


class LionArgs(C.Structure):
    _fields_ = [
        ("B", _i32), ("S", _i32), ("H", _i32), ("head_dim", _i32), ("degree", _i32), ("chunk", _i32),
        ("x", _vp), ("x_dtype", _i32), ("x_stride_b", _i64), ("x_stride_s", _i64),
        ("coeffs", _vp), ("momentum", _vp), ("gate_global", _vp), ("dynamic_lambda", _vp),
        ("ema_momentum", _f32), ("base_lr", _f32), ("beta1", _f32), ("beta2", _f32),
        ("weight_decay", _f32),
        ("lut", _vp), ("out", _vp), ("out_dtype", _i32), ("out_stride_b", _i64), ("out_stride_s", _i64),
        ("tanh_out", _vp), ("final_state", _vp), ("flags", C.c_uint32), ("coeff_trace", _vp),
    ]


class TttArgs(C.Structure):
    _fields_ = [
        ("B", _i32), ("L", _i32), ("H", _i32), ("head_dim", _i32), ("degree", _i32),
        ("x", _vp), ("x_dtype", _i32), ("x_stride_b", _i64), ("x_stride_s", _i64),
        ("coeffs", _vp), ("m", _vp), ("v", _vp), ("lam_h", _vp), ("momentum", _f32), ("lam_tok", _vp),
        ("gs", _vp), ("lr", _f32), ("beta1", _f32), ("beta2", _f32), ("eps", _f32), ("spectral_pow", _f32),
        ("step", _i32), ("forget", _i32),
    ]


class TttRunArgs(C.Structure):
    _fields_ = [
        ("B", _i32), ("S", _i32), ("H", _i32), ("head_dim", _i32), ("degree", _i32), ("chunk", _i32),
        ("x", _vp), ("x_dtype", _i32), ("x_stride_b", _i64), ("x_stride_s", _i64),
        ("coeffs", _vp), ("m", _vp), ("v", _vp), ("lam_h", _vp), ("momentum", _f32),
        ("gate_w", _vp), ("gate_b", _vp), ("gate_scale", _f32), ("gate_lo", _f32), ("gate_hi", _f32),
        ("w_pred", _vp), ("init_state", _vp), ("final_state", _vp), ("out", _vp),
        ("lr", _f32), ("beta1", _f32), ("beta2", _f32), ("eps", _f32), ("spectral_pow", _f32),
        ("step0", _i32), ("forget", _i32), ("flags", C.c_uint32),
    ]


class BwdArgs(C.Structure):
    _fields_ = [
        ("B", _i32), ("S", _i32), ("H", _i32), ("head_dim", _i32), ("degree", _i32),
        ("x", _vp), ("x_dtype", _i32), ("x_stride_b", _i64), ("x_stride_s", _i64),
        ("coeffs", _vp), ("lam_h", _vp), ("momentum", _f32), ("lam_tok", _vp), ("init_state", _vp),
        ("grad_out", _vp), ("grad_out_dtype", _i32), ("grad_out_stride_b", _i64), ("grad_out_stride_s", _i64),
        ("grad_x", _vp), ("grad_x_dtype", _i32), ("grad_x_stride_b", _i64), ("grad_x_stride_s", _i64),
        ("grad_coeffs", _vp), ("grad_init", _vp), ("segment", _i32), ("segment_coeffs", _vp),
        ("flags", C.c_uint32),
    ]


_lock = threading.Lock()
_lib = None


def _declare(lib):
    lib.ossm_fwd_workspace_bytes.restype = C.c_size_t
    lib.ossm_fwd_workspace_bytes.argtypes = [C.POINTER(FwdArgs)]
    lib.ossm_fwd_path.restype = C.c_int
    lib.ossm_fwd_path.argtypes = [C.POINTER(FwdArgs)]
    lib.ossm_cheby_ema_fwd.restype = C.c_int
    lib.ossm_cheby_ema_fwd.argtypes = [C.POINTER(FwdArgs), _vp, C.c_size_t, _vp]
    lib.ossm_cheby_ema_fwd_noalloc.restype = C.c_int
    lib.ossm_cheby_ema_fwd_noalloc.argtypes = [C.POINTER(FwdArgs), _vp, C.POINTER(_vp)]
    lib.ossm_fwd_host_workspace_bytes.restype = C.c_size_t
    lib.ossm_fwd_host_workspace_bytes.argtypes = [C.POINTER(FwdArgs), C.c_int]
    lib.ossm_cheby_ema_fwd_host.restype = C.c_int
    lib.ossm_cheby_ema_fwd_host.argtypes = [C.POINTER(FwdArgs), C.c_int, _vp, C.c_size_t, _vp]
    lib.ossm_fwd_shard_aggregate.restype = C.c_int
    lib.ossm_fwd_shard_aggregate.argtypes = [C.POINTER(FwdArgs), C.c_int, _vp, C.c_size_t, _vp, _vp, _vp]
    lib.ossm_fwd_shard_output.restype = C.c_int
    lib.ossm_fwd_shard_output.argtypes = [C.POINTER(FwdArgs), C.c_int, _vp, _vp, _vp, C.c_size_t, _vp]
    lib.ossm_fwd_shard_fold.restype = C.c_int
    lib.ossm_fwd_shard_fold.argtypes = [C.c_int32, C.c_int32, C.c_int32, C.c_int32, _vp, _vp, _vp, _vp]
    lib.ossm_gate_decay.restype = C.c_int
    lib.ossm_gate_decay.argtypes = [C.POINTER(FwdArgs), _vp, _vp]
    lib.ossm_workspace_status.restype = C.c_int
    lib.ossm_workspace_status.argtypes = [_vp, C.c_int, _vp, C.POINTER(_i32)]
    lib.ossm_cheby_rkv_lion.restype = C.c_int
    lib.ossm_cheby_rkv_lion.argtypes = [C.POINTER(LionArgs), _vp]
    lib.ossm_version.restype = C.c_char_p
    lib.ossm_status_string.restype = C.c_char_p
    lib.ossm_status_string.argtypes = [C.c_int]
    lib.ossm_sizeof_fwd_args.restype = C.c_size_t
    lib.ossm_sizeof_lion_args.restype = C.c_size_t
    lib.ossm_sizeof_ttt_args.restype = C.c_size_t
    lib.ossm_sizeof_bwd_args.restype = C.c_size_t
    lib.ossm_bwd_workspace_bytes.restype = C.c_size_t
    lib.ossm_bwd_workspace_bytes.argtypes = [C.POINTER(BwdArgs)]
    lib.ossm_cheby_ema_bwd.restype = C.c_int
    lib.ossm_cheby_ema_bwd.argtypes = [C.POINTER(BwdArgs), _vp, C.c_size_t, _vp]
    lib.ossm_ttt_workspace_bytes.restype = C.c_size_t
    lib.ossm_ttt_workspace_bytes.argtypes = [C.POINTER(TttArgs)]
    lib.ossm_ttt_wpred_step.restype = C.c_int
    lib.ossm_ttt_wpred_step.argtypes = [C.POINTER(TttArgs), _vp, C.c_size_t, _vp]
    lib.ossm_ttt_run_workspace_bytes.restype = C.c_size_t
    lib.ossm_ttt_run_workspace_bytes.argtypes = [C.POINTER(TttRunArgs)]
    lib.ossm_ttt_wpred_run.restype = C.c_int
    lib.ossm_ttt_wpred_run.argtypes = [C.POINTER(TttRunArgs), _vp, C.c_size_t, _vp]
    lib.ossm_sizeof_ttt_run_args.restype = C.c_size_t
    if lib.ossm_sizeof_ttt_run_args() != C.sizeof(TttRunArgs):
        raise RuntimeError("orthossm_b200: ctypes struct layout does not match the C ABI")
    if (lib.ossm_sizeof_fwd_args() != C.sizeof(FwdArgs) or lib.ossm_sizeof_lion_args() != C.sizeof(LionArgs)
            or lib.ossm_sizeof_ttt_args() != C.sizeof(TttArgs) or lib.ossm_sizeof_bwd_args() != C.sizeof(BwdArgs)):
        raise RuntimeError("orthossm_b200: ctypes struct layout does not match the C ABI")
    return lib


def lib():
    """Load (building first if the library is absent and nvcc exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = _build.lib_path()
            if not os.path.exists(path):
                try:
                    path = _build.build()
                except Exception as e:  # no silent fallback: the op cannot run
                    raise RuntimeError(f"orthossm_b200: CUDA library missing and build failed: {e}")
            _lib = _declare(C.CDLL(path))
    return _lib


def check(status: int, what: str):
    if status != OSSM_OK:
        msg = lib().ossm_status_string(status).decode()
        raise RuntimeError(f"orthossm_b200: {what} failed: {msg} (status {status})")
