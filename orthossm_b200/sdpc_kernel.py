"""Host-side mirror of the reference op API (Eddym06/OrthoSSM ``sdpc_kernel.py``).

Same names, argument meanings and return values as the reference's public
surface for the Cheby-RKV path, backed by hand-written sm_100a CUDA through
the C ABI in ``include/orthossm_b200.h``:

* ``apply_cheby_rkv_v10`` / ``apply_cheby_rkv_core`` (sdpc_kernel.py:2522-2610)
* ``FusedChebyRKVv10.apply`` (:2351-2515, 16 positional arguments)
* ``get_chebyshev_lut`` / ``LUT_TABLE_SIZE`` / ``MAX_DEGREE`` (:59-96)
* ``MULTI_SCALE_LAMBDA`` (:1416), ``init_chebyshev_coefficients`` (:1833-1867),
  ``GatedComplexityPredictor`` (:1818-1830)

plus the BASELINE-semantics forward ``cheby_ema_forward`` (per-head decay,
per-token dynamic decay from a Linear(D->H) gate, carried state, bf16 I/O).

Tensors must live on a CUDA device; there is no CPU path and no fallback.
"""
from __future__ import annotations

import threading

import torch
import torch.nn as nn

from . import _lib as L

LUT_TABLE_SIZE: int = 256
MAX_DEGREE: int = 8
MULTI_SCALE_LAMBDA = [0.9995, 0.9995, 0.997, 0.997, 0.995, 0.995, 0.97, 0.95]
BASELINE_LAMBDA = [0.9995, 0.9995, 0.997, 0.997, 0.995, 0.995, 0.95, 0.95]

_DT = {torch.float32: L.OSSM_F32, torch.bfloat16: L.OSSM_BF16}


# ----------------------------------------------------------------------------
# reference helpers
# ----------------------------------------------------------------------------

def _build_chebyshev_lut(table_size: int = LUT_TABLE_SIZE, max_degree: int = MAX_DEGREE):
    """T_k(u) for u on a uniform grid of [0, 1] (half table; odd degrees are
    mirrored with the sign of x), float32 [max_degree, table_size]."""
    u = torch.linspace(0.0, 1.0, table_size)
    T = torch.empty(max_degree, table_size)
    T[0] = 1.0
    if max_degree > 1:
        T[1] = u
    for k in range(2, max_degree):
        T[k] = 2.0 * u * T[k - 1] - T[k - 2]
    return T


_LUT_CPU = _build_chebyshev_lut()
_LUT_DEV: dict = {}
_LUT_LOCK = threading.Lock()


def get_chebyshev_lut(device):
    """Per-device cached LUT (thread safe)."""
    key = torch.device(device)
    t = _LUT_DEV.get(key)
    if t is None:
        with _LUT_LOCK:
            t = _LUT_DEV.get(key)
            if t is None:
                t = _LUT_CPU.to(key).contiguous()
                _LUT_DEV[key] = t
    return t


class GatedComplexityPredictor(nn.Module):
    """Global TTT gate from mean(x): Linear(D, D/4) - SiLU - Linear(D/4, 1) - Sigmoid."""

    def __init__(self, d_model):
        super().__init__()
        self.net = nn.Sequential(nn.Linear(d_model, d_model // 4), nn.SiLU(),
                                 nn.Linear(d_model // 4, 1), nn.Sigmoid())

    def forward(self, x_mean):
        return self.net(x_mean)


def init_chebyshev_coefficients(batch, n_heads, degree, head_dim, device):
    """Spectral init c ~ N(0, (0.1/(k+1))^2) with heads orthogonalised by QR
    (or a Parseval tight frame by SVD when degree*head_dim < n_heads)."""
    k = torch.arange(degree, device=device, dtype=torch.float32)
    sigma = (0.1 / (k + 1.0)).view(1, 1, degree, 1)
    c = torch.randn(batch, n_heads, degree, head_dim, device=device) * sigma
    if n_heads < 2:
        return c
    flat = c.reshape(batch, n_heads, degree * head_dim)
    norms = flat.norm(dim=2, keepdim=True)
    if degree * head_dim >= n_heads:
        q, _ = torch.linalg.qr(flat.transpose(1, 2))
        return (q.transpose(1, 2) * norms).reshape(batch, n_heads, degree, head_dim)
    unit = flat / (norms + 1e-8)
    rank = min(n_heads, degree * head_dim)
    scale = (n_heads / rank) ** 0.5
    for b in range(batch):
        U, _, Vh = torch.linalg.svd(unit[b], full_matrices=False)
        unit[b] = U[:, :rank] @ Vh[:rank] * scale
    return (unit * norms).reshape(batch, n_heads, degree, head_dim)


# ----------------------------------------------------------------------------
# workspace (look-back flags / aggregates); one per (device, stream)
# ----------------------------------------------------------------------------

_WS: dict = {}
_WS_HOST: dict = {}  # host-buffer calls: staging buffers inside, never shared with the others
_WS_LOCK = threading.Lock()


def _workspace(device, stream, nbytes, host=False):
    key = (device, stream.cuda_stream)
    cache = _WS_HOST if host else _WS
    with _WS_LOCK:
        ws = cache.get(key)
        if ws is None or ws.numel() < nbytes:
            # zero-filled once: ticket / epoch / flags start at 0
            ws = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
            cache[key] = ws
    return ws


def workspace_status(device=None, clear=True):
    """Sticky device status over every workspace of a device (0 = ok,
    3 = a look-back wait timed out).  Synchronises each workspace's stream."""
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    worst = 0
    for (d, sptr), ws in list(_WS.items()) + list(_WS_HOST.items()):
        if d != device:
            continue
        st = L._i32(0)
        L.check(L.lib().ossm_workspace_status(ws.data_ptr(), int(clear), sptr, L.C.byref(st)),
                "workspace_status")
        worst = max(worst, int(st.value))
    return worst


def _ptr(t):
    return None if t is None else t.data_ptr()


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("orthossm_b200 ops run on CUDA tensors only (no CPU path)")


def _rowmajor(x):
    """[B,S,D] with unit channel stride (copy otherwise)."""
    return x if x.stride(-1) == 1 else x.contiguous()


# ----------------------------------------------------------------------------
# BASELINE-semantics forward
# ----------------------------------------------------------------------------

def _fwd_args(x, coeffs, *, lambda_per_head=None, ema_momentum=0.9, gate_weight=None, gate_bias=None,
              gate_scale=0.008, gate_range=(0.0, 1.0), init_state=None, out_dtype=None, return_tanh=False,
              eval_mode="clenshaw", fast_path_semantics=False, precise=None, out=None, final_state=None,
              lam_tok=None, force_generic=False, extra_flags=0, host=False, device=None):
    """ossm_fwd_args for a forward call; returns (args, tensors to keep alive,
    out, final_state).  extra_flags: further OSSM_F_* kernel selections.
    host: x, out, init_state and final_state are host tensors (given, for
    ``out`` and ``final_state``), every other tensor lives on ``device``."""
    if host:
        _need_cuda(coeffs)
        if x.is_cuda or not x.is_contiguous() or x.dtype not in _DT:
            raise ValueError("host forward: x must be a contiguous bf16 or fp32 host tensor")
    else:
        _need_cuda(x, coeffs)
        x = _rowmajor(x)
        if x.dtype not in _DT:
            x = x.float()
    B, S, D = x.shape
    coeffs = coeffs.contiguous().float()
    H, K, hd = coeffs.shape[1], coeffs.shape[2], coeffs.shape[3]
    if H * hd != D or coeffs.shape[0] != B:
        raise ValueError(f"coeffs {tuple(coeffs.shape)} do not match x {tuple(x.shape)}")
    dev = torch.device(device) if host else x.device
    odt = out_dtype or x.dtype
    if out is None:
        out = torch.empty(B, S, D, device=dev, dtype=odt)
    if final_state is None:
        final_state = torch.empty(B, D, device=dev, dtype=torch.float32)
    lam = None
    if lambda_per_head is not None:
        lam = torch.as_tensor(lambda_per_head, dtype=torch.float32, device=dev).contiguous()
    if gate_weight is not None:
        gate_weight = gate_weight.to(dev, torch.float32).contiguous()
        gate_bias = gate_bias.to(dev, torch.float32).contiguous()
        if lam is None:
            lam = torch.full((H,), float(ema_momentum), device=dev)
    if init_state is not None:
        init_state = init_state.to(torch.device("cpu") if host else dev, torch.float32).contiguous()
    if lam_tok is not None:
        _need_cuda(lam_tok)
        lam_tok = lam_tok.float().contiguous()
        if tuple(lam_tok.shape) != (B, S, H):
            raise ValueError(f"lam_tok must be [B,S,H] = {(B, S, H)}")
    tanh = torch.empty(B, S, D, device=dev, dtype=torch.float32) if return_tanh else None
    if tanh is not None and out.stride() != tanh.stride():
        raise ValueError("tanh cache needs the output's strides")
    flags = {"clenshaw": L.OSSM_EVAL_CLENSHAW, "lut": L.OSSM_EVAL_LUT,
             "clenshaw_deg4": L.OSSM_EVAL_CLENSHAW_DEG4}[eval_mode]
    if fast_path_semantics:
        flags |= L.OSSM_F_FASTPATH
    if precise:
        flags |= L.OSSM_F_PRECISE
    if force_generic:
        flags |= L.OSSM_F_GENERIC
    flags |= int(extra_flags)
    lut = get_chebyshev_lut(dev) if eval_mode == "lut" else None
    a = L.FwdArgs(B=B, S=S, H=H, head_dim=hd, degree=K,
                  x=x.data_ptr(), x_dtype=_DT[x.dtype], x_stride_b=x.stride(0), x_stride_s=x.stride(1),
                  coeffs=coeffs.data_ptr(), lam_h=_ptr(lam), momentum=float(ema_momentum),
                  gate_w=_ptr(gate_weight), gate_b=_ptr(gate_bias), gate_scale=float(gate_scale),
                  gate_lo=float(gate_range[0]), gate_hi=float(gate_range[1]),
                  lut=_ptr(lut), init_state=_ptr(init_state), final_state=_ptr(final_state),
                  out=out.data_ptr(), out_dtype=_DT[out.dtype], out_stride_b=out.stride(0),
                  out_stride_s=out.stride(1), tanh_out=_ptr(tanh), lam_tok=_ptr(lam_tok), flags=flags)
    keep = (x, coeffs, lam, gate_weight, gate_bias, init_state, lam_tok, tanh, lut)
    return a, keep, out, final_state


def forward_path(x, coeffs, **kw):
    """Which kernels ``cheby_ema_forward(x, coeffs, **kw)`` runs on x's device:
    "generic", "three_pass", "parked" (three-pass with u parked in L2) or
    "grouped" (no launch)."""
    a, keep, _, _ = _fwd_args(x, coeffs, **kw)
    r = L.lib().ossm_fwd_path(L.C.byref(a))
    del keep
    if r < 0:
        L.check(L.OSSM_EINVAL, "forward_path (argument check)")
    return {L.OSSM_PATH_GENERIC: "generic", L.OSSM_PATH_THREE_PASS: "three_pass", L.OSSM_PATH_GROUPED: "grouped",
            L.OSSM_PATH_PARKED: "parked"}[r]


def cheby_ema_forward(x, coeffs, *, lambda_per_head=None, ema_momentum=0.9, gate_weight=None,
                      gate_bias=None, gate_scale=0.008, gate_range=(0.0, 1.0), init_state=None,
                      out_dtype=None, return_tanh=False, eval_mode="clenshaw",
                      fast_path_semantics=False, precise=None, out=None, final_state=None,
                      lam_tok=None, force_generic=False):
    """Fused softsign -> degree-K Chebyshev -> gamma_h -> tanh -> lambda-EMA,
    differentiable in ``x``, ``coeffs`` and ``init_state`` when autograd needs
    it (``ossm_cheby_ema_bwd``; the decays are constants, as in the
    reference's backward).  See ``_cheby_ema_forward`` for the arguments."""
    needs_grad = torch.is_grad_enabled() and any(
        t is not None and isinstance(t, torch.Tensor) and t.requires_grad for t in (x, coeffs, init_state))
    if not needs_grad:
        return _cheby_ema_forward(
            x, coeffs, lambda_per_head=lambda_per_head, ema_momentum=ema_momentum, gate_weight=gate_weight,
            gate_bias=gate_bias, gate_scale=gate_scale, gate_range=gate_range, init_state=init_state,
            out_dtype=out_dtype, return_tanh=return_tanh, eval_mode=eval_mode,
            fast_path_semantics=fast_path_semantics, precise=precise, out=out, final_state=final_state,
            lam_tok=lam_tok, force_generic=force_generic)
    if eval_mode != "clenshaw" or return_tanh or out is not None or final_state is not None:
        raise NotImplementedError("orthossm_b200: the backward covers the Clenshaw forward with fresh outputs")
    H = coeffs.shape[1]
    lam = torch.as_tensor(lambda_per_head if lambda_per_head is not None else [ema_momentum] * H,
                          dtype=torch.float32, device=x.device).contiguous()
    if lam_tok is None and gate_weight is not None:  # the gate's decays, held constant
        lam_tok = gate_decay(x.detach(), gate_weight.detach(), gate_bias.detach(), lam, gate_scale=gate_scale,
                             gate_range=gate_range)
    opts = dict(ema_momentum=float(ema_momentum), out_dtype=out_dtype, precise=precise,
                force_generic=force_generic, fast_path_semantics=fast_path_semantics)
    return _ChebyEmaFn.apply(x, coeffs, init_state, lam, lam_tok, opts)


def _rev_backward(x, g, coeffs, *, lam=None, momentum=0.9, lam_tok=None, init=None, want_init=False,
                  segment=0, segment_coeffs=None, fastpath=False):
    """ossm_cheby_ema_bwd: (grad_x f32, grad_coeffs f32, grad_init or None)."""
    x = _rowmajor(x.detach())
    if x.dtype not in _DT:
        x = x.float()
    B, S, D = x.shape
    c = coeffs.detach().contiguous().float()
    H, K, hd = c.shape[1], c.shape[2], c.shape[3]
    g = g.float().contiguous()
    gx = torch.empty(B, S, D, device=x.device, dtype=torch.float32)
    gc = torch.empty_like(c)
    gi = torch.empty(B, D, device=x.device) if want_init else None
    init = None if init is None else init.detach().float().contiguous()
    sc = None if segment_coeffs is None else segment_coeffs.detach().float().contiguous()
    a = L.BwdArgs(B=B, S=S, H=H, head_dim=hd, degree=K, x=x.data_ptr(), x_dtype=_DT[x.dtype],
                  x_stride_b=x.stride(0), x_stride_s=x.stride(1), coeffs=c.data_ptr(), lam_h=_ptr(lam),
                  momentum=float(momentum), lam_tok=_ptr(lam_tok), init_state=_ptr(init), grad_out=g.data_ptr(),
                  grad_out_dtype=L.OSSM_F32, grad_out_stride_b=g.stride(0), grad_out_stride_s=g.stride(1),
                  grad_x=gx.data_ptr(), grad_x_dtype=L.OSSM_F32, grad_x_stride_b=gx.stride(0),
                  grad_x_stride_s=gx.stride(1), grad_coeffs=gc.data_ptr(), grad_init=_ptr(gi),
                  segment=int(segment), segment_coeffs=_ptr(sc), flags=L.OSSM_F_FASTPATH if fastpath else 0)
    lib = L.lib()
    nbytes = lib.ossm_bwd_workspace_bytes(L.C.byref(a))
    if nbytes == 0:
        L.check(L.OSSM_EINVAL, "backward (argument check)")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    L.check(lib.ossm_cheby_ema_bwd(L.C.byref(a), ws.data_ptr(), nbytes,
                                   torch.cuda.current_stream(x.device).cuda_stream), "cheby_ema_bwd")
    return gx, gc, gi


class _ChebyEmaFn(torch.autograd.Function):
    """Autograd node of the forward; backward through ``ossm_cheby_ema_bwd``."""

    @staticmethod
    def forward(ctx, x, coeffs, init_state, lam, lam_tok, opts):
        out, fin = _cheby_ema_forward(x.detach(), coeffs.detach(), lambda_per_head=lam, lam_tok=lam_tok,
                                      init_state=None if init_state is None else init_state.detach(), **opts)
        ctx.save_for_backward(x, coeffs, init_state, lam, lam_tok)
        ctx.has_init = init_state is not None
        ctx.momentum = opts["ema_momentum"]
        ctx.fastpath = bool(opts.get("fast_path_semantics"))
        return out, fin

    @staticmethod
    def backward(ctx, g_out, g_fin):
        x, coeffs, init_state, lam, lam_tok = ctx.saved_tensors
        B, S, D = x.shape
        g = torch.zeros(B, S, D, device=x.device) if g_out is None else g_out.float().clone()
        if g_fin is not None:  # the final state is the last token's state
            g[:, -1] += g_fin.float()
        gx, gc, gi = _rev_backward(x, g, coeffs, lam=lam, momentum=ctx.momentum, lam_tok=lam_tok,
                                   init=init_state, want_init=ctx.has_init, fastpath=ctx.fastpath)
        return gx.to(x.dtype), gc.to(coeffs.dtype), gi, None, None, None


def _cheby_ema_forward(x, coeffs, *, lambda_per_head=None, ema_momentum=0.9, gate_weight=None,
                       gate_bias=None, gate_scale=0.008, gate_range=(0.0, 1.0), init_state=None,
                       out_dtype=None, return_tanh=False, eval_mode="clenshaw",
                       fast_path_semantics=False, precise=None, out=None, final_state=None,
                       lam_tok=None, force_generic=False, extra_flags=0):
    """Fused softsign -> degree-K Chebyshev -> gamma_h -> tanh -> lambda-EMA.

    x: [B,S,D] float32 or bfloat16 (CUDA); coeffs: [B,H,K,hd] float32.
    lambda_per_head: [H] decay per head (None: scalar ``ema_momentum``).
    gate_weight [H,D] / gate_bias [H]: per-token decay
    ``clamp(lambda_h + gate_scale*(sigmoid(W x_t + b) - 0.5), *gate_range)``.
    init_state: [B,D] float32 carried-in EMA state (None: zeros).
    lam_tok: optional precomputed per-token decay [B,S,H] float32 (e.g. from
    ``gate_decay``); overrides the gate.
    force_generic: run the generic kernel even where the TMA / tcgen05 path
    applies (bf16 x, head_dim 64); both compute the same function.
    extra_flags: further OSSM_F_* kernel selections (e.g. OSSM_F_ONE_STREAM),
    all computing the same function.
    Returns (out [B,S,D] in out_dtype (default x.dtype), final_state [B,D] f32)
    and the f32 tanh cache when ``return_tanh``."""
    a, keep, out, final_state = _fwd_args(
        x, coeffs, lambda_per_head=lambda_per_head, ema_momentum=ema_momentum, gate_weight=gate_weight,
        gate_bias=gate_bias, gate_scale=gate_scale, gate_range=gate_range, init_state=init_state,
        out_dtype=out_dtype, return_tanh=return_tanh, eval_mode=eval_mode,
        fast_path_semantics=fast_path_semantics, precise=precise, out=out, final_state=final_state,
        lam_tok=lam_tok, force_generic=force_generic, extra_flags=extra_flags)
    tanh = keep[7]
    dev = out.device
    lib = L.lib()
    nbytes = lib.ossm_fwd_workspace_bytes(L.C.byref(a))
    if nbytes == 0:
        L.check(L.OSSM_EINVAL, "cheby_ema_forward (argument check)")
    stream = torch.cuda.current_stream(dev)
    ws = _workspace(dev, stream, nbytes)
    L.check(lib.ossm_cheby_ema_fwd(L.C.byref(a), ws.data_ptr(), ws.numel(), stream.cuda_stream),
            "cheby_ema_forward")
    if return_tanh:
        return out, final_state, tanh
    return out, final_state


# ----------------------------------------------------------------------------
# sequence sharding across ranks
# ----------------------------------------------------------------------------

def fold_shard_carries(decays, states, upto, init=None):
    """State entering shard ``upto`` from every earlier shard's totals.

    decays[q]: [B, H] decay product over shard q; states[q]: [B, D] state at
    the end of shard q from a zero state (shard 0: from ``init``).  Folds
    X_0 = init (or 0), X_{q+1} = decays[q] * X_q + states[q] in rank order, so
    every rank computes bitwise the same carries.  Pure torch: runs on any
    device (the multi-rank tests run it on CPU under gloo)."""
    B, D = states[0].shape
    H = decays[0].shape[-1]
    X = torch.zeros(B, D, dtype=torch.float32, device=states[0].device) if init is None else init.float().clone()
    for q in range(upto):
        dq = decays[q].reshape(B, H, 1).expand(B, H, D // H).reshape(B, D)
        X = torch.addcmul(states[q].reshape(B, D), dq, X)
    return X


def exchange_shard_totals(decay, state, group=None):
    """All-gather every rank's shard totals; returns (decays, states), one
    entry per rank.  The CUDA path packs both into one record and gathers
    once (``cheby_ema_forward_seqpar``); this two-tensor form serves hosts
    that fold on the CPU."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    decays = [torch.empty_like(decay) for _ in range(world)]
    states = [torch.empty_like(state) for _ in range(world)]
    dist.all_gather(decays, decay.contiguous(), group=group)
    dist.all_gather(states, state.contiguous(), group=group)
    return decays, states


def _shard_aggregate(a, starts, ws, record, B, H, stream):
    """Step 1 of the sharded forward on this device: the shard's chunk
    aggregates and carries, and its totals packed into ``record``
    [B*H + B*D] (decays, then end states)."""
    lib = L.lib()
    L.check(lib.ossm_fwd_shard_aggregate(L.C.byref(a), int(starts), ws.data_ptr(), ws.numel(), record.data_ptr(),
                                         record.data_ptr() + B * H * 4, stream.cuda_stream), "shard aggregate")


def _shard_output(a, shard, ws, totals, seq_init, stream):
    """Step 3: the state entering ``shard`` folded on the device from the
    gathered ``totals`` [nshards, B*H + B*D] and ``seq_init``, then the
    shard's outputs."""
    lib = L.lib()
    L.check(lib.ossm_fwd_shard_output(L.C.byref(a), int(shard), totals.data_ptr(), _ptr(seq_init), ws.data_ptr(),
                                      ws.numel(), stream.cuda_stream), "shard output")


def _shard_fold(B, H, hd, nshards, totals, seq_init, stream, out=None):
    """The state after the first ``nshards`` shards, [B, H*hd] float32."""
    lib = L.lib()
    if out is None:
        out = torch.empty(B, H * hd, device=totals.device, dtype=torch.float32)
    L.check(lib.ossm_fwd_shard_fold(B, H, hd, int(nshards), totals.data_ptr(), _ptr(seq_init), out.data_ptr(),
                                    stream.cuda_stream), "shard fold")
    return out


def cheby_ema_forward_seqpar(x, coeffs, *, group=None, lambda_per_head=None, ema_momentum=0.9, gate_weight=None,
                             gate_bias=None, gate_scale=0.008, gate_range=(0.0, 1.0), init_state=None,
                             eval_mode="clenshaw", precise=None, out=None):
    """``cheby_ema_forward`` over a sequence sharded across the ranks of
    ``group`` (torch.distributed, one GPU per rank): rank r holds tokens
    [r*S_shard, (r+1)*S_shard) of every sequence as ``x`` [B, S_shard, D]
    (bf16, 8 heads of 64).  Each rank scans its shard from a zero state, one
    all-gather exchanges the shard totals (B*(H + D) floats per rank, packed
    in one record), and each rank folds the state entering its shard on the
    device (in rank order, so every rank folds bitwise the same carries) and
    writes its outputs.

    ``init_state`` is the state before token 0 (pass the same tensor or None
    on every rank).  Returns (out [B, S_shard, D] bf16, final_state [B, D]
    f32, the state after the last token of the whole sequence, identical on
    every rank)."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    _need_cuda(x, coeffs)
    if x.dtype != torch.bfloat16:
        raise ValueError("cheby_ema_forward_seqpar: x must be bfloat16 (the fast path)")
    a, keep, out, fin = _fwd_args(x, coeffs, lambda_per_head=lambda_per_head, ema_momentum=ema_momentum,
                                  gate_weight=gate_weight, gate_bias=gate_bias, gate_scale=gate_scale,
                                  gate_range=gate_range, init_state=init_state if rank == 0 else None,
                                  out_dtype=torch.bfloat16, eval_mode=eval_mode, precise=precise, out=out)
    B, S, D = x.shape
    H = coeffs.shape[1]
    dev = x.device
    lib = L.lib()
    nbytes = lib.ossm_fwd_workspace_bytes(L.C.byref(a))
    if nbytes == 0:
        L.check(L.OSSM_EINVAL, "cheby_ema_forward_seqpar (argument check)")
    stream = torch.cuda.current_stream(dev)
    ws = _workspace(dev, stream, nbytes)
    rec = B * H + B * D
    record = torch.empty(rec, device=dev, dtype=torch.float32)
    _shard_aggregate(a, rank == 0, ws, record, B, H, stream)
    totals = torch.empty(world, rec, device=dev, dtype=torch.float32)
    dist.all_gather_into_tensor(totals, record, group=group)
    init = None if init_state is None else init_state.to(dev, torch.float32).contiguous()
    _shard_output(a, rank, ws, totals, init, stream)
    final = _shard_fold(B, H, D // H, world, totals, init, stream)
    del keep
    return out, final


def cheby_ema_forward_shards_local(x, coeffs, nshards, *, init_state=None, **kw):
    """The sequence-sharded protocol of ``cheby_ema_forward_seqpar`` with all
    ``nshards`` shards on this device (the all-gather becomes a copy): every
    shard's aggregate pass, then every shard's output pass from the packed
    totals.  Same arithmetic as a multi-GPU run, so it checks the sharded
    path on one GPU.  x: [B, S, D] bf16; returns (out [B, S, D] bf16,
    final_state [B, D])."""
    _need_cuda(x, coeffs)
    B, S, D = x.shape
    H = coeffs.shape[1]
    dev = x.device
    stream = torch.cuda.current_stream(dev)
    lib = L.lib()
    bounds = [S * r // nshards for r in range(nshards + 1)]
    init = None if init_state is None else init_state.to(dev, torch.float32).contiguous()
    out = torch.empty(B, S, D, device=dev, dtype=torch.bfloat16)
    rec = B * H + B * D
    totals = torch.empty(nshards, rec, device=dev, dtype=torch.float32)
    calls = []
    for r in range(nshards):
        xs = x[:, bounds[r]:bounds[r + 1]]
        a, keep, o, f = _fwd_args(xs, coeffs, init_state=init if r == 0 else None, out_dtype=torch.bfloat16,
                                  out=out[:, bounds[r]:bounds[r + 1]], **kw)
        nb = lib.ossm_fwd_workspace_bytes(L.C.byref(a))
        if nb == 0:
            L.check(L.OSSM_EINVAL, "cheby_ema_forward_shards_local (argument check)")
        ws = torch.zeros(nb, dtype=torch.uint8, device=dev)
        _shard_aggregate(a, r == 0, ws, totals[r], B, H, stream)
        calls.append((a, keep, ws))
    for r, (a, keep, ws) in enumerate(calls):
        _shard_output(a, r, ws, totals, init, stream)
    final = _shard_fold(B, H, D // H, nshards, totals, init, stream)
    torch.cuda.current_stream(dev).synchronize()
    del calls
    return out, final


# ----------------------------------------------------------------------------
# host-resident batches: copies overlapped with the forward
# ----------------------------------------------------------------------------


def cheby_ema_forward_host(x_host, coeffs, *, out_host=None, final_host=None, device=None, pieces=8, **kw):
    """``cheby_ema_forward`` of a batch that lives in pinned host memory,
    through the library's host-buffer entry point ``ossm_cheby_ema_fwd_host``.

    The batch goes through the GPU in about ``pieces`` parts: groups of whole
    sequences when there are at least ``pieces`` sequences, else every
    sequence cut into consecutive token ranges (its EMA state carried from
    range to range).  The library overlaps the host-to-device copy of part
    k+1, the forward of part k and the device-to-host copy of part k-1 on its
    own side streams; a PCIe link moves both directions at once, and only
    the first part's copy in and the last part's copy out are not overlapped.
    Eight parts measured best on B200 over PCIe (each copy has a fixed cost,
    so smaller parts lose more than they save at the pipeline's ends).  The
    current stream waits for all of it, so a later host read after a
    synchronisation (or an event on the current stream) sees the results.

    x_host: pinned CPU tensor [B, S, D] (bf16 or fp32), contiguous;
    ``init_state`` is read from the host (a device or pageable one is first
    copied to pinned memory); coeffs and the other keyword arguments as for
    ``cheby_ema_forward`` (device tensors, or small CPU ones, moved once; a
    per-token ``lam_tok`` [B, S, H] stays on the device and is cut with the
    parts).  Returns (out_host [B, S, D] in x's dtype unless ``out_dtype``
    says otherwise, final_host [B, D] fp32), both pinned."""
    if x_host.is_cuda or not x_host.is_pinned():
        raise ValueError("cheby_ema_forward_host: x_host must be a pinned CPU tensor")
    if kw.get("return_tanh"):
        raise NotImplementedError("cheby_ema_forward_host: return_tanh is not supported")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    B, S, D = x_host.shape
    odt = kw.pop("out_dtype", None) or x_host.dtype
    if out_host is None:
        out_host = torch.empty(B, S, D, dtype=odt).pin_memory()
    if final_host is None:
        final_host = torch.empty(B, D, dtype=torch.float32).pin_memory()
    if out_host.is_cuda or not out_host.is_pinned() or not out_host.is_contiguous():
        raise ValueError("cheby_ema_forward_host: out_host must be a contiguous pinned CPU tensor")
    init = kw.pop("init_state", None)
    if init is not None and (init.is_cuda or not init.is_pinned() or init.dtype != torch.float32):
        init = init.detach().to("cpu", torch.float32).contiguous().pin_memory()
    mv = lambda t: t.to(dev, non_blocking=True) if isinstance(t, torch.Tensor) and not t.is_cuda else t  # noqa: E731
    coeffs = mv(coeffs)
    kw = {k: mv(v) for k, v in kw.items()}
    with torch.cuda.device(dev):
        a, keep, _, _ = _fwd_args(x_host, coeffs, init_state=init, out=out_host, final_state=final_host,
                                  out_dtype=odt, host=True, device=dev, **kw)
        lib = L.lib()
        nbytes = lib.ossm_fwd_host_workspace_bytes(L.C.byref(a), int(pieces))
        if nbytes == 0:
            L.check(L.OSSM_EINVAL, "cheby_ema_forward_host (argument check)")
        stream = torch.cuda.current_stream(dev)
        ws = _workspace(dev, stream, nbytes, host=True)
        L.check(lib.ossm_cheby_ema_fwd_host(L.C.byref(a), int(pieces), ws.data_ptr(), ws.numel(), stream.cuda_stream),
                "cheby_ema_forward_host")
    return out_host, final_host


# ----------------------------------------------------------------------------
# BASELINE-mode TTT: W_pred MSE objective + forget-gated Adam
# ----------------------------------------------------------------------------

class _matmul_precision:
    """fp32 matmuls on TF32 tensor cores ("tf32") or in full fp32 ("fp32") for
    the enclosed calls; the caller's setting is restored on exit."""

    def __init__(self, mode):
        if mode not in ("tf32", "fp32"):
            raise ValueError(f"gemm must be 'tf32' or 'fp32', got {mode!r}")
        self.mode = mode

    def __enter__(self):
        self.prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = self.mode == "tf32"

    def __exit__(self, *exc):
        torch.backends.cuda.matmul.allow_tf32 = self.prev


def ttt_wpred_adam(x, coeffs, m, v, step, W_pred, *, lambda_per_head=None, ema_momentum=0.9, gate_weight=None,
                   gate_bias=None, gate_scale=0.008, gate_range=(0.0, 1.0), init_state=None, chunk=2048,
                   lr=1e-3, betas=(0.9, 0.999), eps=1e-8, spectral_pow=2.0, forget=True, gemm="tf32"):
    """Chunked forward + test-time training of the Chebyshev coefficients.

    For each chunk of ``chunk`` tokens: the forward with the chunk-start
    coefficients and the carried EMA state (fp32 states), the loss
    mean_{t<L-1,d} (W_pred s_t - x_{t+1})^2 per sequence, its gradient through
    the EMA, tanh and Chebyshev basis, scaled by 1/(k+1)^spectral_pow, and one
    Adam step with the forget gate c <- lambda_h c - lr mhat/(sqrt(vhat)+eps).
    ``gemm="tf32"`` (default): the whole chunk loop is one native call
    (``ossm_ttt_wpred_run``): per chunk the gate, the forward, one tcgen05
    kernel forming dL/ds = (2/N)(G s_t - W_pred^T x_{t+1}), G = W_pred^T W_pred
    (s . G on TF32 tensor cores, x . W_pred with W_pred split into two bf16
    terms), and the reverse adjoint / gradient / Adam of
    ``ossm_ttt_wpred_step``; it needs H*head_dim a multiple of 256 and
    16-byte aligned rows of x.  ``gemm="fp32"`` (or other shapes) runs the
    chunk loop from Python with the two W_pred products on cuBLAS in full
    fp32 (``"tf32"`` there: TF32 cuBLAS).

    x: [B,S,D] (CUDA, bf16 or fp32); coeffs, m, v: [B,H,K,hd] (not modified);
    step: Adam steps already taken.  Returns dict(out [B,S,D] fp32, coeffs, m,
    v, step, final [B,D])."""
    _need_cuda(x, coeffs, W_pred)
    x = _rowmajor(x)
    B, S, D = x.shape
    dev = x.device
    c = coeffs.detach().float().contiguous().clone()
    m = m.detach().float().contiguous().clone()
    v = v.detach().float().contiguous().clone()
    H, K, hd = c.shape[1], c.shape[2], c.shape[3]
    Wp = W_pred.to(dev, torch.float32).contiguous()
    lam = torch.as_tensor(lambda_per_head if lambda_per_head is not None else [ema_momentum] * H,
                          dtype=torch.float32, device=dev).contiguous()
    state = None if init_state is None else init_state.to(dev, torch.float32).contiguous()
    out = torch.empty(B, S, D, device=dev, dtype=torch.float32)
    lib = L.lib()
    stream = torch.cuda.current_stream(dev)
    xdt = x.dtype if x.dtype in _DT else torch.float32
    x = x.to(xdt)
    if gemm == "tf32":
        gw = gb = None
        if gate_weight is not None:
            gw = gate_weight.to(dev, torch.float32).contiguous()
            gb = gate_bias.to(dev, torch.float32).contiguous()
        fin = torch.empty(B, D, device=dev, dtype=torch.float32)
        a = L.TttRunArgs(B=B, S=S, H=H, head_dim=hd, degree=K, chunk=int(chunk), x=x.data_ptr(), x_dtype=_DT[xdt],
                         x_stride_b=x.stride(0), x_stride_s=x.stride(1), coeffs=c.data_ptr(), m=m.data_ptr(),
                         v=v.data_ptr(), lam_h=lam.data_ptr(), momentum=float(ema_momentum), gate_w=_ptr(gw),
                         gate_b=_ptr(gb), gate_scale=float(gate_scale), gate_lo=float(gate_range[0]),
                         gate_hi=float(gate_range[1]), w_pred=Wp.data_ptr(), init_state=_ptr(state),
                         final_state=fin.data_ptr(), out=out.data_ptr(), lr=float(lr), beta1=float(betas[0]),
                         beta2=float(betas[1]), eps=float(eps), spectral_pow=float(spectral_pow), step0=int(step),
                         forget=int(bool(forget)), flags=0)
        nbytes = lib.ossm_ttt_run_workspace_bytes(L.C.byref(a))
        if nbytes:
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
            L.check(lib.ossm_ttt_wpred_run(L.C.byref(a), ws.data_ptr(), nbytes, stream.cuda_stream), "ttt_wpred_run")
            nch = (S + chunk - 1) // chunk
            return dict(out=out, coeffs=c, m=m, v=v, step=step + nch, final=fin)
    for t0 in range(0, S, chunk):
        Lc = min(chunk, S - t0)
        xc = x[:, t0:t0 + Lc]
        lt = None
        if gate_weight is not None:
            lt = gate_decay(xc, gate_weight, gate_bias, lam, gate_scale=gate_scale, gate_range=gate_range)
        s, fin = cheby_ema_forward(xc, c, lambda_per_head=lam, lam_tok=lt, init_state=state,
                                   out_dtype=torch.float32, out=out[:, t0:t0 + Lc])
        gs = None
        if Lc > 1:
            # one elementwise launch subtracts the bf16 next tokens in fp32 (no
            # separate conversion); the 2/N scale rides in the second GEMM's alpha
            with _matmul_precision(gemm):
                r = torch.matmul(s[:, :-1], Wp.t())
                r.sub_(xc[:, 1:])
                r2 = r.view(-1, D)
                gs = torch.addmm(r2, r2, Wp, beta=0.0, alpha=2.0 / ((Lc - 1) * D)).view(B, Lc - 1, D)
        step += 1
        a = L.TttArgs(B=B, L=Lc, H=H, head_dim=hd, degree=K, x=xc.data_ptr(), x_dtype=_DT[xdt],
                      x_stride_b=xc.stride(0), x_stride_s=xc.stride(1), coeffs=c.data_ptr(), m=m.data_ptr(),
                      v=v.data_ptr(), lam_h=lam.data_ptr(), momentum=float(ema_momentum), lam_tok=_ptr(lt),
                      gs=_ptr(gs), lr=float(lr), beta1=float(betas[0]), beta2=float(betas[1]), eps=float(eps),
                      spectral_pow=float(spectral_pow), step=int(step), forget=int(bool(forget)))
        nbytes = lib.ossm_ttt_workspace_bytes(L.C.byref(a))
        if nbytes == 0:
            L.check(L.OSSM_EINVAL, "ttt_wpred_adam (argument check)")
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        L.check(lib.ossm_ttt_wpred_step(L.C.byref(a), ws.data_ptr(), nbytes, stream.cuda_stream), "ttt_wpred_step")
        state = fin
    return dict(out=out, coeffs=c, m=m, v=v, step=step, final=state)


def gate_decay(x, gate_weight, gate_bias, lambda_per_head, *, gate_scale=0.008,
               gate_range=(0.0, 1.0), out=None):
    """Per-token decay of the dynamic-lambda gate, [B,S,H] float32:
    ``clamp(lambda_h + gate_scale*(sigmoid(W x_t + b)[h] - 0.5), *gate_range)``."""
    _need_cuda(x)
    x = _rowmajor(x)
    if x.dtype not in _DT:
        x = x.float()
    B, S, D = x.shape
    dev = x.device
    W = gate_weight.to(dev, torch.float32).contiguous()
    bvec = gate_bias.to(dev, torch.float32).contiguous()
    H = W.shape[0]
    lam = torch.as_tensor(lambda_per_head, dtype=torch.float32, device=dev).contiguous()
    if out is None:
        out = torch.empty(B, S, H, device=dev, dtype=torch.float32)
    a = L.FwdArgs(B=B, S=S, H=H, head_dim=D // H, degree=1, x=x.data_ptr(), x_dtype=_DT[x.dtype],
                  x_stride_b=x.stride(0), x_stride_s=x.stride(1), coeffs=lam.data_ptr(),
                  lam_h=lam.data_ptr(), gate_w=W.data_ptr(), gate_b=bvec.data_ptr(),
                  gate_scale=float(gate_scale), gate_lo=float(gate_range[0]),
                  gate_hi=float(gate_range[1]), out=x.data_ptr(), out_dtype=_DT[x.dtype],
                  out_stride_b=x.stride(0), out_stride_s=x.stride(1))
    stream = torch.cuda.current_stream(dev)
    L.check(L.lib().ossm_gate_decay(L.C.byref(a), out.data_ptr(), stream.cuda_stream), "gate_decay")
    return out


# ----------------------------------------------------------------------------
# reference op: apply_cheby_rkv_v10
# ----------------------------------------------------------------------------

def _per_batch(v, B, dev):
    if v is None:
        return None
    t = torch.as_tensor(v, device=dev).float().reshape(-1)
    if t.numel() < B:
        t = t.expand(B) if t.numel() == 1 else t
    return t[:B].contiguous()


def _lion_full_path(x, coeffs, momentum_buf, n_heads, base_lr, ema_momentum, lion_beta1,
                    lion_beta2, lion_wd, chunk_size, gate_global, dynamic_lambda, use_lut,
                    out_dtype=torch.float32, final_state=None, trace=None):
    """All chunks of the reference's full path in one launch.  Returns
    (out [B,S,D] bf16-rounded values, new coeffs, new momentum); ``trace``
    ([n_chunks,B,H,K,hd] f32) receives the coefficients each chunk starts from."""
    _need_cuda(x, coeffs)
    x = _rowmajor(x)
    if x.dtype not in _DT:
        x = x.float()
    B, S, D = x.shape
    hd = D // n_heads
    if hd * n_heads != D:
        raise ValueError("D must be divisible by n_heads")
    dev = x.device
    c = coeffs.float().contiguous().clone()
    m = momentum_buf.float().contiguous().clone() if momentum_buf is not None else torch.zeros_like(c)
    K = c.shape[2]
    if tuple(c.shape) != (B, n_heads, K, hd):
        raise ValueError(f"coeffs {tuple(c.shape)} vs expected {(B, n_heads, K, hd)}")
    out = torch.empty(B, S, D, device=dev, dtype=out_dtype)
    lut = get_chebyshev_lut(dev) if use_lut else None
    gg = _per_batch(gate_global, B, dev)
    dl = _per_batch(dynamic_lambda, B, dev)
    a = L.LionArgs(B=B, S=S, H=n_heads, head_dim=hd, degree=K, chunk=int(chunk_size),
                   x=x.data_ptr(), x_dtype=_DT[x.dtype], x_stride_b=x.stride(0), x_stride_s=x.stride(1),
                   coeffs=c.data_ptr(), momentum=m.data_ptr(), gate_global=_ptr(gg),
                   dynamic_lambda=_ptr(dl), ema_momentum=float(ema_momentum), base_lr=float(base_lr),
                   beta1=float(lion_beta1), beta2=float(lion_beta2), weight_decay=float(lion_wd),
                   lut=_ptr(lut), out=out.data_ptr(), out_dtype=_DT[out_dtype],
                   out_stride_b=out.stride(0), out_stride_s=out.stride(1), tanh_out=None,
                   final_state=_ptr(final_state),
                   flags=L.OSSM_EVAL_LUT if use_lut else L.OSSM_EVAL_CLENSHAW_DEG4, coeff_trace=_ptr(trace))
    stream = torch.cuda.current_stream(dev)
    L.check(L.lib().ossm_cheby_rkv_lion(L.C.byref(a), stream.cuda_stream), "cheby_rkv_lion")
    return out, c, m


class _RkvFullFn(torch.autograd.Function):
    """The reference's full path (Lion TTT chunk by chunk) as one autograd node.

    Gradients follow the reference's chunk loop (sdpc_kernel.py:2574-2606 with
    FusedChebyRKVv10.backward, :2435-2515): each chunk's EMA restarts from zero,
    so the adjoint is cut at every chunk start; each chunk is differentiated
    against the coefficients it started from; the coefficients passed between
    chunks are detached, so the input coefficients receive a gradient only when
    the sequence is a single chunk."""

    @staticmethod
    def forward(ctx, x, coeffs, momentum_buf, opts):
        B, S, _ = x.shape
        chunk = int(opts["chunk_size"])
        n_chunks = (S + chunk - 1) // chunk
        trace = torch.empty((n_chunks,) + tuple(coeffs.shape), device=x.device, dtype=torch.float32)
        out, c, m = _lion_full_path(x.detach(), coeffs.detach(), None if momentum_buf is None else momentum_buf.detach(),
                                    opts["n_heads"], opts["base_lr"], opts["ema_momentum"], opts["lion_beta1"],
                                    opts["lion_beta2"], opts["lion_wd"], chunk, opts["gate_global"],
                                    opts["dynamic_lambda"], opts["use_lut"], trace=trace)
        ctx.save_for_backward(x, coeffs, trace)
        ctx.mu = float(opts["ema_momentum"])
        ctx.chunk = chunk
        ctx.mark_non_differentiable(c, m)
        return out, c, m

    @staticmethod
    def backward(ctx, g_out, g_c, g_m):
        x, coeffs, trace = ctx.saved_tensors
        if g_out is None:
            return None, None, None, None
        single = trace.shape[0] == 1
        gx, gc, _ = _rev_backward(x, g_out, trace[0], momentum=ctx.mu,
                                  segment=0 if single else ctx.chunk, segment_coeffs=None if single else trace)
        return gx.to(x.dtype), (gc.to(coeffs.dtype) if single else None), None, None


class FusedChebyRKVv10(torch.autograd.Function):
    """One full-path call over the whole sequence as a single chunk
    (reference: sdpc_kernel.py:2351-2515).  Same 16 positional arguments;
    backward as the reference's: gradients for x and coeffs."""

    @staticmethod
    def forward(ctx, x, coeffs, momentum_buf, n_heads=4, base_lr=0.005, ema_momentum=0.9,
                lion_beta1=0.9, lion_beta2=0.99, lion_wd=0.01, chunk_size=256, use_bf16=False,
                gate_global=None, dynamic_lambda=None, use_lut=True, seq_threshold=384,
                lion_max_norm=14.0):
        S = x.shape[1]
        trace = torch.empty((1,) + tuple(coeffs.shape), device=x.device, dtype=torch.float32)
        out, c, m = _lion_full_path(x, coeffs, momentum_buf, n_heads, base_lr, ema_momentum,
                                    lion_beta1, lion_beta2, lion_wd, S, gate_global,
                                    dynamic_lambda, use_lut, trace=trace)
        ctx.save_for_backward(x, coeffs)
        ctx.mu = float(ema_momentum)
        ctx.mark_non_differentiable(c, m)
        return out, c, m

    @staticmethod
    def backward(ctx, grad_out, grad_c, grad_m):
        x, coeffs = ctx.saved_tensors
        gx, gc, _ = _rev_backward(x, grad_out, coeffs, momentum=ctx.mu)
        return (gx.to(x.dtype), gc.to(coeffs.dtype)) + (None,) * 14


def apply_cheby_rkv_v10(x, coeffs, momentum_buf, n_heads=4, base_lr=0.005, ema_momentum=0.9,
                        lion_beta1=0.9, lion_beta2=0.99, lion_wd=0.01, chunk_size=256,
                        use_bf16=False, gate_global=None, dynamic_lambda=None, use_lut=True,
                        seq_threshold=384, lion_max_norm=14.0):
    """OrthoSSM V10 core op (reference: sdpc_kernel.py:2522-2606).

    Returns (output float32 [B,S,D], new_coeffs, new_momentum).  Below
    ``seq_threshold`` tokens: fast path (no TTT, coefficients returned
    unchanged).  Otherwise the reference's chunked Lion TTT over
    ``chunk_size``-token chunks, all chunks in one device launch.
    ``use_bf16`` and ``lion_max_norm`` are accepted and, as in the reference's
    live path, unused."""
    B, S, D = x.shape
    if coeffs.dtype != torch.float32:
        coeffs = coeffs.float()
    if momentum_buf is not None and momentum_buf.dtype != torch.float32:
        momentum_buf = momentum_buf.float()
    if seq_threshold > 0 and S < seq_threshold:
        xf = x if x.dtype in _DT else x.float()
        out, _ = cheby_ema_forward(xf, coeffs, ema_momentum=ema_momentum, fast_path_semantics=True,
                                   out_dtype=torch.float32 if x.dtype != torch.bfloat16 else x.dtype)
        return out, coeffs, momentum_buf
    if torch.is_grad_enabled() and (x.requires_grad or coeffs.requires_grad):
        opts = dict(n_heads=n_heads, base_lr=base_lr, ema_momentum=ema_momentum, lion_beta1=lion_beta1,
                    lion_beta2=lion_beta2, lion_wd=lion_wd, chunk_size=min(int(chunk_size), S),
                    gate_global=gate_global, dynamic_lambda=dynamic_lambda, use_lut=use_lut)
        return _RkvFullFn.apply(x, coeffs, momentum_buf, opts)
    return _lion_full_path(x, coeffs, momentum_buf, n_heads, base_lr, ema_momentum, lion_beta1,
                           lion_beta2, lion_wd, chunk_size, gate_global, dynamic_lambda, use_lut)


apply_cheby_rkv_core = apply_cheby_rkv_v10
