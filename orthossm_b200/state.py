"""Streaming state of the Cheby-RKV path and its on-disk format.

The reference carries a layer's recurrent state between calls as the tuple
``(coeffs, momentum)`` ([B, H, K, hd] fp32 each): ``apply_cheby_rkv_v10``
returns it (sdpc_kernel.py:2522-2606, detached between chunks at :2589-2592),
the engine hands it back as ``cheby_state`` on the next call
(sdpc_engine.py:175-191, :262) and accepts the older 3-tuple
``(coeffs, m1, m2)`` by dropping ``m2`` (:183-185).  The EMA state is reset
on every call there (sdpc_kernel.py:2398).  BASELINE semantics also carry
the EMA state [B, D] across calls, and the Adam TTT (BASELINE.json
configs[3]) carries a second moment and a step count.

``ChebyStreamState`` holds all of it and serialises it to a small
self-describing binary format, so a long stream can be checkpointed and
resumed on another process or device:

    magic  b"OSSMST\\x00\\x01"        8 bytes (format version 1)
    n      uint32 little-endian     length of the JSON header
    header JSON                      {"version", "mode", "step", "tokens_seen",
                                      "meta", "tensors": [{name, dtype, shape,
                                      offset, nbytes, crc32}, ...]}
    padding to 16 bytes, then each tensor's raw little-endian bytes at its
    offset (16-byte aligned), in C order.

Loading checks the magic, the version, each tensor's size and CRC32, and the
shapes against each other; any mismatch raises ``ValueError``.

``StreamingChebyRKV`` drives a stream chunk by chunk through either the
reference's op (``apply_cheby_rkv_v10``: Lion TTT, EMA reset per call, fast
path below ``seq_threshold``) or the BASELINE forward (carried EMA state;
optionally the W_pred Adam TTT of ``ttt_wpred_adam``).  All compute runs in
the CUDA kernels behind those functions; this module is host bookkeeping.
"""
from __future__ import annotations

import dataclasses
import io
import json
import struct
import zlib
from typing import Optional

import torch

MAGIC = b"OSSMST\x00\x01"
VERSION = 1
_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}
_NAMES = ("coeffs", "momentum", "adam_v", "ema")


def _dtype_name(t: torch.Tensor) -> str:
    for k, v in _DTYPES.items():
        if t.dtype == v:
            return k
    raise ValueError(f"unsupported state dtype {t.dtype}")


@dataclasses.dataclass
class ChebyStreamState:
    """Recurrent state of one Cheby-RKV layer for a batch of streams.

    coeffs:   [B, H, K, hd] Chebyshev coefficients (fp32).
    momentum: [B, H, K, hd] Lion momentum (reference mode) or Adam first
              moment (BASELINE TTT); None when nothing updates the coefficients.
    adam_v:   [B, H, K, hd] Adam second moment (BASELINE TTT) or None.
    ema:      [B, H*hd] EMA state after the last token (BASELINE mode) or None
              (reference mode resets it every call).
    step:     optimiser steps taken so far (Adam bias correction).
    tokens_seen: tokens consumed per stream so far.
    meta:     free-form JSON-serialisable settings saved alongside.
    """
    coeffs: torch.Tensor
    momentum: Optional[torch.Tensor] = None
    adam_v: Optional[torch.Tensor] = None
    ema: Optional[torch.Tensor] = None
    step: int = 0
    tokens_seen: int = 0
    meta: dict = dataclasses.field(default_factory=dict)

    # ------------------------------------------------------------------ checks
    def validate(self) -> "ChebyStreamState":
        c = self.coeffs
        if c.dim() != 4:
            raise ValueError(f"coeffs must be [B,H,K,hd], got {tuple(c.shape)}")
        for name in ("momentum", "adam_v"):
            t = getattr(self, name)
            if t is not None and tuple(t.shape) != tuple(c.shape):
                raise ValueError(f"{name} {tuple(t.shape)} does not match coeffs {tuple(c.shape)}")
        if self.ema is not None:
            B, H, _, hd = c.shape
            if tuple(self.ema.shape) != (B, H * hd):
                raise ValueError(f"ema {tuple(self.ema.shape)} must be [B, H*hd] = {(B, H * hd)}")
        if self.step < 0 or self.tokens_seen < 0:
            raise ValueError("step and tokens_seen must be >= 0")
        return self

    # ------------------------------------------------------- reference tuple
    @classmethod
    def from_reference(cls, cheby_state, **kw) -> "ChebyStreamState":
        """From the engine's ``cheby_state``: a (coeffs, momentum) or legacy
        (coeffs, m1, m2) tuple, or a bare coefficient tensor (zero momentum,
        degree padded to the tensor's), as sdpc_engine.py:175-191 accepts."""
        if isinstance(cheby_state, (tuple, list)):
            if len(cheby_state) not in (2, 3):
                raise ValueError("cheby_state tuples hold 2 or 3 tensors")
            coeffs, momentum = cheby_state[0], cheby_state[1]
        else:
            coeffs = cheby_state
            if coeffs.dim() == 3:
                coeffs = coeffs.unsqueeze(1)
            momentum = torch.zeros_like(coeffs)
        return cls(coeffs=coeffs.detach().float(), momentum=momentum.detach().float(), **kw).validate()

    def to_reference(self):
        """The engine's ``(coeffs, momentum)`` tuple."""
        mom = self.momentum if self.momentum is not None else torch.zeros_like(self.coeffs)
        return self.coeffs, mom

    # -------------------------------------------------------------- devices
    def to(self, device) -> "ChebyStreamState":
        mv = lambda t: None if t is None else t.to(device)  # noqa: E731
        return dataclasses.replace(self, coeffs=self.coeffs.to(device), momentum=mv(self.momentum),
                                   adam_v=mv(self.adam_v), ema=mv(self.ema), meta=dict(self.meta))

    def clone(self) -> "ChebyStreamState":
        cl = lambda t: None if t is None else t.detach().clone()  # noqa: E731
        return dataclasses.replace(self, coeffs=cl(self.coeffs), momentum=cl(self.momentum),
                                   adam_v=cl(self.adam_v), ema=cl(self.ema), meta=dict(self.meta))

    # ---------------------------------------------------------------- bytes
    def to_bytes(self) -> bytes:
        self.validate()
        entries, blobs, off = [], [], 0
        for name in _NAMES:
            t = getattr(self, name)
            if t is None:
                continue
            raw = t.detach().contiguous().cpu()
            data = raw.view(torch.uint8).numpy().tobytes() if raw.numel() else b""
            entries.append(dict(name=name, dtype=_dtype_name(raw), shape=list(raw.shape), offset=off,
                                nbytes=len(data), crc32=zlib.crc32(data) & 0xFFFFFFFF))
            blobs.append(data)
            off += (len(data) + 15) & ~15
        header = json.dumps(dict(version=VERSION, step=int(self.step), tokens_seen=int(self.tokens_seen),
                                 meta=self.meta, tensors=entries), sort_keys=True).encode()
        out = io.BytesIO()
        out.write(MAGIC)
        out.write(struct.pack("<I", len(header)))
        out.write(header)
        out.write(b"\x00" * ((-out.tell()) % 16))
        base = out.tell()
        for e, data in zip(entries, blobs):
            out.write(b"\x00" * (base + e["offset"] - out.tell()))
            out.write(data)
        return out.getvalue()

    @classmethod
    def from_bytes(cls, data: bytes, device=None) -> "ChebyStreamState":
        if len(data) < 12 or data[:6] != MAGIC[:6]:
            raise ValueError("not an orthossm_b200 stream state (bad magic)")
        if data[:8] != MAGIC:
            raise ValueError(f"unsupported stream-state format version {data[6]}.{data[7]}")
        (n,) = struct.unpack("<I", data[8:12])
        if 12 + n > len(data):
            raise ValueError("truncated stream-state header")
        hdr = json.loads(data[12:12 + n].decode())
        if hdr.get("version") != VERSION:
            raise ValueError(f"unsupported stream-state version {hdr.get('version')}")
        base = (12 + n + 15) & ~15
        fields = {}
        for e in hdr["tensors"]:
            if e["name"] not in _NAMES or e["dtype"] not in _DTYPES:
                raise ValueError(f"unknown tensor entry {e['name']} / {e['dtype']}")
            lo, hi = base + e["offset"], base + e["offset"] + e["nbytes"]
            if hi > len(data):
                raise ValueError(f"truncated stream state: {e['name']}")
            blob = data[lo:hi]
            if zlib.crc32(blob) & 0xFFFFFFFF != e["crc32"]:
                raise ValueError(f"checksum mismatch in {e['name']}")
            dt = _DTYPES[e["dtype"]]
            n_el = 1
            for d in e["shape"]:
                n_el *= d
            if n_el * torch.empty(0, dtype=dt).element_size() != e["nbytes"]:
                raise ValueError(f"size mismatch in {e['name']}")
            t = torch.frombuffer(bytearray(blob), dtype=dt).reshape(e["shape"]) if n_el else \
                torch.empty(e["shape"], dtype=dt)
            fields[e["name"]] = t.to(device) if device is not None else t
        if "coeffs" not in fields:
            raise ValueError("stream state without coefficients")
        return cls(step=int(hdr["step"]), tokens_seen=int(hdr["tokens_seen"]), meta=hdr.get("meta", {}),
                   **fields).validate()

    def save(self, path) -> None:
        with open(path, "wb") as f:
            f.write(self.to_bytes())

    @classmethod
    def load(cls, path, device=None) -> "ChebyStreamState":
        with open(path, "rb") as f:
            return cls.from_bytes(f.read(), device=device)


class StreamingChebyRKV:
    """Feeds one layer's Cheby-RKV path a stream of chunks, carrying its state.

    mode "reference": each call is ``apply_cheby_rkv_v10`` on the chunk with
    the carried (coeffs, momentum), as the engine does call after call; the
    EMA restarts at every call (reference semantics).  Extra keyword arguments
    go to ``apply_cheby_rkv_v10``.

    mode "baseline": the BASELINE forward with the EMA state carried from
    chunk to chunk (so the outputs equal one call over the whole stream), with
    per-head decays ``lambda_per_head`` and the optional per-token gate.  With
    ``W_pred`` set, the coefficients also take the W_pred Adam TTT step of
    ``ttt_wpred_adam`` over ``ttt_chunk``-token chunks.

    ``state`` can be saved at any chunk boundary (``state.save``) and a new
    ``StreamingChebyRKV`` built from the loaded state continues the stream
    exactly where the old one stopped."""

    def __init__(self, state: ChebyStreamState, *, mode: str = "baseline", lambda_per_head=None,
                 ema_momentum: float = 0.9, gate_weight=None, gate_bias=None, W_pred=None,
                 ttt_chunk: int = 2048, out_dtype=None, **ref_kwargs):
        if mode not in ("baseline", "reference"):
            raise ValueError(f"mode must be 'baseline' or 'reference', got {mode!r}")
        self.state = state.validate()
        self.mode = mode
        self.lambda_per_head = lambda_per_head
        self.ema_momentum = ema_momentum
        self.gate_weight, self.gate_bias = gate_weight, gate_bias
        self.W_pred = W_pred
        self.ttt_chunk = int(ttt_chunk)
        self.out_dtype = out_dtype
        self.ref_kwargs = ref_kwargs
        if mode == "reference" and state.momentum is None:
            self.state.momentum = torch.zeros_like(state.coeffs)
        if mode == "baseline" and W_pred is not None:
            if self.state.momentum is None:
                self.state.momentum = torch.zeros_like(state.coeffs)
            if self.state.adam_v is None:
                self.state.adam_v = torch.zeros_like(state.coeffs)

    @torch.no_grad()
    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        from . import sdpc_kernel as K
        st = self.state
        B, S, D = x.shape
        if self.mode == "reference":
            out, st.coeffs, st.momentum = K.apply_cheby_rkv_v10(
                x, st.coeffs, st.momentum, n_heads=st.coeffs.shape[1], ema_momentum=self.ema_momentum,
                **self.ref_kwargs)
            st.step += 1
        elif self.W_pred is not None:
            r = K.ttt_wpred_adam(x, st.coeffs, st.momentum, st.adam_v, st.step, self.W_pred,
                                 lambda_per_head=self.lambda_per_head, ema_momentum=self.ema_momentum,
                                 gate_weight=self.gate_weight, gate_bias=self.gate_bias, init_state=st.ema,
                                 chunk=self.ttt_chunk)
            out = r["out"] if self.out_dtype is None else r["out"].to(self.out_dtype)
            st.coeffs, st.momentum, st.adam_v, st.step, st.ema = r["coeffs"], r["m"], r["v"], r["step"], r["final"]
        else:
            out, st.ema = K.cheby_ema_forward(x, st.coeffs, lambda_per_head=self.lambda_per_head,
                                              ema_momentum=self.ema_momentum, gate_weight=self.gate_weight,
                                              gate_bias=self.gate_bias, init_state=st.ema,
                                              out_dtype=self.out_dtype)
        st.tokens_seen += S
        return out
