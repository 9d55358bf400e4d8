"""Config-5 language model: an SDPC-engine LM whose
every layer runs the Cheby-RKV global path on this package's fused kernel.

Layer layout, V8 (README.md:40-80 "SDPC Engine V8"
"the Cheby-RKV path plus NSA local SDPA (window 512) and a LayerNorm+Linear
combine"):

    h      = RMSNorm(x)
    global = cheby_ema_forward(h)          per-head lambda, per-token gate
                                           Linear(d -> H) on h, EMA state carried
    local  = causal attention of each token over the last `window` tokens
             (q, k, v, o projections, H heads of d/H)
    x      = x + Linear(LayerNorm(global + local))

The model around the layers follows model.py:23-187: token embedding, the
layer stack, a final RMSNorm and an LM head tied to the embedding
(model.py's default ``tie_weights=True``), fresh Chebyshev states per layer
from ``init_chebyshev_coefficients`` (model.py ``fresh_states``).

Left out, with the modules the reference does not ship (``nsa_module.py``,
``landmark_archive.py``): NSA's landmark and archive cross-attention, the
landmark archive, state refresh, recall residual and the cross-layer bus.
The spec's "~72M params" counts the reference engine with those parts; this
layout has 24.3M parameters at the spec's sizes (16.4M of them the tied
embedding).

The global path runs in the sm_100a kernels of this package (bf16 in and out,
fp32 state); the projections are cuBLAS bf16 GEMMs and the local attention is
flash-attention's sliding-window kernel (library kernels, the spec's
"SDPA").  ``local_window_attention_blocked`` restates that attention with
torch's scaled_dot_product_attention over 2*window-key blocks; the tests check
the two against each other and against dense masked attention.
"""
from __future__ import annotations

import dataclasses
import math
from typing import List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .sdpc_kernel import BASELINE_LAMBDA, cheby_ema_forward, init_chebyshev_coefficients
from .state import ChebyStreamState


@dataclasses.dataclass
class OrthoLMConfig:
    vocab_size: int = 32000
    d_model: int = 512
    n_heads: int = 8          # Chebyshev heads and attention heads
    n_layers: int = 6
    window: int = 512         # local attention: each token sees the last `window` tokens
    degree: int = 8
    lambda_per_head: tuple = tuple(BASELINE_LAMBDA)
    gate_scale: float = 0.008

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads


def local_window_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window: int) -> torch.Tensor:
    """Causal attention of query t over keys t-window+1 .. t (flash-attention's
    sliding window; CUDA tensors, bf16 or fp16).  q, k, v: [B, S, H, hd]."""
    from flash_attn import flash_attn_func
    return flash_attn_func(q, k, v, causal=True, window_size=(window - 1, 0))


def local_window_attention_blocked(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window: int) -> torch.Tensor:
    """The same attention with torch's SDPA (any device and dtype).

    q, k, v: [B, S, H, hd].  The sequence is cut into blocks of `window`
    queries; each block attends to its own keys and the previous block's
    (2*window keys) under a band mask, in one batched SDPA call.  Returns
    [B, S, H, hd]."""
    B, S, H, hd = q.shape
    W = window
    nb = (S + W - 1) // W
    pad = nb * W - S
    if pad:
        q, k, v = (F.pad(t, (0, 0, 0, 0, 0, pad)) for t in (q, k, v))
    qb = q.view(B, nb, W, H, hd)
    kb = k.view(B, nb, W, H, hd)
    vb = v.view(B, nb, W, H, hd)
    zero = torch.zeros_like(kb[:, :1])
    k2 = torch.cat([torch.cat([zero, kb[:, :-1]], 1), kb], 2)  # [B, nb, 2W, H, hd]: previous block, own block
    v2 = torch.cat([torch.cat([zero, vb[:, :-1]], 1), vb], 2)
    i = torch.arange(W, device=q.device).view(W, 1)
    j = torch.arange(2 * W, device=q.device).view(1, 2 * W)
    band = (j - W <= i) & (j - W > i - W)  # key position (j - W) in (i - W, i] relative to the block start
    mask = band.expand(nb, W, 2 * W).clone()
    mask[0, :, :W] = False  # block 0 has no previous block
    o = F.scaled_dot_product_attention(
        qb.permute(0, 1, 3, 2, 4).reshape(B * nb, H, W, hd),
        k2.permute(0, 1, 3, 2, 4).reshape(B * nb, H, 2 * W, hd),
        v2.permute(0, 1, 3, 2, 4).reshape(B * nb, H, 2 * W, hd),
        attn_mask=mask.unsqueeze(1).repeat(B, 1, 1, 1).view(B * nb, 1, W, 2 * W))
    o = o.view(B, nb, H, W, hd).permute(0, 1, 3, 2, 4).reshape(B, nb * W, H, hd)
    return o[:, :S]


class V8Layer(nn.Module):
    def __init__(self, cfg: OrthoLMConfig):
        super().__init__()
        d, H = cfg.d_model, cfg.n_heads
        self.cfg = cfg
        self.norm_in = nn.RMSNorm(d)
        self.gate = nn.Linear(d, H)  # per-token decay gate of the global path
        self.qkv = nn.Linear(d, 3 * d, bias=False)
        self.o = nn.Linear(d, d, bias=False)
        self.norm_comb = nn.LayerNorm(d)
        self.out_proj = nn.Linear(d, d, bias=False)
        # The decays stay fp32 whatever dtype the module is cast to (0.9995
        # rounds to 1.0 in bf16), so they are kept outside the buffers.
        self._lam = {}

    def lam(self, device) -> torch.Tensor:
        t = self._lam.get(device)
        if t is None:
            t = self._lam[device] = torch.tensor(self.cfg.lambda_per_head, dtype=torch.float32, device=device)
        return t

    def forward(self, x: torch.Tensor, coeffs: torch.Tensor, ema: Optional[torch.Tensor]):
        B, S, d = x.shape
        H = self.cfg.n_heads
        h = self.norm_in(x)
        g, fin = cheby_ema_forward(h, coeffs, lambda_per_head=self.lam(h.device), gate_weight=self.gate.weight.float(),
                                   gate_bias=self.gate.bias.float(), gate_scale=self.cfg.gate_scale,
                                   init_state=ema, out_dtype=h.dtype)
        q, k, v = self.qkv(h).view(B, S, 3, H, d // H).unbind(2)
        attn = local_window_attention if h.dtype in (torch.bfloat16, torch.float16) else local_window_attention_blocked
        loc = self.o(attn(q, k, v, self.cfg.window).reshape(B, S, d))
        return x + self.out_proj(self.norm_comb(g + loc)), fin


class OrthoSSMLM(nn.Module):
    """Token ids [B, S] -> logits [B, S, vocab] (activations and weights in the
    parameters' dtype, bf16 for config 5)."""

    def __init__(self, cfg: OrthoLMConfig = OrthoLMConfig()):
        super().__init__()
        self.cfg = cfg
        self.embedding = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.layers = nn.ModuleList([V8Layer(cfg) for _ in range(cfg.n_layers)])
        self.final_norm = nn.RMSNorm(cfg.d_model)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        self.lm_head.weight = self.embedding.weight
        self._init_weights()

    def _init_weights(self, std: float = 0.02):
        """N(0, 0.02) weights, out_proj scaled by 1/sqrt(2 n_layers), zero
        biases (model.py _init_weights)."""
        scale = 1.0 / math.sqrt(2 * self.cfg.n_layers)
        for name, p in self.named_parameters():
            if p.dim() >= 2:
                nn.init.normal_(p, 0.0, std * (scale if "out_proj" in name else 1.0))
            elif "bias" in name:
                nn.init.zeros_(p)

    def fresh_states(self, batch: int, device, generator_seed: Optional[int] = None) -> List[ChebyStreamState]:
        """Fresh Chebyshev coefficients per layer (model.py fresh_states) and
        no EMA state."""
        cfg = self.cfg
        if generator_seed is not None:
            torch.manual_seed(generator_seed)
        return [ChebyStreamState(coeffs=init_chebyshev_coefficients(batch, cfg.n_heads, cfg.degree, cfg.head_dim,
                                                                    device))
                for _ in range(cfg.n_layers)]

    def forward(self, input_ids: torch.Tensor, states: Optional[List[ChebyStreamState]] = None,
                return_state: bool = False):
        B, S = input_ids.shape
        if states is None:
            states = self.fresh_states(B, input_ids.device)
        x = self.embedding(input_ids)
        new_states = []
        for layer, st in zip(self.layers, states):
            x, fin = layer(x, st.coeffs, st.ema)
            new_states.append(dataclasses.replace(st, ema=fin, tokens_seen=st.tokens_seen + S))
        logits = self.lm_head(self.final_norm(x))
        return (logits, new_states) if return_state else logits


def n_params(model: nn.Module) -> int:
    return sum(p.numel() for p in {id(p): p for p in model.parameters()}.values())
