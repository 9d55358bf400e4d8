"""SDPC engine layer (sdpc_engine.py:55-467) with the Cheby-RKV path on this
package's kernels: a drop-in for ``SpectralDualPathContextEngine`` and
``build_ortho_stack``, parameter for parameter (a reference ``state_dict``
loads unchanged).

What each part follows:

* ``SpectralDualPathContextEngine``: the constructor and the three length
  routes of sdpc_engine.py:63-429 (fast below 384 tokens, hybrid below 1024,
  full otherwise).  The Chebyshev path is ``apply_cheby_rkv_v10`` of this
  package.  Unlike the reference, a forward makes no host synchronisation.
  The reference reads the EMA-momentum schedule (:209) and a batch of control
  values (:336) back to the host every call.  Here the token counter and the
  archive size are mirrored on the host (they change by host-known amounts),
  and the recall residual's decision (:389-412) is applied with device-side
  masks instead of branches.  The outputs are the same.
* ``SpectralLocalRefiner``: slr_module.py:363-669: routing by the
  Chebyshev path's autoregressive error, top-k token selection, RoPE at the
  original positions, differential attention with a per-head sigmoid(lambda).
  The attention follows the reference's CUDA route (its fused kernel,
  slr_module.py:83-243).  Every selected query sees every selected key at or
  before its position and within ``window_size`` positions.  It runs as masked
  scaled-dot-product attention over query blocks.
* ``LandmarkArchive`` and ``AsyncLightBus``: the reference does not ship
  ``landmark_archive.py`` (imported at sdpc_engine.py:44); only its interface
  is known from the call sites (sdpc_engine.py:114-117, 354-363, 376-381,
  431-447; model.py:141, 163; test_v10.py:248-260).  The versions here are
  this package's own design, stated in their docstrings.

The diagnostics hooks of the reference (``DIAG``, ortho_diagnostics.py) do not
change any output and are left out.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .sdpc_kernel import GatedComplexityPredictor, apply_cheby_rkv_v10

FAST_PATH_THRESHOLD = 384     # sdpc_engine.py:53
HYBRID_PATH_THRESHOLD = 1024  # sdpc_engine.py:54


# ----------------------------------------------------------------------------
# archive and bus (interfaces of the missing landmark_archive.py; own design)
# ----------------------------------------------------------------------------

class AsyncLightBus:
    """Cross-layer summary bus (sdpc_engine.py:360-381, test_v10.py:248-260).

    ``publish(layer, summary [B, dim])`` stores a layer's summary (detached:
    the bus is an asynchronous residual, no gradient crosses layers);
    ``gather(layer, B, device)`` returns the mean of the summaries published by
    lower layers, or None when there are none; ``clear`` empties it (once per
    model forward, model.py:141); ``snapshot`` returns a copy of what is
    held."""

    def __init__(self, summary_dim: int = 64, n_layers: int = 2):
        self.summary_dim = summary_dim
        self.n_layers = n_layers
        self._slots: dict = {}

    def publish(self, layer_idx: int, summary: torch.Tensor) -> None:
        self._slots[int(layer_idx)] = summary.detach()

    def gather(self, layer_idx: int, batch: int, device) -> Optional[torch.Tensor]:
        lower = [v for k, v in sorted(self._slots.items()) if k < layer_idx and v.shape[0] == batch]
        if not lower:
            return None
        return torch.stack(lower, 0).mean(0).to(device)

    def clear(self) -> None:
        self._slots.clear()

    def snapshot(self) -> dict:
        return dict(self._slots)


class LandmarkArchive(nn.Module):
    """Archive of Chebyshev-coefficient snapshots (landmarks).

    Every ``archive_interval`` tokens the batch mean of the coefficients is
    archived.  Once ``max_landmarks`` are held, the new snapshot is merged into
    the most similar one (cosine), as ``0.9 old + 0.1 new`` (the reference
    describes an importance-based archive with exponential merge of similar
    entries, README.md "Landmark Archive + Recall Residual").
    ``state_to_embedding`` maps a flattened snapshot to a d_model embedding;
    ``get_landmark_embeddings(B, device)`` returns ([B, n, d_model] or None,
    n).  The number held is mirrored on the host (``n_host``), so callers
    need no device read."""

    def __init__(self, d_model, n_heads, head_dim, degree, max_landmarks=64, archive_interval=131072):
        super().__init__()
        self.max_landmarks = int(max_landmarks)
        self.archive_interval = int(archive_interval)
        flat = n_heads * degree * head_dim
        self.state_to_embedding = nn.Linear(flat, d_model)
        self.register_buffer("archived_states", torch.zeros(self.max_landmarks, n_heads, degree, head_dim))
        self.register_buffer("n_archived", torch.tensor(0, dtype=torch.long))
        self.register_buffer("tokens_since", torch.tensor(0, dtype=torch.long))
        self._host = None  # (n_archived, tokens_since) mirrored on the host

    def _sync_host(self):
        if self._host is None:  # once, after construction or a state_dict load
            self._host = [int(self.n_archived.item()), int(self.tokens_since.item())]
        return self._host

    def _load_from_state_dict(self, *args, **kwargs):
        super()._load_from_state_dict(*args, **kwargs)
        self._host = None

    @property
    def n_host(self) -> int:
        return self._sync_host()[0]

    @torch.no_grad()
    def maybe_archive(self, coeffs: torch.Tensor, seq_len: int, complexity_score=None) -> None:
        h = self._sync_host()
        h[1] += int(seq_len)
        self.tokens_since.fill_(h[1])
        if h[1] < self.archive_interval:
            return
        h[1] = 0
        self.tokens_since.zero_()
        snap = coeffs.detach().float().mean(0)
        n = h[0]
        if n < self.max_landmarks:
            self.archived_states[n].copy_(snap)
            h[0] = n + 1
            self.n_archived.fill_(n + 1)
        else:
            sim = F.cosine_similarity(self.archived_states.flatten(1), snap.flatten().unsqueeze(0), dim=1)
            j = sim.argmax()
            self.archived_states[j] = 0.9 * self.archived_states[j] + 0.1 * snap

    def get_landmark_embeddings(self, batch: int, device):
        n = self.n_host
        if n == 0:
            return None, 0
        emb = self.state_to_embedding(self.archived_states[:n].flatten(1).to(device))
        return emb.unsqueeze(0).expand(batch, -1, -1), n


# ----------------------------------------------------------------------------
# Spectral Local Refiner
# ----------------------------------------------------------------------------

def rope_tables(positions: torch.Tensor, head_dim: int):
    """cos / sin [B, 1, L, head_dim/2] of RoPE (base 10000) at integer positions
    [B, L] (slr_module.py:332-344)."""
    inv = 1.0 / (10000.0 ** (torch.arange(0, head_dim, 2, device=positions.device, dtype=torch.float32) / head_dim))
    ang = positions.float().unsqueeze(-1) * inv.view(1, 1, -1)
    return ang.cos().unsqueeze(1), ang.sin().unsqueeze(1)


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs (x[2i], x[2i+1]) of x [B, H, L, hd]
    (slr_module.py:347-356)."""
    a, b = x[..., 0::2], x[..., 1::2]
    return torch.stack((a * cos - b * sin, a * sin + b * cos), dim=-1).flatten(-2)


class SpectralLocalRefiner(nn.Module):
    """Spectral-routed differential local attention (slr_module.py:363-669);
    same constructor and parameters as the reference."""

    def __init__(self, d_model, n_heads, window_size=512, select_ratio=0.125, min_select=16, max_select=4096,
                 attn_chunk_size=256):
        super().__init__()
        if d_model % n_heads or (d_model // n_heads) % 2:
            raise ValueError("d_model must split into n_heads heads of even size")
        self.d_model, self.n_heads, self.head_dim = d_model, n_heads, d_model // n_heads
        self.window_size = window_size
        self.select_ratio, self.min_select, self.max_select = select_ratio, min_select, max_select
        self.attn_chunk_size = attn_chunk_size
        self.q1q2kv = nn.Linear(d_model, 4 * d_model, bias=False)
        self.o_proj = nn.Linear(d_model, d_model, bias=False)
        self.diff_lambda_logit = nn.Parameter(torch.zeros(n_heads))
        self.post_norm = nn.RMSNorm(d_model)

    @staticmethod
    @torch.no_grad()
    def compute_routing_scores(x_normed: torch.Tensor, cheby_out: torch.Tensor) -> torch.Tensor:
        """Per-token score [B, S]: mean |xn[t+1] - s[t]| over channels (torch
        softsign, x.sign()), the last token taking the row maximum
        (slr_module.py:424-462)."""
        S = x_normed.shape[1]
        if S < 2:
            return x_normed.abs().mean(-1)
        m = x_normed.abs().clamp(min=1e-7)
        xn = x_normed.sign() * (1.0 - 1.0 / (1.0 + m))
        sc = (xn[:, 1:] - cheby_out[:, :-1]).abs().mean(-1)
        return torch.cat([sc, sc.max(-1, keepdim=True).values], -1)

    def _select_tokens(self, scores: torch.Tensor):
        """The K = clamp(ceil(S * ratio), min_select, min(S, max_select))
        best-scored positions, in increasing order (slr_module.py:464-490)."""
        S = scores.shape[1]
        K = min(max(self.min_select, int(math.ceil(S * self.select_ratio))), S, self.max_select)
        idx = torch.topk(scores, K, dim=-1, sorted=False).indices
        return torch.sort(idx, dim=-1).values, K

    def _window_attention(self, q1, q2, k, v, pos):
        """Softmax attention of each selected query over the selected keys at
        or before its position and less than window_size positions back;
        returns (out1, out2) for the two queries.  Query blocks of
        attn_chunk_size bound the mask's size."""
        B, H, K, hd = q1.shape
        out1, out2 = torch.empty_like(q1), torch.empty_like(q2)
        C = max(int(self.attn_chunk_size), 1)
        pk = pos.unsqueeze(1)  # [B, 1, K]
        for q0 in range(0, K, C):
            q1e = min(q0 + C, K)
            pq = pos[:, q0:q1e].unsqueeze(-1)  # [B, Cq, 1]
            mask = ((pk <= pq) & (pq - pk < self.window_size))[:, None, :, :q1e]  # keys past the block are later
            kk, vv = k[:, :, :q1e], v[:, :, :q1e]
            out1[:, :, q0:q1e] = F.scaled_dot_product_attention(q1[:, :, q0:q1e], kk, vv, attn_mask=mask)
            out2[:, :, q0:q1e] = F.scaled_dot_product_attention(q2[:, :, q0:q1e], kk, vv, attn_mask=mask)
        return out1, out2

    def forward(self, x: torch.Tensor, cheby_out: Optional[torch.Tensor] = None,
                routing_scores: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, S, D = x.shape
        H, hd = self.n_heads, self.head_dim
        routed = S > 2 * self.min_select and cheby_out is not None
        if routed:
            if routing_scores is None:
                routing_scores = self.compute_routing_scores(x, cheby_out)
            idx, K = self._select_tokens(routing_scores)
        else:
            idx, K = torch.arange(S, device=x.device).unsqueeze(0).expand(B, -1), S
        gidx = idx.unsqueeze(-1).expand(B, K, D)
        q1, q2, k, v = (t.reshape(B, K, H, hd).transpose(1, 2)
                        for t in self.q1q2kv(torch.gather(x, 1, gidx)).chunk(4, dim=-1))
        cos, sin = rope_tables(idx, hd)
        q1, q2, k = rope_apply(q1, cos, sin), rope_apply(q2, cos, sin), rope_apply(k, cos, sin)
        if routed:
            o1, o2 = self._window_attention(q1, q2, k, v, idx)
        else:  # every token: plain causal attention (slr_module.py route C)
            o1 = F.scaled_dot_product_attention(q1, k, v, is_causal=True)
            o2 = F.scaled_dot_product_attention(q2, k, v, is_causal=True)
        diff = o1 - torch.sigmoid(self.diff_lambda_logit).view(1, H, 1, 1) * o2
        out = torch.zeros(B, S, D, device=x.device, dtype=x.dtype)
        out.scatter_(1, gidx, diff.transpose(1, 2).reshape(B, K, D).to(x.dtype))
        return self.post_norm(self.o_proj(out))


# ----------------------------------------------------------------------------
# the engine layer
# ----------------------------------------------------------------------------

class SpectralDualPathContextEngine(nn.Module):
    """Length-routed dual-path layer (sdpc_engine.py:56-447): the Chebyshev-RKV
    global path on this package's kernels, the spectral local refiner, the
    landmark archive with state refresh and recall residual, the light bus,
    and the SwiGLU fusion.  Same constructor, parameters and forward as the
    reference; returns ``out`` or ``(out, (coeffs, momentum))``."""

    def __init__(self, d_model, n_attn_heads, n_cheby_heads=8, window_size=512, max_degree=4, chunk_size=256,
                 max_landmarks=64, archive_interval=131072, use_bf16=False, layer_idx=0, light_bus=None,
                 use_lut=True, gradient_ckpt=False):
        super().__init__()
        self.d_model, self.n_cheby_heads = d_model, n_cheby_heads
        self.head_dim = d_model // n_cheby_heads
        self.max_degree, self.chunk_size = max_degree, chunk_size
        self.use_bf16, self.layer_idx, self.light_bus = use_bf16, layer_idx, light_bus
        self.use_lut, self.gradient_ckpt = use_lut, gradient_ckpt
        n_h, hd, deg = n_cheby_heads, self.head_dim, max_degree

        self.complexity_gate = GatedComplexityPredictor(d_model)
        self.coeff_init_proj = nn.Sequential(nn.Linear(d_model, d_model // 4), nn.SiLU(),
                                             nn.Linear(d_model // 4, n_h * deg * hd))
        nn.init.zeros_(self.coeff_init_proj[-1].weight)
        nn.init.zeros_(self.coeff_init_proj[-1].bias)
        self.register_buffer("coeff_spectral_scale",
                             (0.1 / (torch.arange(deg, dtype=torch.float32) + 1.0)).view(1, 1, deg, 1))
        self.slr = SpectralLocalRefiner(d_model, n_attn_heads, window_size)
        self.archive = LandmarkArchive(d_model, n_h, hd, deg, max_landmarks, archive_interval)
        self.refresh_interval = 16384
        self.refresh_proj = nn.Sequential(nn.Linear(d_model, d_model // 2), nn.SiLU(),
                                          nn.Linear(d_model // 2, n_h * hd))
        self.refresh_gate = nn.Sequential(nn.Linear(d_model, n_h * hd), nn.Sigmoid())
        self.recall_proj = nn.Linear(d_model, n_h * deg * hd)
        self.recall_gate = nn.Sequential(nn.Linear(d_model, n_h), nn.Sigmoid())
        self.register_buffer("recall_cooldown", torch.tensor(0, dtype=torch.long))
        if light_bus is not None:
            self.bus_summary_proj = nn.Linear(d_model, 64)
            self.bus_inject_proj = nn.Linear(64, d_model)
        self.input_norm = nn.RMSNorm(d_model)
        self.pre_norm_cheby = nn.RMSNorm(d_model)
        self.pre_norm_slr = nn.RMSNorm(d_model)
        self.fused_gate_value = nn.Linear(2 * d_model, 2 * d_model, bias=False)
        self.out_proj = nn.Linear(d_model, d_model, bias=False)
        self.post_norm = nn.RMSNorm(d_model)
        self.register_buffer("ema_base", torch.tensor(0.9))
        self.register_buffer("total_tokens_seen", torch.tensor(0, dtype=torch.long))
        self._host = None  # (total_tokens_seen, ema_base) mirrored on the host
        self._archive_emb_cache = None  # (n archived, embeddings [n, d_model])

    def _load_from_state_dict(self, *args, **kwargs):
        super()._load_from_state_dict(*args, **kwargs)
        self._host = None

    def _host_counters(self):
        if self._host is None:  # once, after construction or a state_dict load
            self._host = [int(self.total_tokens_seen.item()), float(self.ema_base.item())]
        return self._host

    # ---------------------------------------------------------------- pieces
    def _cheby(self, x_normed, coeffs, momentum, ema_momentum, gate_global, seq_threshold):
        return apply_cheby_rkv_v10(x_normed, coeffs, momentum, n_heads=self.n_cheby_heads, base_lr=0.005,
                                   ema_momentum=ema_momentum, use_bf16=self.use_bf16, gate_global=gate_global,
                                   dynamic_lambda=gate_global, use_lut=self.use_lut, seq_threshold=seq_threshold)

    def _fuse(self, x, cheby_out, slr_out):
        gv = self.fused_gate_value(torch.cat([self.pre_norm_cheby(cheby_out), self.pre_norm_slr(slr_out)], -1))
        gate, value = gv.split(self.d_model, dim=-1)
        return x + self.out_proj(self.post_norm(F.silu(gate) * value))

    @torch.no_grad()
    def _archive_embs(self, n: int) -> torch.Tensor:
        """Embeddings of the n archived landmarks, recomputed only when n
        changes (sdpc_engine.py:431-447: a merge into a full archive keeps the
        old embeddings until n changes).  Kept on the device."""
        if self._archive_emb_cache is None or self._archive_emb_cache[0] != n:
            st = self.archive.archived_states[:n]
            self._archive_emb_cache = (n, self.archive.state_to_embedding(st.flatten(1)).detach())
        return self._archive_emb_cache[1]

    # --------------------------------------------------------------- forward
    def forward(self, x, cheby_state=None, return_state=False):
        B, S, D = x.shape
        n_h, hd, deg = self.n_cheby_heads, self.head_dim, self.max_degree
        x_normed = self.input_norm(x)
        if cheby_state is None:  # input-dependent init (sdpc_engine.py:175-181)
            coeffs = self.coeff_init_proj(x_normed.mean(dim=1)).view(B, n_h, deg, hd) * self.coeff_spectral_scale
            momentum = torch.zeros(B, n_h, deg, hd, device=x.device)
        elif isinstance(cheby_state, (tuple, list)) and len(cheby_state) in (2, 3):
            coeffs, momentum = cheby_state[0], cheby_state[1]
        else:
            coeffs = cheby_state
            if coeffs.dim() == 3:
                coeffs = coeffs.unsqueeze(1)
            if coeffs.shape[2] < deg:
                coeffs = F.pad(coeffs, (0, 0, 0, deg - coeffs.shape[2]))
            momentum = torch.zeros_like(coeffs)
        gate_global = self.complexity_gate(x_normed.mean(dim=1))  # [B, 1]
        complexity = gate_global.mean()

        # EMA-momentum schedule 0.9 -> 0.7 over 1e8 tokens (sdpc_engine.py:200-209), from the host mirror
        hc = self._host_counters()
        hc[0] += S
        with torch.no_grad():
            self.total_tokens_seen.add_(S)
        ema_momentum = _momentum_schedule(hc[0], hc[1])

        if S < FAST_PATH_THRESHOLD:
            cheby_out, coeffs, momentum = self._cheby(x_normed, coeffs, momentum, ema_momentum, gate_global,
                                                      FAST_PATH_THRESHOLD)
            out = self._fuse(x, cheby_out, self.slr(x_normed, cheby_out=cheby_out))
        elif S < HYBRID_PATH_THRESHOLD:
            cheby_out, coeffs, momentum = self._cheby(x_normed, coeffs, momentum, ema_momentum, gate_global, 0)
            out = self._fuse(x, cheby_out, self.slr(x_normed, cheby_out=cheby_out))
        else:
            out, coeffs, momentum = self._full_path(x, x_normed, coeffs, momentum, ema_momentum, gate_global,
                                                    complexity, hc[0])
        new_state = (coeffs.detach(), momentum.detach())
        return (out, new_state) if return_state else out

    def _full_path(self, x, x_normed, coeffs, momentum, ema_momentum, gate_global, complexity, total):
        B, S, D = x.shape
        n_h, hd, deg = self.n_cheby_heads, self.head_dim, self.max_degree
        if self.gradient_ckpt and self.training:
            from torch.utils.checkpoint import checkpoint
            cheby_out, coeffs, momentum = checkpoint(self._cheby, x_normed, coeffs, momentum, ema_momentum,
                                                     gate_global, 0, use_reentrant=False)
        else:
            cheby_out, coeffs, momentum = self._cheby(x_normed, coeffs, momentum, ema_momentum, gate_global, 0)

        self.archive.maybe_archive(coeffs, S, complexity_score=complexity)
        landmark_embs, _ = self.archive.get_landmark_embeddings(B, x.device)
        if self.light_bus is not None and landmark_embs is not None:
            self.light_bus.publish(self.layer_idx, self.bus_summary_proj(landmark_embs.mean(dim=1)))
        slr_out = self.slr(x_normed, cheby_out)
        if self.light_bus is not None and self.layer_idx > 0:
            bus_ctx = self.light_bus.gather(self.layer_idx, B, x.device)
            if bus_ctx is not None:
                slr_out = slr_out + self.bus_inject_proj(bus_ctx).unsqueeze(1) * 0.1

        # gated state refresh each refresh_interval tokens (sdpc_engine.py:383-388)
        if total > 0 and (total % self.refresh_interval) < S and landmark_embs is not None:
            summary = landmark_embs.mean(dim=1)
            coeffs = coeffs + 0.1 * self.refresh_gate(summary).view(B, n_h, 1, hd) * \
                self.refresh_proj(summary).view(B, n_h, 1, hd)

        # recall residual (sdpc_engine.py:390-412), decided on the device
        n = self.archive.n_host
        cooldown_prev = self.recall_cooldown.clone()
        with torch.no_grad():
            self.recall_cooldown.sub_(S).clamp_(min=0)
        if n > 0:
            archived = self._archive_embs(n).unsqueeze(0).expand(B, -1, -1)
            with torch.no_grad():
                sim = torch.bmm(F.normalize(archived, dim=-1),
                                F.normalize(x_normed.mean(dim=1), dim=-1).unsqueeze(-1)).squeeze(-1)
                max_sim, max_idx = sim.max(dim=-1)
                armed = (cooldown_prev - S <= 0) & (complexity > 0.5)
                inject = (max_sim > 0.15) & armed  # [B]
            best = torch.gather(archived, 1, max_idx.view(B, 1, 1).expand(B, 1, D)).squeeze(1)
            vec = self.recall_proj(best).view(B, n_h, deg, hd)
            g = self.recall_gate(best).view(B, n_h, 1, 1)
            coeffs = coeffs + inject.float().view(B, 1, 1, 1) * 0.08 * g * vec
            with torch.no_grad():
                self.recall_cooldown.copy_(torch.where(inject.any(), torch.full_like(self.recall_cooldown, 4096),
                                                       self.recall_cooldown))
        return self._fuse(x, cheby_out, slr_out), coeffs, momentum


def _momentum_schedule(total: int, ema_base: float) -> float:
    """0.7 + 0.5 (ema_base - 0.7)(1 + cos(pi min(total / 1e8, 1))) in fp32, as the
    reference evaluates it on its buffers (sdpc_engine.py:200-209), here on the
    host."""
    t = torch.tensor(float(total), dtype=torch.float32)
    prog = (t / 1e8).clamp(0.0, 1.0)
    base = torch.tensor(ema_base, dtype=torch.float32)
    return float(0.7 + 0.5 * (base - 0.7) * (1.0 + torch.cos(prog * math.pi)))


def build_ortho_stack(d_model, n_attn_heads, n_cheby_heads=8, n_layers=2, max_degree=4, use_lut=True,
                      gradient_ckpt=False, **kwargs):
    """``n_layers`` engine layers sharing one light bus (sdpc_engine.py:450-467)."""
    bus = AsyncLightBus(summary_dim=64, n_layers=n_layers)
    layers = nn.ModuleList([SpectralDualPathContextEngine(d_model, n_attn_heads, n_cheby_heads, max_degree=max_degree,
                                                          layer_idx=i, light_bus=bus, use_lut=use_lut,
                                                          gradient_ckpt=gradient_ckpt, **kwargs)
                            for i in range(n_layers)])
    return layers, bus


class OrthoSSMLanguageModel(nn.Module):
    """The reference's V10 language model (model.py:23-187) on this engine:
    embedding, an engine stack sharing one light bus, final RMSNorm, LM head
    (tied by default).  forward(input_ids, states=None, return_state=False)."""

    def __init__(self, vocab_size=131072, d_model=256, n_attn_heads=4, n_cheby_heads=8, n_layers=2, max_degree=4,
                 window_size=512, tie_weights=True, use_bf16=False, gradient_ckpt=False, compile_model=False,
                 use_lut=True, **engine_kwargs):
        super().__init__()
        self.d_model, self.n_layers = d_model, n_layers
        self.n_cheby_heads, self.max_degree = n_cheby_heads, max_degree
        self.gradient_ckpt = gradient_ckpt
        self.embedding = nn.Embedding(vocab_size, d_model)
        self.layers, self.light_bus = build_ortho_stack(d_model=d_model, n_attn_heads=n_attn_heads,
                                                        n_cheby_heads=n_cheby_heads, n_layers=n_layers,
                                                        max_degree=max_degree, window_size=window_size,
                                                        use_bf16=use_bf16, use_lut=use_lut,
                                                        gradient_ckpt=gradient_ckpt, **engine_kwargs)
        self.final_norm = nn.RMSNorm(d_model)
        self.lm_head = nn.Linear(d_model, vocab_size, bias=False)
        if tie_weights:
            self.lm_head.weight = self.embedding.weight
        scale = 1.0 / (2 * n_layers) ** 0.5  # model.py _init_weights
        for name, p in self.named_parameters():
            if p.dim() >= 2:
                nn.init.normal_(p, 0.0, 0.02 * (scale if "out_proj" in name else 1.0))
            elif "bias" in name:
                nn.init.zeros_(p)

    def fresh_states(self, batch, device):
        from .sdpc_kernel import init_chebyshev_coefficients
        hd = self.d_model // self.n_cheby_heads
        out = []
        for _ in range(self.n_layers):
            c = init_chebyshev_coefficients(batch, self.n_cheby_heads, self.max_degree, hd, device)
            out.append((c, torch.zeros_like(c)))
        return out

    def forward(self, input_ids, states=None, return_state=False):
        x = self.embedding(input_ids)
        self.light_bus.clear()
        new_states = []
        for i, layer in enumerate(self.layers):
            st = states[i] if states is not None else None
            if self.gradient_ckpt and self.training:
                from torch.utils.checkpoint import checkpoint
                x, st = checkpoint(layer, x, st, True, use_reentrant=False)
            else:
                x, st = layer(x, cheby_state=st, return_state=True)
            new_states.append(st)
        self.light_bus.snapshot()
        logits = self.lm_head(self.final_norm(x))
        return (logits, new_states) if return_state else logits
