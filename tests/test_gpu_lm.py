"""Config-5 LM (orthossm_b200.lm) on the GPU against a float64 restatement of
the same network on the CPU, whose global path is the oracle's
cheby_ema_forward (per-head lambda, per-token gate, carried state)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import cheby_ref as R
from orthossm_b200.lm import OrthoLMConfig, OrthoSSMLM
from orthossm_b200.state import ChebyStreamState
from tests.test_oracle_golden import relerr

pytestmark = pytest.mark.gpu


def ref_forward(model, ids, states):
    """float64 forward of `model` (weights as stored) from the same states."""
    cfg = model.cfg
    P = {n: p.detach().double().cpu() for n, p in model.named_parameters()}
    x = P["embedding.weight"][ids.cpu()]
    finals = []
    for li, (layer, st) in enumerate(zip(model.layers, states)):
        pre = f"layers.{li}."
        h = F.rms_norm(x, (cfg.d_model,), P[pre + "norm_in.weight"], layer.norm_in.eps)
        ema = None if st.ema is None else st.ema.double().cpu().numpy()
        o = R.cheby_ema_forward(h.numpy(), st.coeffs.double().cpu().numpy(),
                                lam=np.asarray(cfg.lambda_per_head, np.float32).astype(np.float64),
                                gate=dict(W=P[pre + "gate.weight"].numpy(), b=P[pre + "gate.bias"].numpy(),
                                          scale=cfg.gate_scale), init=ema)
        g = torch.from_numpy(o["out"])
        finals.append(o["final"])
        B, S, d = x.shape
        H = cfg.n_heads
        q, k, v = (h @ P[pre + "qkv.weight"].t()).view(B, S, 3, H, d // H).unbind(2)
        i = torch.arange(S).view(S, 1)
        j = torch.arange(S).view(1, S)
        mask = (j <= i) & (j > i - cfg.window)
        a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           attn_mask=mask).transpose(1, 2).reshape(B, S, d)
        loc = a @ P[pre + "o.weight"].t()
        c = F.layer_norm(g + loc, (d,), P[pre + "norm_comb.weight"], P[pre + "norm_comb.bias"], layer.norm_comb.eps)
        x = x + c @ P[pre + "out_proj.weight"].t()
    x = F.rms_norm(x, (cfg.d_model,), P["final_norm.weight"], model.final_norm.eps)
    return x @ P["embedding.weight"].t(), finals


@pytest.mark.parametrize("dtype,tol,state_tol", [(torch.float32, 1e-4, 1e-4), (torch.bfloat16, 2e-2, 5e-3)])
def test_lm_forward_matches_float64(dtype, tol, state_tol):
    """The whole network in fp32 and in bf16 (the decays stay fp32 in a bf16
    model: 0.9995 would round to 1.0) against float64."""
    torch.manual_seed(0)
    cfg = OrthoLMConfig(vocab_size=1000, n_layers=2, window=64)
    model = OrthoSSMLM(cfg).to("cuda", dtype)
    B, S = 2, 300
    ids = torch.randint(0, cfg.vocab_size, (B, S), device="cuda")
    states = model.fresh_states(B, "cuda", generator_seed=1)
    states[1] = ChebyStreamState(coeffs=states[1].coeffs, ema=0.1 * torch.randn(B, cfg.d_model, device="cuda"))
    with torch.no_grad():
        logits, new = model(ids, states, return_state=True)
    torch.cuda.synchronize()
    ref, finals = ref_forward(model, ids, states)
    assert relerr(logits.float().cpu().numpy(), ref.numpy()) < tol
    for st, f in zip(new, finals):
        assert relerr(st.ema.cpu().numpy(), f) < state_tol
        assert st.tokens_seen == S


def test_lm_streaming_carries_the_global_state():
    """Two calls carrying the layers' EMA states leave the first layer (whose
    input depends on the tokens alone) in the state one call over the whole
    sequence reaches; deeper layers differ only through the local window,
    which restarts at a call boundary."""
    torch.manual_seed(1)
    cfg = OrthoLMConfig(vocab_size=1000, n_layers=2, window=64)
    model = OrthoSSMLM(cfg).to("cuda", torch.float32)
    ids = torch.randint(0, cfg.vocab_size, (2, 400), device="cuda")
    st0 = model.fresh_states(2, "cuda", generator_seed=2)
    with torch.no_grad():
        _, whole = model(ids, st0, return_state=True)
        _, mid = model(ids[:, :150], st0, return_state=True)
        _, end = model(ids[:, 150:], mid, return_state=True)
    assert relerr(end[0].ema.cpu().numpy(), whole[0].ema.cpu().numpy()) < 1e-5
    assert end[0].tokens_seen == 400


def test_lm_global_path_calls_bf16(monkeypatch):
    """In the bf16 model, every layer's global-path call (bf16 input, gate,
    carried state) matches the oracle on that same input within the bf16-I/O
    tolerance."""
    import orthossm_b200.lm as LM
    calls = []
    real = LM.cheby_ema_forward

    def rec(h, coeffs, **kw):
        out, fin = real(h, coeffs, **kw)
        calls.append((h.detach().float().cpu().numpy(), coeffs.detach().cpu().numpy(), kw, out.float().cpu().numpy(),
                      fin.cpu().numpy()))
        return out, fin

    monkeypatch.setattr(LM, "cheby_ema_forward", rec)
    torch.manual_seed(3)
    cfg = OrthoLMConfig(vocab_size=1000, n_layers=2, window=64)
    model = OrthoSSMLM(cfg).to("cuda", torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size, (2, 300), device="cuda")
    states = model.fresh_states(2, "cuda", generator_seed=4)
    with torch.no_grad():
        model(ids, states)
    assert len(calls) == 2
    for h, c, kw, out, fin in calls:
        init = None if kw["init_state"] is None else kw["init_state"].cpu().numpy()
        o = R.cheby_ema_forward(h, c, lam=kw["lambda_per_head"].cpu().numpy().astype(np.float64),
                                gate=dict(W=kw["gate_weight"].cpu().numpy(), b=kw["gate_bias"].cpu().numpy(),
                                          scale=kw["gate_scale"]), init=init)
        assert relerr(out, o["out"]) < 2e-2
        assert relerr(fin, o["final"]) < 2e-2


def test_flash_window_matches_blocked():
    """The sliding-window kernel the bf16 layer uses against the blocked SDPA
    restatement (fp32 on the same bf16 inputs)."""
    from orthossm_b200.lm import local_window_attention, local_window_attention_blocked
    torch.manual_seed(5)
    q, k, v = (torch.randn(2, 1500, 8, 64, device="cuda").to(torch.bfloat16) for _ in range(3))
    a = local_window_attention(q, k, v, 512).float()
    b = local_window_attention_blocked(q.float(), k.float(), v.float(), 512)
    assert relerr(a.cpu().numpy(), b.cpu().numpy()) < 1e-2
