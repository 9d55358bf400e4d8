"""SDPC engine drop-in (orthossm_b200.engine) against the reference's own
engine: a 2-layer stack loaded from the reference's state_dict replays the
golden call sequence (fast, hybrid, full, full; archive, state refresh, recall
residual and light bus all active), and a forward makes no host sync."""
import os

import numpy as np
import pytest
import torch

from tests.test_oracle_golden import relerr

pytestmark = pytest.mark.gpu
FIX = os.path.join(os.path.dirname(__file__), "golden", "engine_stack.npz")
CFG = dict(d_model=64, n_attn_heads=2, n_cheby_heads=8, n_layers=2, max_degree=4, use_lut=True, window_size=64,
           max_landmarks=4, archive_interval=512)


def _stack(z):
    from orthossm_b200.engine import build_ortho_stack
    layers, bus = build_ortho_stack(**CFG)
    for L in layers:
        L.refresh_interval = 2048
    sd = {k[3:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("sd/")}
    layers.load_state_dict(sd, strict=True)
    return layers.to("cuda").eval(), bus


def test_engine_stack_matches_reference_golden():
    z = np.load(FIX)
    layers, bus = _stack(z)
    states = [None, None]
    for ci in range(4):
        h = torch.from_numpy(z[f"c{ci}/x"]).cuda()
        bus.clear()
        with torch.no_grad():
            for li, L in enumerate(layers):
                h, st = L(h, cheby_state=states[li], return_state=True)
                states[li] = st
                tag = f"call {ci} layer {li}"
                assert relerr(h.cpu().numpy(), z[f"c{ci}/l{li}/out"]) < 1e-4, tag
                assert relerr(st[0].cpu().numpy(), z[f"c{ci}/l{li}/coeffs"]) < 1e-4, tag
                assert relerr(st[1].cpu().numpy(), z[f"c{ci}/l{li}/momentum"]) < 1e-4, tag
    # the recall residual fired in layer 0 of the last call (cooldown reset), the archive holds 2
    assert [int(L.recall_cooldown) for L in layers] == [4096, 0]
    assert [int(L.archive.n_archived) for L in layers] == [2, 2]


def test_engine_forward_makes_no_host_sync():
    z = np.load(FIX)
    layers, bus = _stack(z)
    x = torch.randn(1, 1100, 64, device="cuda")
    with torch.no_grad():
        layers[0](x, return_state=True)  # first call: host mirrors read once
        torch.cuda.synchronize()
        torch.cuda.set_sync_debug_mode("error")
        try:
            for S in (64, 512, 1100):
                out, st = layers[0](x[:, :S], return_state=True)
                out, st = layers[0](x[:, :S], cheby_state=st, return_state=True)
        finally:
            torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()


def test_language_model_v10_runs_and_carries_states():
    from orthossm_b200.engine import OrthoSSMLanguageModel
    torch.manual_seed(0)
    m = OrthoSSMLanguageModel(vocab_size=1000, d_model=64, n_attn_heads=4, n_cheby_heads=8, n_layers=2,
                              window_size=256).cuda().eval()
    with torch.no_grad():
        for S in (64, 1024):
            ids = torch.randint(0, 1000, (2, S), device="cuda")
            logits, st = m(ids, return_state=True)
            assert logits.shape == (2, S, 1000) and torch.isfinite(logits).all()
            assert len(st) == 2 and st[0][0].shape == (2, 8, 4, 8)
