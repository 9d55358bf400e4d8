"""Generate the engine-level golden fixture by running the reference's own SDPC
engine (sdpc_engine.py) and local refiner (slr_module.py) on CPU.

The reference does not ship ``landmark_archive.py``; this script injects
``orthossm_b200.engine``'s ``AsyncLightBus`` / ``LandmarkArchive`` under that
module name, so both sides run the same archive and everything else is the
reference's code.  Triton kernels run under ``TRITON_INTERPRET=1``.  It is run
once, offline (it needs the reference checkout); tests read only the
committed ``engine_stack.npz``.

    python tests/golden/make_engine_golden.py --ref <path-to-OrthoSSM>

Fixture: a 2-layer ``build_ortho_stack`` (d_model 64, 2 attention heads,
8 Chebyshev heads of 8, degree 4, LUT, window 64, 4 landmarks archived every
512 tokens, state refresh every 2048 tokens) called four times in a row on
B=1 sequences of 64, 512, 1100 and 1100 tokens (fast, hybrid, full, full),
each call starting from the states the previous one returned and a cleared
bus (as model.py:141 does).  It stores the initial state_dict and, per call,
the input and each layer's output and returned (coeffs, momentum).
"""
from __future__ import annotations

import argparse
import os
import sys
import time
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

CALLS = (64, 512, 1100, 1100)
CFG = dict(d_model=64, n_attn_heads=2, n_cheby_heads=8, n_layers=2, max_degree=4, use_lut=True, window_size=64,
           max_landmarks=4, archive_interval=512)
REFRESH = 2048


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("OSSM_REFERENCE"))
    ap.add_argument("--out", default=os.path.join(HERE, "engine_stack.npz"))
    a = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, a.ref)
    import torch

    from orthossm_b200 import engine as ours
    shim = types.ModuleType("landmark_archive")
    shim.AsyncLightBus, shim.LandmarkArchive = ours.AsyncLightBus, ours.LandmarkArchive
    sys.modules["landmark_archive"] = shim
    import sdpc_engine as E

    torch.manual_seed(20251)
    layers, bus = E.build_ortho_stack(**CFG)
    for L in layers:
        L.refresh_interval = REFRESH
        for name, p in L.named_parameters():  # non-zero everywhere, so every path shows
            if "coeff_init_proj.2" in name:
                torch.nn.init.normal_(p, 0.0, 0.05)
    g = torch.Generator().manual_seed(7)
    xs = [torch.randn(1, S, CFG["d_model"], generator=g) for S in CALLS]
    with torch.no_grad():
        for L in layers:  # a complexity gate above 0.5 arms the recall residual
            L.complexity_gate.net[2].bias.fill_(2.0)
        # layer 0's landmark embeddings point along the last call's mean normed
        # input, so its recall similarity clears 0.15 and the residual is injected
        d = layers[0].input_norm(xs[-1]).mean(1)[0]
        layers[0].archive.state_to_embedding.bias.copy_(8.0 * d / d.norm())
    layers.eval()
    sd = {k: v.detach().clone() for k, v in layers.state_dict().items()}
    fix = {f"sd/{k}": v.numpy() for k, v in sd.items()}
    states = [None] * CFG["n_layers"]
    for ci, S in enumerate(CALLS):
        x = xs[ci]
        fix[f"c{ci}/x"] = x.numpy()
        bus.clear()
        h = x
        t0 = time.time()
        with torch.no_grad():
            for li, L in enumerate(layers):
                h, st = L(h, cheby_state=states[li], return_state=True)
                states[li] = st
                fix[f"c{ci}/l{li}/out"] = h.numpy()
                fix[f"c{ci}/l{li}/coeffs"] = st[0].numpy()
                fix[f"c{ci}/l{li}/momentum"] = st[1].numpy()
        print(f"call {ci} (S={S}) done in {time.time() - t0:.1f} s; per layer (archived, recall cooldown):",
              [(int(L.archive.n_archived), int(L.recall_cooldown)) for L in layers], flush=True)
    np.savez_compressed(a.out, **fix)
    print("wrote", a.out, os.path.getsize(a.out), "bytes")


if __name__ == "__main__":
    main()
