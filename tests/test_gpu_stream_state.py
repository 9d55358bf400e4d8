"""Streaming with a save / resume in the middle (orthossm_b200.state) equals
the uninterrupted stream, on the GPU, in all three stream modes."""
import numpy as np
import pytest
import torch

from oracle import cheby_ref as R
from orthossm_b200.state import ChebyStreamState, StreamingChebyRKV
from tests.golden.inputs import det_normal, linear_init, spectral_coeffs
from tests.test_oracle_golden import relerr

pytestmark = pytest.mark.gpu


def _t(a, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dt)


def _stream(make, x, cuts, resume_at):
    """Run x through the stream in pieces; at piece ``resume_at`` serialise the
    state, drop the streamer and continue from the loaded bytes."""
    s = make(None)
    outs = []
    for i, (a, b) in enumerate(zip(cuts[:-1], cuts[1:])):
        if i == resume_at:
            blob = s.state.to_bytes()
            del s
            s = make(ChebyStreamState.from_bytes(blob, device="cuda"))
        outs.append(s(x[:, a:b]))
    torch.cuda.synchronize()
    return torch.cat(outs, 1), s.state


def test_baseline_stream_resume_equals_one_call():
    import orthossm_b200 as O
    B, S, D, H = 2, 6000, 512, 8
    x = _t(R.bf16_round(det_normal((B, S, D), 2100)), torch.bfloat16)
    c = _t(spectral_coeffs(B, H, 8, 64, 2101))
    W, b = linear_init(H, D, 2102)
    init = _t(det_normal((B, D), 2103, 0.1))
    lam = list(R.BASELINE_LAMBDA)
    kw = dict(lambda_per_head=lam, gate_weight=_t(W), gate_bias=_t(b))

    def make(st):
        st = st or ChebyStreamState(coeffs=c.clone(), ema=init.clone())
        return StreamingChebyRKV(st, mode="baseline", **kw)

    out, st = _stream(make, x, [0, 1000, 2500, 2501, 4096, 6000], resume_at=2)
    ref, fin = O.cheby_ema_forward(x, c, init_state=init, **kw)
    assert (out.float() - ref.float()).abs().max().item() <= 2 ** -7
    assert relerr(st.ema.cpu().numpy(), fin.cpu().numpy()) < 1e-5
    assert st.tokens_seen == S


def test_reference_stream_resume_is_exact():
    """Reference mode (Lion TTT, EMA reset per call): resuming from the saved
    bytes changes nothing, bit for bit."""
    B, S, D, H = 2, 2048, 512, 8
    x = _t(det_normal((B, S, D), 2200))
    c = _t(spectral_coeffs(B, H, 8, 64, 2201))

    def make(st):
        st = st or ChebyStreamState.from_reference((c.clone(), torch.zeros_like(c)))
        return StreamingChebyRKV(st, mode="reference", chunk_size=256)

    cuts = [0, 512, 1024, 1536, 2048]
    a, sa = _stream(make, x, cuts, resume_at=-1)
    b, sb = _stream(make, x, cuts, resume_at=2)
    assert torch.equal(a, b)
    assert torch.equal(sa.coeffs, sb.coeffs) and torch.equal(sa.momentum, sb.momentum)
    assert sb.step == 4


def test_baseline_ttt_stream_resume_is_exact():
    """BASELINE TTT (W_pred Adam): coefficients, moments, step and EMA state
    all survive the round trip, so the resumed stream is bit for bit the same."""
    B, S, D, H = 2, 1024, 512, 8
    x = _t(R.bf16_round(det_normal((B, S, D), 2300)), torch.bfloat16)
    c = _t(spectral_coeffs(B, H, 8, 64, 2301))
    Wp = _t(det_normal((D, D), 2302, 0.02))
    lam = list(R.BASELINE_LAMBDA)

    def make(st):
        st = st or ChebyStreamState(coeffs=c.clone())
        return StreamingChebyRKV(st, mode="baseline", lambda_per_head=lam, W_pred=Wp, ttt_chunk=256)

    cuts = [0, 256, 512, 768, 1024]
    a, sa = _stream(make, x, cuts, resume_at=-1)
    b, sb = _stream(make, x, cuts, resume_at=2)
    assert torch.equal(a, b)
    for n in ("coeffs", "momentum", "adam_v", "ema"):
        assert torch.equal(getattr(sa, n), getattr(sb, n)), n
    assert sa.step == sb.step == 4
