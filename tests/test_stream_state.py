"""Stream-state format (orthossm_b200.state): round trips, the reference's
cheby_state tuple forms, and rejection of damaged or foreign files.  CPU only."""
import hashlib

import pytest
import torch

from orthossm_b200.state import MAGIC, ChebyStreamState


def _state(B=2, H=8, K=8, hd=64, full=True, seed=0):
    g = torch.Generator().manual_seed(seed)
    c = torch.randn(B, H, K, hd, generator=g)
    kw = {}
    if full:
        kw = dict(momentum=torch.randn(B, H, K, hd, generator=g), adam_v=torch.rand(B, H, K, hd, generator=g),
                  ema=torch.randn(B, H * hd, generator=g), step=7, tokens_seen=123456, meta={"mode": "baseline"})
    return ChebyStreamState(coeffs=c, **kw)


def _eq(a, b):
    assert a.step == b.step and a.tokens_seen == b.tokens_seen and a.meta == b.meta
    for n in ("coeffs", "momentum", "adam_v", "ema"):
        x, y = getattr(a, n), getattr(b, n)
        assert (x is None) == (y is None)
        if x is not None:
            assert x.dtype == y.dtype and torch.equal(x, y)


@pytest.mark.parametrize("full", [True, False])
def test_round_trip_bytes_and_file(full, tmp_path):
    s = _state(full=full)
    _eq(s, ChebyStreamState.from_bytes(s.to_bytes()))
    p = tmp_path / "s.ossm"
    s.save(p)
    _eq(s, ChebyStreamState.load(p))


def test_bf16_ema_round_trip():
    s = _state()
    s.ema = s.ema.to(torch.bfloat16)
    _eq(s, ChebyStreamState.from_bytes(s.to_bytes()))


def test_format_is_stable():
    """A fixed state serialises to fixed bytes (format version 1)."""
    c = torch.arange(2 * 2 * 3 * 4, dtype=torch.float32).reshape(2, 2, 3, 4) / 7
    s = ChebyStreamState(coeffs=c, momentum=-c, ema=torch.ones(2, 8), step=3, tokens_seen=99)
    data = s.to_bytes()
    assert data[:8] == MAGIC
    assert hashlib.sha256(data).hexdigest() == DIGEST_V1


@pytest.mark.parametrize("damage", ["magic", "version", "crc", "truncate", "header"])
def test_damaged_input_is_rejected(damage):
    data = bytearray(_state().to_bytes())
    if damage == "magic":
        data[0] ^= 0xFF
    elif damage == "version":
        data[7] = 9
    elif damage == "crc":
        data[-5] ^= 0x01
    elif damage == "truncate":
        data = data[:-100]
    else:
        data[8:12] = (10 ** 9).to_bytes(4, "little")
    with pytest.raises(ValueError):
        ChebyStreamState.from_bytes(bytes(data))


def test_shape_checks():
    c = torch.zeros(2, 8, 8, 64)
    with pytest.raises(ValueError):
        ChebyStreamState(coeffs=c, momentum=torch.zeros(2, 8, 4, 64)).validate()
    with pytest.raises(ValueError):
        ChebyStreamState(coeffs=c, ema=torch.zeros(2, 256)).validate()
    with pytest.raises(ValueError):
        ChebyStreamState(coeffs=torch.zeros(8, 8, 64)).validate()


def test_reference_tuple_forms():
    """(coeffs, momentum), legacy (coeffs, m1, m2) and a bare [B, K, hd] or
    [B, H, K, hd] tensor, as the engine accepts them (sdpc_engine.py:175-191)."""
    c = torch.randn(2, 8, 8, 64)
    m = torch.randn(2, 8, 8, 64)
    s = ChebyStreamState.from_reference((c, m))
    assert torch.equal(s.coeffs, c) and torch.equal(s.momentum, m)
    s3 = ChebyStreamState.from_reference((c, m, torch.ones_like(m)))
    assert torch.equal(s3.momentum, m)
    sb = ChebyStreamState.from_reference(c[:, 0])
    assert sb.coeffs.shape == (2, 1, 8, 64) and not sb.momentum.any()
    cc, mm = s.to_reference()
    assert torch.equal(cc, c) and torch.equal(mm, m)


DIGEST_V1 = "e340411fae13320fd3610512e421fd5b395d6cb5df4a1f3f85978a40d954e178"
