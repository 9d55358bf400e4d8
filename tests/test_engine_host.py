"""Host-side parts of the engine drop-in that need no GPU: the light bus
(test_v10.py:248-260 semantics) and the landmark archive."""
import torch

from orthossm_b200.engine import AsyncLightBus, LandmarkArchive, rope_apply, rope_tables


def test_light_bus_publish_gather():
    bus = AsyncLightBus(summary_dim=64, n_layers=4)
    s0 = torch.randn(2, 64)
    bus.publish(0, s0)
    g = bus.gather(1, 2, "cpu")
    assert g is not None and g.shape == (2, 64) and torch.equal(g, s0)
    assert bus.gather(0, 2, "cpu") is None
    bus.publish(1, 3 * s0)
    assert torch.allclose(bus.gather(2, 2, "cpu"), 2 * s0)
    bus.clear()
    assert bus.gather(3, 2, "cpu") is None


def test_archive_interval_and_merge():
    a = LandmarkArchive(d_model=16, n_heads=2, head_dim=4, degree=2, max_landmarks=2, archive_interval=100)
    c = torch.randn(3, 2, 2, 4)
    a.maybe_archive(c, 60)
    assert a.n_host == 0 and a.get_landmark_embeddings(3, "cpu")[0] is None
    a.maybe_archive(c, 60)  # 120 >= 100: archived
    assert a.n_host == 1 and int(a.n_archived) == 1 and int(a.tokens_since) == 0
    assert torch.allclose(a.archived_states[0], c.mean(0))
    a.maybe_archive(2 * c, 100)
    e, n = a.get_landmark_embeddings(3, "cpu")
    assert n == 2 and e.shape == (3, 2, 16)
    a.maybe_archive(-c, 100)  # full: merged into the most similar entry
    assert a.n_host == 2
    ref0, ref1 = c.mean(0), 2 * c.mean(0)
    # -c is most similar (cosine) to neither direction more than the other; one entry moved by 0.1 (-c - e)
    moved = [not torch.allclose(a.archived_states[i], r) for i, r in enumerate((ref0, ref1))]
    assert sum(moved) == 1
    b = LandmarkArchive(d_model=16, n_heads=2, head_dim=4, degree=2, max_landmarks=2, archive_interval=100)
    b.load_state_dict(a.state_dict())
    assert b.n_host == 2


def test_rope_rotates_pairs():
    pos = torch.tensor([[0, 3, 7]])
    cos, sin = rope_tables(pos, 4)
    x = torch.randn(1, 2, 3, 4)
    y = rope_apply(x, cos, sin)
    assert torch.allclose(y[:, :, 0], x[:, :, 0])  # position 0: identity
    assert torch.allclose(y.norm(dim=-1), x.norm(dim=-1), atol=1e-6)  # rotations keep the norm
