"""Sequence sharding, host side, on CPU: two gloo ranks each take one shard of
a sequence, compute its totals with the oracle, exchange them through
``exchange_shard_totals`` (torch.distributed all-gather) and fold the state
entering their shard with ``fold_shard_carries``.  The carries and the final
state must equal the oracle's single-sequence scan at the shard boundaries."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import cheby_ref as R
from tests.golden.inputs import det_normal, linear_init, spectral_coeffs

B, S, H, HD = 2, 96, 8, 8
D = H * HD


def _problem():
    x = R.bf16_round(det_normal((B, S, D), 71))
    c = spectral_coeffs(B, H, 8, HD, 72)
    W, b = linear_init(H, D, 73)
    init = det_normal((B, D), 74, 0.1)
    lam = np.asarray(R.BASELINE_LAMBDA, np.float64)
    return x, c, dict(W=W, b=b), init, lam


def _shard_totals(rank, world):
    """(decay [B,H], end state [B,D]) of shard `rank`, from the oracle."""
    x, c, gate, init, lam = _problem()
    L = S // world
    xs = x[:, rank * L:(rank + 1) * L]
    r = R.cheby_ema_forward(xs, c, lam=lam, gate=gate, init=init if rank == 0 else None)
    lam_t = r["lam_t"]  # [B, L, H]
    decay = np.prod(lam_t, axis=1)
    if rank == 0:
        decay = np.zeros_like(decay)  # token 0 of the sequence takes the carried-in state
    return decay, r["final"]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from orthossm_b200.sdpc_kernel import exchange_shard_totals, fold_shard_carries
        d, e = _shard_totals(rank, world)
        decays, states = exchange_shard_totals(torch.from_numpy(d).float(), torch.from_numpy(e).float())
        init = torch.from_numpy(_problem()[3]).float()
        carry = fold_shard_carries(decays, states, rank, init)
        final = fold_shard_carries(decays, states, world, init)
        q.put((rank, carry.numpy(), final.numpy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_shard_carries_match_oracle(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, carry, final = q.get(timeout=120)
        res[rank] = (carry, final)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, c, gate, init, lam = _problem()
    full = R.cheby_ema_forward(x, c, lam=lam, gate=gate, init=init)
    L = S // world
    for r in range(world):
        carry, final = res[r]
        want = init if r == 0 else full["out"][:, r * L - 1]
        np.testing.assert_allclose(carry, want, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(final, full["final"], rtol=1e-5, atol=1e-6)
        # identical on every rank
        np.testing.assert_array_equal(final, res[0][1])


def test_fold_matches_numpy_fold():
    rng = np.random.default_rng(3)
    ends = [rng.normal(size=(B, D)) for _ in range(3)]
    decs = [rng.uniform(0.5, 1.0, size=(B, H)) for _ in range(3)]
    from orthossm_b200.sdpc_kernel import fold_shard_carries
    init = rng.normal(size=(B, D))
    got = [fold_shard_carries([torch.tensor(d, dtype=torch.float32) for d in decs],
                              [torch.tensor(e, dtype=torch.float32) for e in ends], r,
                              torch.tensor(init, dtype=torch.float32)).numpy() for r in range(3)]
    want = R.fold_shard_carries(ends, [np.repeat(d, HD, axis=1) for d in decs], init)
    for g, w in zip(got, want):
        np.testing.assert_allclose(g, w, rtol=1e-5, atol=1e-6)
