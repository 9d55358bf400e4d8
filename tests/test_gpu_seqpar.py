"""Sequence sharding on the GPU, through the C ABI (ossm_fwd_shard_aggregate /
ossm_fwd_shard_output) and through ``cheby_ema_forward_seqpar``.

* one GPU: the sequence is cut into G shards that run one after another on
  the same device, with the carry folded on the host side in between; the
  joined outputs must match the unsharded forward and the oracle;
* two GPUs (skipped when the box has one): two NCCL ranks, each with its
  shard, against the unsharded forward."""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch

from oracle import cheby_ref as R
from orthossm_b200 import _lib as L
from tests.golden.inputs import det_normal, linear_init, spectral_coeffs
from tests.test_oracle_golden import relerr

pytestmark = pytest.mark.gpu


def _t(a, dt=torch.float32, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt)


def _problem(B, S, seed):
    D, H = 512, 8
    x = R.bf16_round(det_normal((B, S, D), seed)).astype(np.float32)
    c = spectral_coeffs(B, H, 8, 64, seed + 1)
    W, b = linear_init(H, D, seed + 2)
    init = det_normal((B, D), seed + 3, 0.1)
    lam = np.asarray(R.BASELINE_LAMBDA, np.float32)
    return x, c, W, b, init, lam


@pytest.mark.parametrize("B,S,G,gate", [(2, 4096, 2, True), (1, 3000, 4, True), (2, 2048, 4, False),
                                        (1, 40000, 8, True), (1, 70001, 2, True)])
def test_shards_on_one_gpu_match_unsharded(B, S, G, gate):
    """The sharded protocol with every shard on one GPU (aggregates, packed
    totals, device fold, outputs) against the unsharded forward and the
    oracle; the device fold against the host fold of the same totals."""
    import orthossm_b200 as O
    from orthossm_b200.sdpc_kernel import cheby_ema_forward_shards_local, fold_shard_carries, _shard_fold
    x, c, W, b, init, lam = _problem(B, S, 900 + S + G)
    xb = _t(x, torch.bfloat16)
    kw = dict(lambda_per_head=lam.tolist())
    if gate:
        kw.update(gate_weight=_t(W), gate_bias=_t(b))
    full, fin_full = O.cheby_ema_forward(xb, _t(c), init_state=_t(init), **kw)
    joined, fin = cheby_ema_forward_shards_local(xb, _t(c), G, init_state=_t(init), **kw)
    torch.cuda.synchronize()
    j = joined.float().cpu().numpy()
    assert np.abs(j - full.float().cpu().numpy()).max() <= 2 ** -7
    assert relerr(fin.cpu().numpy(), fin_full.cpu().numpy()) < 1e-5
    o = R.cheby_ema_forward(x, c, lam=lam.astype(np.float64), gate=dict(W=W, b=b) if gate else None, init=init)
    assert relerr(j, o["out"]) < 2e-2
    assert relerr(fin.cpu().numpy(), o["final"]) < 1e-3
    assert O.workspace_status() == 0


def test_device_fold_is_the_host_fold():
    """ossm_fwd_shard_fold against fold_shard_carries on random packed
    totals: the same fold order, so the same carries to fp32 rounding of
    one multiply-add per shard."""
    from orthossm_b200.sdpc_kernel import fold_shard_carries, _shard_fold
    g = torch.Generator().manual_seed(5)
    B, H, hd, G = 3, 8, 64, 8
    D = H * hd
    dec = torch.rand(G, B, H, generator=g) * 0.5 + 0.5
    st = torch.randn(G, B, D, generator=g)
    init = 0.1 * torch.randn(B, D, generator=g)
    totals = torch.cat([dec.reshape(G, -1), st.reshape(G, -1)], dim=1).cuda()
    stream = torch.cuda.current_stream()
    for upto in range(G + 1):
        dev = _shard_fold(B, H, hd, upto, totals, init.cuda(), stream).cpu()
        host = fold_shard_carries(list(dec), list(st), upto, init)
        assert torch.allclose(dev, host, rtol=1e-6, atol=1e-6), upto
    assert torch.equal(_shard_fold(B, H, hd, 0, totals, None, stream).cpu(), torch.zeros(B, D))


def test_shard_entry_points_reject_other_paths():
    """fp32 x (the generic kernel) has no sharded path: EINVAL, nothing launched."""
    from orthossm_b200.sdpc_kernel import _fwd_args
    x, c, W, b, init, lam = _problem(1, 256, 5)
    a, keep, out, fin = _fwd_args(_t(x), _t(c), lambda_per_head=lam.tolist())
    lib = L.lib()
    nb = lib.ossm_fwd_workspace_bytes(C.byref(a))
    ws = torch.zeros(max(nb, 1 << 20), dtype=torch.uint8, device="cuda")
    dec = torch.empty(1, 8, device="cuda")
    st = torch.empty(1, 512, device="cuda")
    assert lib.ossm_fwd_shard_aggregate(C.byref(a), 1, ws.data_ptr(), ws.numel(), dec.data_ptr(), st.data_ptr(),
                                        None) == L.OSSM_EINVAL


def _nccl_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import orthossm_b200 as O
        B, S = 2, 8192
        x, c, W, b, init, lam = _problem(B, S, 4242)
        dev = f"cuda:{rank}"
        kw = dict(lambda_per_head=lam.tolist(), gate_weight=_t(W, dev=dev), gate_bias=_t(b, dev=dev))
        xb = _t(x, torch.bfloat16, dev)
        full, fin_full = O.cheby_ema_forward(xb, _t(c, dev=dev), init_state=_t(init, dev=dev), **kw)
        L_ = S // world
        xs = xb[:, rank * L_:(rank + 1) * L_].contiguous()
        out, fin = O.cheby_ema_forward_seqpar(xs, _t(c, dev=dev), init_state=_t(init, dev=dev), **kw)
        torch.cuda.synchronize()
        err = (out.float() - full[:, rank * L_:(rank + 1) * L_].float()).abs().max().item()
        ferr = relerr(fin.cpu().numpy(), fin_full.cpu().numpy())
        q.put((rank, err, ferr))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpus_nccl_match_unsharded():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err, ferr in res:
        assert err <= 2 ** -7, (rank, err)
        assert ferr < 1e-5, (rank, ferr)
