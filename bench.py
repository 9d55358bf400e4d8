#!/usr/bin/env python
"""Benchmark of the fused Cheby-EMA forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one forward pass over one batch: B=8 sequences per GPU of S=16384
tokens, D=512 (8 heads x 64), Chebyshev degree 8, bf16 input/output, fp32
state, per-token dynamic decay from a random-init Linear(512->8) gate, carried
state ~N(0, 0.1).  Multi-GPU: batch sharding (each rank its own B=8 batch,
weak scaling, no collective on the data path).  Rank 0 prints one JSON line.

--impl reference times the oracle's C port (the reference algorithm on the
host cores, all threads) on the same workload; under torchrun only rank 0
runs it.

--workload cfg3 times BASELINE.json configs[2]: one sequence of S=1,048,576
tokens (bf16, fixed per-head decays, no gate) sharded along the sequence over
the ranks (strong scaling; one NCCL all-gather of the shard totals).
--workload cfg4 times configs[3]: the W_pred Adam TTT over B=4 x S=32768 per
GPU in 2048-token chunks (weak scaling, batch-parallel).

--workload cfg5 times instead the config-5 LM forward (BASELINE.json
configs[4]; orthossm_b200.lm): per GPU B=2 x S=65536 token ids, 6 V8 layers
of d_model 512, vocab 32000, bf16.  Its JSON line reports tokens/s of the
forward (value), of ids-in / loss-out through the model (e2e), and the share of
the step spent in this package's Cheby-EMA kernels.
--workload lion times the reference's live op (apply_cheby_rkv_v10 with its
chunked Lion TTT) at B=2 x S=65536 per GPU.

The default line also carries sub-records for those workloads (seqpar, cfg4,
lion, cfg5) and for the opt-in single-evaluation forward (single_eval), each
timed with CUDA events on the bench's stream, max over ranks.
--profile-once (cfg2, cfg3, cfg4, lion) runs 3 warm-up steps and one more,
nothing timed: the command that ncu captures.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, S, D, H, K = 8, 16384, 512, 8, 8
HD = D // H
LAMBDA = [0.9995, 0.9995, 0.997, 0.997, 0.995, 0.995, 0.95, 0.95]
WORKLOAD = ("cfg2: per GPU B=8 x S=16384 tokens, D=512 (8 heads x 64), Chebyshev degree 8, "
            "bf16 in/out, fp32 state, per-token decay gate Linear(512->8), carried state N(0,0.1)")


def config_dict(world):
    """The workload description both arms print, so their lines compare."""
    return {"workload": WORKLOAD, "global_batch": B * world, "seq_len": S,
            "parallelism": f"batch-sharded x{world} (no collective)",
            "l2": "inputs larger than L2: two rotating 134 MB input buffers"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--soak-s", type=float, default=1.5, help="loaded seconds sampled for clocks before timing")
    ap.add_argument("--workload", choices=["cfg2", "cfg3", "cfg4", "cfg5", "lion"], default="cfg2")
    ap.add_argument("--profile-once", action="store_true",
                    help="3 warm-up steps + 1 step, nothing else: for ncu")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ----------------------------------------------------------------------------
# CPU baseline: the oracle's C port (reference algorithm), all host threads
# ----------------------------------------------------------------------------

def host_threads():
    """Threads for the CPU legs: every core this process may run on.  (torchrun
    sets OMP_NUM_THREADS=1 for its ranks, so OpenMP's own default would give
    the reference arm one thread under N > 1.)"""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample(x_bits, c, W, b, init, lam, budget_s=8.0, max_reps=20):
    """Time the C port on the full per-GPU workload (one step = B*S tokens),
    repeated until ~budget_s of CPU time; returns (tokens/s, threads, sample)."""
    import numpy as np
    from oracle import cref
    out = np.empty(x_bits.shape, np.uint16)
    fin = np.empty((x_bits.shape[0], x_bits.shape[2]), np.float32)
    nth = host_threads()
    ts = []
    t_all = time.perf_counter()
    while len(ts) < max_reps and (time.perf_counter() - t_all) < budget_s:
        t0 = time.perf_counter()
        cref.forward(x_bits, c, lam=lam, gate=dict(W=W, b=b), init=init, out_bf16=True,
                     x_is_bf16_bits=True, out=out, fin=fin, nthreads=nth)
        ts.append(time.perf_counter() - t0)
    tok = x_bits.shape[0] * x_bits.shape[1]
    best = min(ts)
    sample = (f"oracle C port (oracle/cheby_ref.c, fp32, OpenMP) on the full per-GPU step "
              f"({x_bits.shape[0]}x{x_bits.shape[1]} tokens), best of {len(ts)} reps")
    return tok / best, nth, sample


def small_inputs(seed):
    """Deterministic coefficients, gate weights and carried state (numpy)."""
    from tests.golden.inputs import det_normal, linear_init, spectral_coeffs
    c = spectral_coeffs(B, H, K, HD, seed + 1)
    W, b = linear_init(H, D, seed + 2)
    init = det_normal((B, D), seed + 3, 0.1)
    return c, W, b, init


def x_bits_host(seed):
    """x ~ N(0,1) rounded to bf16, as uint16 bits [B,S,D] (numpy, host)."""
    import numpy as np
    import torch
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, S, D, generator=g).to(torch.bfloat16)
    return x.view(torch.int16).numpy().view(np.uint16)


def run_reference(args):
    import numpy as np
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    x_bits = x_bits_host(1234)
    c, W, b, init = small_inputs(1234)
    lam = np.asarray(LAMBDA, np.float32)
    from oracle import cref
    nth = host_threads()
    out = np.empty(x_bits.shape, np.uint16)
    fin = np.empty((B, D), np.float32)
    for _ in range(max(args.warmup, 0)):
        cref.forward(x_bits, c, lam=lam, gate=dict(W=W, b=b), init=init, out_bf16=True,
                     x_is_bf16_bits=True, out=out, fin=fin, nthreads=nth)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cref.forward(x_bits, c, lam=lam, gate=dict(W=W, b=b), init=init, out_bf16=True,
                     x_is_bf16_bits=True, out=out, fin=fin, nthreads=nth)
    dt = time.perf_counter() - t0
    v = B * S * args.steps / dt
    sample = (f"oracle C port (oracle/cheby_ref.c, fp32, OpenMP, {nth} threads): the reference "
              f"algorithm on the host cores; each step the full per-GPU workload {B}x{S} tokens")
    line = {
        "impl": "reference", "metric": "tokens/sec", "value": v, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 compute (bf16 in/out)", "data": "synthetic",
        "config": config_dict(int(os.environ.get("WORLD_SIZE", "1"))),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": nth, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.idx = gpu_id  # nvidia-smi -i accepts "GPU-<uuid>"
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 9]
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                util = float(r[4])
                mhz = float(r[1])
                smax = float(r[2])
            except ValueError:
                continue
            if util > 0:
                sm.append(mhz)
                for n, v in zip(names, r[6:10]):
                    if v.strip().lower().startswith("active"):
                        reasons.add(n)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": smax, "reasons": sorted(reasons), "samples_under_load": len(sm)}


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    import orthossm_b200 as O

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- inputs (per rank; 2 rotating buffers, each 134 MB > 126 MB L2) ----
    x_bits = x_bits_host(1234 + 17 * rank)
    c_np, W_np, b_np, init_np = small_inputs(1234 + 17 * rank)
    x_pin = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16).pin_memory()
    xs = [x_pin.to(dev), x_pin.to(dev).flip(1).contiguous()]
    c = torch.from_numpy(c_np).to(dev)
    W = torch.from_numpy(W_np).to(dev)
    bvec = torch.from_numpy(b_np).to(dev)
    init = torch.from_numpy(init_np).to(dev)
    lam = torch.tensor(LAMBDA, device=dev)  # device tensor: no host copy inside graph capture
    outs = [torch.empty(B, S, D, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    fin = torch.empty(B, D, device=dev)

    def step(i):
        O.cheby_ema_forward(xs[i % 2], c, lambda_per_head=lam, gate_weight=W, gate_bias=bvec,
                            init_state=init, out=outs[i % 2], final_state=fin)

    stream = torch.cuda.Stream(dev)
    if args.profile_once:
        with torch.cuda.stream(stream):
            for i in range(4):  # 3 warm-up steps + the profiled one
                step(i)
        torch.cuda.synchronize()
        print("profile-once done, status", O.workspace_status())
        return
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(i)
    torch.cuda.synchronize()
    if O.workspace_status() != 0:
        raise RuntimeError("look-back timeout during warm-up")

    # CUDA graph of two steps (one per rotating buffer): removes host launch overhead
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step(0)
        step(1)
    torch.cuda.synchronize()
    # the kernels this step runs: the parked three-pass kernels (bf16 outputs:
    # p3_prep once, then per slab of sequences p3_agg, which parks u in L2 as
    # fp16 and forms the carries, and p3_outp, which reads u back; slabs of
    # about 16 MB of u on up to 5 streams), the three-pass kernels (p3_prep,
    # p3_agg, p3_carry, p3_out per group of sequences), or the grouped
    # single-evaluation kernel (one launch)
    path = O.forward_path(xs[0], c, lambda_per_head=lam, gate_weight=W, gate_bias=bvec, init_state=init)
    seq_u = ((S + 31) // 32) * 32 * D * 2
    slab = max(1, min(B, (16 << 20) // seq_u))
    nslab = (B + slab - 1) // slab
    groups = 2 if B >= 2 and (B // 2) * ((S + 31) // 32) >= 1024 else 1
    launches_per_step = {"grouped": 1, "parked": 1 + 2 * nslab}.get(path, 4 * groups)
    eval_passes = 1 if path in ("grouped", "parked") else 2  # evaluations of each element per step
    kernel_label = ("grp_fwd_kernel: one CTA per SM, each sequence owned by a group of CTAs, every element "
                    "evaluated once, local states parked in TMEM, tile aggregates exchanged through a ring in "
                    "global memory two rounds deep"
                    if path == "grouped" else
                    f"forward step: p3_prep_kernel + {nslab} slabs of {slab} sequence(s) on up to 5 streams, each "
                    "p3_agg_kernel (gate, u evaluated once and parked in L2 as fp16, chunk aggregates, carries by "
                    "span and sequence tickets) + p3_outp_kernel (EMA from the parked u, outputs, L2 lines dropped)"
                    if path == "parked" else
                    "forward step: p3_prep_kernel + p3_agg_kernel (gate + chunk aggregates) + p3_carry_kernel + "
                    "p3_out_kernel" + (", two halves of the batch on two streams" if groups == 2 else ""))

    # ---- clocks: sample through a loaded soak and the timed region ----
    try:
        gid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        gid = str(local)
    sampler = ClockSampler(gid)
    sampler.start()
    t_end = time.perf_counter() + args.soak_s
    with torch.cuda.stream(stream):
        while time.perf_counter() < t_end:
            for _ in range(50):
                graph.replay()
            stream.synchronize()

    # ---- timed region: K steps (graph replays of 2 steps each) ----
    K_ = args.steps
    reps = (K_ + 1) // 2
    K_eff = reps * 2
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(20_000_000)  # keep the launch queue ahead of the GPU
        ev0.record(stream)
        for _ in range(reps):
            graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    clocks = sampler.stop()
    value = world * B * S * K_eff / (ms / 1e3)

    # ---- the step (its launches), bracketed by CUDA events: each replay of
    # the two-step graph, and each step launched directly ----
    with torch.cuda.stream(stream):
        gevs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        torch.cuda._sleep(20_000_000)
        for a, bnd in gevs:
            a.record(stream)
            graph.replay()
            bnd.record(stream)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K_eff)]
        torch.cuda._sleep(200_000_000)  # enqueue every launch before the GPU reaches them
        for i, (a, bnd) in enumerate(evs):
            a.record(stream)
            step(i)
            bnd.record(stream)
    torch.cuda.synchronize()
    scan_avg = sum(a.elapsed_time(bnd) for a, bnd in gevs) / (2 * reps)
    scan_avg_direct = sum(a.elapsed_time(bnd) for a, bnd in evs) / K_eff
    elem = B * S * D
    scan_bytes = elem * 2 + elem * 2 + W.numel() * 4 + c.numel() * 4 + 2 * B * D * 4
    peak, peak_kind = peaks()
    achieved = scan_bytes / (scan_avg / 1e3) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        try:
            traffic = json.load(open(tp)).get("fwd_step_cfg2_bytes_per_step")
        except Exception:
            traffic = None

    # ---- end to end through the public API: pinned H2D, forward, D2H ----
    out_pin = torch.empty(B, S, D, dtype=torch.bfloat16).pin_memory()
    fin_pin = torch.empty(B, D).pin_memory()
    e2e_steps = max(3, min(K_eff, 20))
    init_pin = init.cpu().pin_memory()  # the carried state comes from the host too

    def e2e_step():  # the public host-buffer call (ossm_cheby_ema_fwd_host): copies in, forward, copies out
        O.cheby_ema_forward_host(x_pin, c, lambda_per_head=lam, gate_weight=W, gate_bias=bvec, init_state=init_pin,
                                 out_host=out_pin, final_host=fin_pin)

    with torch.cuda.stream(stream):
        for _ in range(2):
            e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = world * B * S * e2e_steps / (e2e_ms / 1e3)
    status = O.workspace_status()

    # ---- the opt-in single-evaluation kernel on the same step, for comparison ----
    single = single_eval_record(args, xs, c, lam, W, bvec, init, outs, fin, stream, scan_bytes, max_over_ranks)

    # ---- BASELINE configs[2] sharded over the ranks (the sequence-parallel design) ----
    seqpar = seqpar_record(args, world, rank, dev, stream, barrier, max_over_ranks)

    # ---- BASELINE configs[3], the reference's live Lion op, configs[4] ----
    ttt = ttt_record(args, world, dev, stream, barrier, max_over_ranks)
    lion = lion_record(args, world, dev, stream, barrier, max_over_ranks)
    lm = lm_record(args, world, dev, stream, barrier, max_over_ranks)

    # ---- CPU baseline on rank 0 at N=1 ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, nth, sample = cpu_sample(x_bits, c_np, W_np, b_np, init_np, np.asarray(LAMBDA, np.float32))
        cpu = {"value": v, "unit": "tokens/s", "cores": nth, "kind": "port", "sample": sample}

    if rank == 0:
        line = {
            "metric": "tokens/sec", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": K_eff, "warmup": max(args.warmup, 3), "ms_per_step": ms / K_eff,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 compute (bf16 in/out)", "data": "synthetic (seeded, BASELINE.json configs[1] shapes)",
            "config": config_dict(world),
            "gpu_launches": launches_per_step * K_eff,
            "hbm_gbs_step": (elem * 4 + B * D * 8) / (ms / K_eff / 1e3) / 1e9,
            "roofline": {"bound": "hbm", "kernel": kernel_label, "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                         "peak_kind": peak_kind, "bytes_per_step": scan_bytes,
                         "avg_step_ms": scan_avg, "timing": "CUDA events around each replay of the two-step graph",
                         "avg_step_ms_direct": scan_avg_direct,
                         "frac_direct": scan_bytes / (scan_avg_direct / 1e3) / 1e9 / peak},
            # the XU (MUFU) pipe: one reciprocal and one tanh per element in each evaluation pass
            "sfu": sfu_record(2 * eval_passes * elem, scan_avg, clocks, dev),
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": elem * 2 + B * D * 4,
                    "d2h_bytes_per_step": elem * 2 + B * D * 4},
            "clocks": clocks,
            "device_status": status,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        line["seqpar"] = seqpar
        line["single_eval"] = single
        line["cfg4"] = ttt
        line["lion"] = lion
        line["cfg5"] = lm
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.destroy_process_group()


def single_eval_record(args, xs, c, lam, W, bvec, init, outs, fin, stream, scan_bytes, max_over_ranks):
    """The same config-2 step through the opt-in single-evaluation grouped
    kernel (OSSM_F_SINGLE_EVAL: x read and every element evaluated once, one
    CTA per SM, tile aggregates exchanged through the workspace): per-step
    CUDA events (plain launches), max over ranks, and its largest output
    difference from the default three-pass step on the same inputs."""
    import torch
    import orthossm_b200 as O
    from orthossm_b200 import _lib as L
    from orthossm_b200.sdpc_kernel import _cheby_ema_forward
    kw = dict(lambda_per_head=lam, gate_weight=W, gate_bias=bvec, init_state=init)
    if O.forward_path(xs[0], c, extra_flags=L.OSSM_F_SINGLE_EVAL, **kw) != "grouped":
        return {"available": False}
    steps = max(4, min(args.steps, 20))

    def step(i):
        _cheby_ema_forward(xs[i % 2], c, out=outs[i % 2], final_state=fin, extra_flags=L.OSSM_F_SINGLE_EVAL, **kw)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(i)
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        torch.cuda._sleep(50_000_000)
        for i, (a, bnd) in enumerate(evs):
            a.record(stream)
            step(i)
            bnd.record(stream)
    torch.cuda.synchronize()
    us = max_over_ranks(sum(a.elapsed_time(bnd) for a, bnd in evs) / steps) * 1e3
    with torch.cuda.stream(stream):
        o1, f1 = _cheby_ema_forward(xs[0], c, extra_flags=L.OSSM_F_SINGLE_EVAL, **kw)
        o3, f3 = _cheby_ema_forward(xs[0], c, **kw)
    torch.cuda.synchronize()
    peak, _ = peaks()
    return {"available": True, "kernel": "grp_fwd_kernel (OSSM_F_SINGLE_EVAL)", "us_per_step": us,
            "tokens_per_s": B * S / (us * 1e-6), "hbm_frac": scan_bytes / (us * 1e-6) / 1e9 / peak,
            "max_abs_diff_vs_default_path": (o1.float() - o3.float()).abs().max().item(),
            "final_state_relerr_vs_default_path": ((f1 - f3).norm() / f3.norm()).item(),
            "device_status": O.workspace_status()}


def seqpar_record(args, world, rank, dev, stream, barrier, max_over_ranks):
    """BASELINE.json configs[2] on the same ranks: one sequence of 1,048,576
    tokens (bf16, per-head decays, no gate, zero initial state) sharded along
    the sequence, rank r holding tokens [r S/N, (r+1) S/N).  Each step is the
    shard's aggregate pass, one NCCL all-gather of the packed shard totals,
    the device fold and the shard's output pass (at N = 1, the unsharded
    forward).  Timed with CUDA events, max over ranks; strong scaling (the
    total work is fixed).  parity_ok compares every rank's outputs with the
    unsharded single-GPU forward of the whole sequence (to one bf16 step) and
    the final state with its final state (1e-4 relative)."""
    import torch
    import torch.distributed as dist
    import orthossm_b200 as O
    S_all = 1 << 20
    Sl = S_all // world
    g = torch.Generator(device=dev).manual_seed(99)
    x = torch.randn(1, S_all, D, generator=g, device=dev).to(torch.bfloat16)
    c = (torch.randn(1, H, K, HD, generator=g, device=dev) / torch.arange(1, K + 1, device=dev).view(1, 1, K, 1))
    lam = torch.tensor(LAMBDA, device=dev)
    xs = x[:, rank * Sl:(rank + 1) * Sl].contiguous()
    out = torch.empty_like(xs)
    if world > 1:
        fn = lambda: O.cheby_ema_forward_seqpar(xs, c, lambda_per_head=lam, out=out)  # noqa: E731
    else:
        fn = lambda: O.cheby_ema_forward(xs, c, lambda_per_head=lam, out=out)  # noqa: E731
    steps = max(3, min(args.steps, 20))
    ms_direct = _timed(fn, steps, args.warmup, stream, barrier, max_over_ranks)
    # the same step as one CUDA graph (its all-gather included): at 8 ranks a
    # step is ~0.1 ms of GPU work, near the host's own cost of enqueuing it
    ms = ms_direct
    graph = torch.cuda.CUDAGraph()
    captured = 1.0
    try:
        with torch.cuda.stream(stream):
            with torch.cuda.graph(graph, stream=stream):
                fn()
        torch.cuda.synchronize()
    except Exception:
        captured = 0.0
    barrier()
    if world > 1:  # every rank replays, or none
        flag = torch.tensor([captured], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        captured = float(flag.item())
    if captured:
        ms = _timed(graph.replay, steps, args.warmup, stream, barrier, max_over_ranks)
    del graph
    torch.cuda.synchronize()
    barrier()
    with torch.cuda.stream(stream):
        _, fin = fn()
        full, fin_full = O.cheby_ema_forward(x, c, lambda_per_head=lam)
    torch.cuda.synchronize()
    err = (out.float() - full[:, rank * Sl:(rank + 1) * Sl].float()).abs().max().item()
    ferr = ((fin - fin_full).norm() / fin_full.norm()).item()
    err, ferr = max_over_ranks(err), max_over_ranks(ferr)
    step_ms = ms / steps
    peak, kind = peaks()
    gbs = S_all * D * 4 / world / (step_ms / 1e3) / 1e9
    del x, full
    return {"workload": "cfg3: one sequence of 1,048,576 tokens, D=512, degree 8, bf16 in/out, per-head decays, "
                        "no gate, sequence-sharded over the ranks", "n_gpus": world, "scaling": "strong",
            "tokens_per_s": S_all / (step_ms / 1e3), "ms_per_sequence": step_ms, "steps": steps,
            "timing": "CUDA-graph replay" if captured else "plain calls",
            "ms_per_sequence_direct": ms_direct / steps,
            "parallelism": ("sequence-sharded x%d: shard aggregates, one NCCL all-gather of the packed shard "
                            "totals, device fold, shard outputs" % world) if world > 1 else "one GPU, unsharded",
            "hbm_gbs_per_gpu": gbs, "hbm_frac_per_gpu": gbs / peak, "peak_kind": kind,
            "parity_ok": bool(err <= 2 ** -7 and ferr < 1e-4), "max_abs_err_vs_unsharded": err,
            "final_state_relerr_vs_unsharded": ferr, "device_status": O.workspace_status()}


def sfu_record(ops, step_ms, clocks, dev):
    """MUFU operations per step against the XU pipe's 16 operations per SM
    per clock at the median SM clock sampled under load (a tanh.approx.f32
    throughput probe on this pool's B200s measured 4.61 T operations/s,
    148 x 16 x 1.95 GHz)."""
    import torch
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    mhz = (clocks or {}).get("sm_mhz") or (clocks or {}).get("sm_max_mhz") or 1965.0
    peak = nsm * 16 * mhz * 1e6
    achieved = ops / (step_ms / 1e3)
    return {"ops_per_step": ops, "achieved_tops": achieved / 1e12, "peak_tops": peak / 1e12,
            "frac": achieved / peak, "peak_kind": "16 per SM per clock at the sampled SM clock"}


def tensor_peak():
    """Sustained cuBLAS bf16 TF/s (the denominator for a kernel timed inside a long step)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        v = d.get("bf16_tflops_sustained") or d.get("bf16_tflops")
        if v:
            return float(v), "measured (sustained)"
    return 1400.0, "fallback (sustained)"


def ttt_record(args, world, dev, stream, barrier, max_over_ranks):
    """BASELINE.json configs[3] per GPU: W_pred MSE TTT with forget-gated Adam,
    B=4 x S=32768, 2048-token chunks, through the public ttt_wpred_adam (one
    native call per step: per chunk the forward, the tcgen05 W_pred gradient
    kernel and the fused reverse adjoint / gradient / Adam kernel).  Both
    bounds: tensor (the two W_pred products per token, 2 * 2 D^2 flops, against
    the sustained bf16 peak) and HBM (x read once in bf16 + the fp32 states
    written once).  Timed as plain calls and as CUDA-graph replays of the same
    call (the step is 80 dependent launches)."""
    import torch
    import orthossm_b200 as O
    Bl, Sl, chunk = 4, 32768, 2048
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(Bl, Sl, D, generator=g, device=dev).to(torch.bfloat16)
    c = torch.randn(Bl, H, K, HD, generator=g, device=dev) / torch.arange(1, K + 1, device=dev).view(1, 1, K, 1)
    Wp = torch.randn(D, D, generator=g, device=dev) * 0.02
    m, v = torch.zeros_like(c), torch.zeros_like(c)
    lam = torch.tensor(LAMBDA, device=dev)
    fn = lambda: O.ttt_wpred_adam(x, c, m, v, 0, Wp, lambda_per_head=lam, chunk=chunk)  # noqa: E731
    steps = max(3, min(args.steps, 20))
    ms_direct = _timed(fn, steps, args.warmup, stream, barrier, max_over_ranks) / steps
    # the same public call captured once in a CUDA graph (as the config-2 step
    # is): its 80 dependent launches replay without per-launch gaps
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fn()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            fn()
    torch.cuda.synchronize()
    ms = _timed(graph.replay, steps, args.warmup, stream, barrier, max_over_ranks) / steps
    del graph
    flops = Bl * Sl * 2 * 2 * D * D
    hbm_bytes = Bl * Sl * D * (2 + 4)
    tpk, tkind = tensor_peak()
    hpk, hkind = peaks()
    tf = flops / (ms / 1e3) / 1e12
    gbs = hbm_bytes / (ms / 1e3) / 1e9
    return {"workload": "cfg4: W_pred MSE TTT with forget-gated Adam, per GPU B=4 x S=32768, 2048-token chunks "
                        "(16 sequential chunk steps), W_pred 512x512, bf16 x, fp32 states",
            "n_gpus": world, "ms_per_step": ms, "tokens_per_s": world * Bl * Sl / (ms / 1e3), "steps": steps,
            "timing": "CUDA-graph replay of the public call (ms_per_step_direct: plain calls)",
            "ms_per_step_direct": ms_direct, "launches_per_chunk": 5, "chunks": Sl // chunk,
            "tensor": {"flops_per_step": flops, "achieved_tflops": tf, "peak": tpk, "peak_kind": tkind,
                       "frac": tf / tpk},
            "hbm": {"bytes_per_step": hbm_bytes, "achieved_gbs": gbs, "peak": hpk, "peak_kind": hkind,
                    "frac": gbs / hpk},
            "bound_note": "16 dependent chunk steps (each chunk's coefficients come from the previous chunk's "
                          "Adam step), 5 launches each: latency-bound, far from either roofline",
            "device_status": O.workspace_status()}


def lion_record(args, world, dev, stream, barrier, max_over_ranks):
    """The reference's live op: apply_cheby_rkv_v10 with its chunked Lion TTT
    (sdpc_kernel.py:2522-2606) at B=2 x S=65536, D=512, 8 heads, degree 8,
    256-token chunks, seq_threshold=0, the reference's defaults otherwise (LUT
    evaluation).  HBM bound: x read once (bf16) + the fp32 output written once."""
    import torch
    import orthossm_b200 as O
    Bl, Sl, chunk = 2, 65536, 256
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(Bl, Sl, D, generator=g, device=dev).to(torch.bfloat16)
    c0 = O.init_chebyshev_coefficients(Bl, H, K, HD, dev)
    c, mom = c0.clone(), torch.zeros_like(c0)

    def fn():
        c.copy_(c0)
        mom.zero_()
        return O.apply_cheby_rkv_v10(x, c, mom, n_heads=H, chunk_size=chunk, seq_threshold=0)

    steps = max(3, min(args.steps, 10))
    ms = _timed(fn, steps, args.warmup, stream, barrier, max_over_ranks) / steps
    hbm_bytes = Bl * Sl * D * (2 + 4)
    hpk, hkind = peaks()
    gbs = hbm_bytes / (ms / 1e3) / 1e9
    return {"workload": "reference live op apply_cheby_rkv_v10 (chunked Lion TTT): per GPU B=2 x S=65536, D=512, "
                        "8 heads, degree 8, 256-token chunks, seq_threshold=0, LUT evaluation",
            "n_gpus": world, "ms_per_step": ms, "tokens_per_s": world * Bl * Sl / (ms / 1e3), "steps": steps,
            "launches_per_step": 1,
            "hbm": {"bytes_per_step": hbm_bytes, "achieved_gbs": gbs, "peak": hpk, "peak_kind": hkind,
                    "frac": gbs / hpk},
            "bound_note": "256 dependent chunk steps per channel (each chunk's Lion update needs the previous "
                          "chunk's coefficients): one warp per channel walks them",
            "device_status": O.workspace_status()}


def lm_record(args, world, dev, stream, barrier, max_over_ranks):
    """BASELINE.json configs[4] per GPU: the config-5 LM forward (bf16) at
    B=2 x S=65536 (its cuBLAS GEMMs and flash-attention window are library
    kernels; the Cheby-RKV path is this package's)."""
    import torch
    from orthossm_b200.lm import OrthoLMConfig, OrthoSSMLM, n_params
    Bl, Sl = 2, 65536
    cfg = OrthoLMConfig()
    torch.manual_seed(42)
    model = OrthoSSMLM(cfg).to(dev, torch.bfloat16).eval()
    ids = torch.randint(0, cfg.vocab_size, (Bl, Sl), dtype=torch.int64, device=dev)
    states = model.fresh_states(Bl, dev, generator_seed=7)
    steps = max(3, min(args.steps, 5))
    with torch.no_grad():
        ms = _timed(lambda: model(ids, states), steps, args.warmup, stream, barrier, max_over_ranks) / steps
    npar = n_params(model)
    del model
    return {"workload": f"cfg5: config-5 LM forward, per GPU B={Bl} x S={Sl}, d_model 512, 8 heads, 6 V8 layers "
                        f"(Cheby-RKV + local attention window 512 + LayerNorm/Linear combine), vocab 32000, "
                        f"{npar / 1e6:.1f}M parameters (configs[4] says ~72M: the named layers hold 24.3M)",
            "n_gpus": world, "ms_per_step": ms, "tokens_per_s": world * Bl * Sl / (ms / 1e3), "steps": steps,
            "dtype": "bf16", "params": npar}


def run_lm(args):
    """Config-5 LM forward (bf16), weak scaling over ranks (batch-parallel)."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    import orthossm_b200 as O
    from orthossm_b200.lm import OrthoLMConfig, OrthoSSMLM, n_params

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    Bl, Sl = 2, 65536
    cfg = OrthoLMConfig()
    torch.manual_seed(42 + rank)
    model = OrthoSSMLM(cfg).to(dev, torch.bfloat16).eval()
    ids_pin = torch.randint(0, cfg.vocab_size, (Bl, Sl), dtype=torch.int64).pin_memory()
    ids = ids_pin.to(dev)
    states = model.fresh_states(Bl, dev, generator_seed=7 + rank)
    stream = torch.cuda.Stream(dev)

    def fwd(x):
        return model(x, states)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.no_grad(), torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            fwd(ids)
        torch.cuda.synchronize()
        try:
            gid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
        except Exception:
            gid = str(local)
        sampler = ClockSampler(gid)
        sampler.start()
        t_end = time.perf_counter() + args.soak_s  # loaded seconds for the clock samples
        while time.perf_counter() < t_end:
            fwd(ids)
            stream.synchronize()
        K_ = args.steps
        barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(K_):
            fwd(ids)
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(ev0.elapsed_time(ev1))
        clocks = sampler.stop()
        # the Cheby-EMA kernels alone: one call per layer on the same shapes
        h = torch.randn(Bl, Sl, cfg.d_model, device=dev).to(torch.bfloat16)
        lam = model.layers[0].lam(dev)
        gw, gb = model.layers[0].gate.weight.float(), model.layers[0].gate.bias.float()
        c0 = states[0].coeffs
        for _ in range(3):
            O.cheby_ema_forward(h, c0, lambda_per_head=lam, gate_weight=gw, gate_bias=gb)
        torch.cuda.synchronize()
        c0e, c1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0e.record(stream)
        for _ in range(cfg.n_layers * 5):
            O.cheby_ema_forward(h, c0, lambda_per_head=lam, gate_weight=gw, gate_bias=gb)
        c1e.record(stream)
        torch.cuda.synchronize()
        cheby_ms = c0e.elapsed_time(c1e) / 5
        # end to end: token ids from pinned host memory, forward, loss back to the host
        loss_pin = torch.empty((), dtype=torch.float32).pin_memory()
        xdev = torch.empty_like(ids)
        n_e2e = max(3, min(K_, 10))

        def e2e_step():
            xdev.copy_(ids_pin, non_blocking=True)
            logits = fwd(xdev)
            loss = F.cross_entropy(logits[:, :-1].reshape(-1, cfg.vocab_size).float(), xdev[:, 1:].reshape(-1))
            loss_pin.copy_(loss, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    if rank == 0:
        step_ms = ms / K_
        print(json.dumps({
            "metric": "tokens/sec", "value": world * Bl * Sl * K_ / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": K_, "warmup": max(args.warmup, 3), "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (token ids uniform over the vocab, random-init weights)",
            "config": {"workload": f"cfg5: config-5 LM forward, per GPU B={Bl} x S={Sl}, d_model 512, 8 heads, "
                                   f"6 V8 layers (Cheby-RKV + local attention window 512 + LayerNorm/Linear "
                                   f"combine), vocab 32000, {n_params(model) / 1e6:.1f}M parameters",
                       "global_batch": Bl * world, "seq_len": Sl, "parallelism": f"batch-sharded x{world}"},
            "cheby_ema_ms_per_step": cheby_ms, "cheby_ema_share": cheby_ms / step_ms,
            "e2e": {"value": world * Bl * Sl * n_e2e / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": Bl * Sl * 8, "d2h_bytes_per_step": 4},
            "clocks": clocks, "device_status": O.workspace_status(),
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _dist_setup(timeout_s=300):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s), device_id=dev)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        if world > 1:
            dist.barrier()
    return world, rank, local, dev, max_over_ranks, barrier


def _timed(fn, steps, warmup, stream, barrier, max_over_ranks):
    """warm-up, then `steps` calls between CUDA events on `stream`; max over ranks (ms)."""
    import torch
    with torch.cuda.stream(stream):
        for _ in range(max(warmup, 3)):
            fn()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
    return max_over_ranks(e0.elapsed_time(e1))


def run_cfg3(args):
    """One 1,048,576-token sequence, sequence-sharded over the ranks."""
    import torch
    import torch.distributed as dist
    import orthossm_b200 as O
    world, rank, local, dev, mor, barrier = _dist_setup()
    S_all = 1 << 20
    Sl = S_all // world
    g = torch.Generator().manual_seed(99)
    x = torch.randn(1, S_all, D, generator=g)[:, rank * Sl:(rank + 1) * Sl].to(torch.bfloat16).contiguous().to(dev)
    c = (torch.randn(1, H, K, HD, generator=g) / torch.arange(1, K + 1).view(1, 1, K, 1)).to(dev)
    lam = torch.tensor(LAMBDA, device=dev)
    out = torch.empty_like(x)
    stream = torch.cuda.Stream(dev)
    try:
        gid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        gid = str(local)
    sampler = ClockSampler(gid)
    sampler.start()
    if world > 1:
        fn = lambda: O.cheby_ema_forward_seqpar(x, c, lambda_per_head=lam, out=out)  # noqa: E731
    else:
        fn = lambda: O.cheby_ema_forward(x, c, lambda_per_head=lam, out=out)  # noqa: E731
    if args.profile_once:  # 3 warm-up calls + the profiled one, nothing timed
        sampler.stop()
        with torch.cuda.stream(stream):
            for _ in range(4):
                fn()
        torch.cuda.synchronize()
        if rank == 0:
            print("profile-once done, status", O.workspace_status())
        if world > 1:
            dist.destroy_process_group()
        return
    t_end = time.perf_counter() + args.soak_s
    with torch.cuda.stream(stream):
        while time.perf_counter() < t_end:
            fn()
            stream.synchronize()
    ms = _timed(fn, args.steps, args.warmup, stream, barrier, mor)
    clocks = sampler.stop()
    if rank == 0:
        step = ms / args.steps
        bytes_step = S_all * D * 4  # x read + out written, whole sequence
        peak, kind = peaks()
        print(json.dumps({
            "metric": "tokens/sec", "value": S_all / (step / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32 compute (bf16 in/out)",
            "data": "synthetic (seeded)",
            "config": {"workload": "cfg3: one sequence of 1,048,576 tokens, D=512, degree 8, bf16 in/out, "
                                   "per-head decays, no gate, sequence-sharded over the ranks",
                       "global_batch": 1, "seq_len": S_all,
                       "parallelism": f"sequence-sharded x{world} (one NCCL all-gather of shard totals)"},
            "hbm_gbs_per_gpu": bytes_step / world / (step / 1e3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": bytes_step / world / (step / 1e3) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": bytes_step / world / (step / 1e3) / 1e9 / peak, "peak_kind": kind},
            "clocks": clocks, "device_status": O.workspace_status(),
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_cfg4(args):
    """W_pred Adam TTT, B=4 x S=32768 per GPU, 2048-token chunks."""
    import torch
    import torch.distributed as dist
    import orthossm_b200 as O
    world, rank, local, dev, mor, barrier = _dist_setup()
    Bl, Sl, chunk = 4, 32768, 2048
    g = torch.Generator().manual_seed(7 + rank)
    x = torch.randn(Bl, Sl, D, generator=g).to(torch.bfloat16).to(dev)
    c = (torch.randn(Bl, H, K, HD, generator=g) / torch.arange(1, K + 1).view(1, 1, K, 1)).to(dev)
    Wp = (torch.randn(D, D, generator=g) * 0.02).to(dev)
    m, v = torch.zeros_like(c), torch.zeros_like(c)
    lam = torch.tensor(LAMBDA, device=dev)
    stream = torch.cuda.Stream(dev)
    fn = lambda: O.ttt_wpred_adam(x, c, m, v, 0, Wp, lambda_per_head=lam, chunk=chunk)  # noqa: E731
    if args.profile_once:  # 3 warm-up calls + the profiled one, nothing timed
        with torch.cuda.stream(stream):
            for _ in range(4):
                fn()
        torch.cuda.synchronize()
        if rank == 0:
            print("profile-once done, status", O.workspace_status())
        if world > 1:
            dist.destroy_process_group()
        return
    try:
        gid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        gid = str(local)
    sampler = ClockSampler(gid)
    sampler.start()
    t_end = time.perf_counter() + args.soak_s
    with torch.cuda.stream(stream):
        while time.perf_counter() < t_end:
            fn()
            stream.synchronize()
    ms_direct = _timed(fn, args.steps, args.warmup, stream, barrier, mor)
    graph = torch.cuda.CUDAGraph()  # the same call as one CUDA graph (80 dependent launches per step)
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            fn()
    torch.cuda.synchronize()
    ms = _timed(graph.replay, args.steps, args.warmup, stream, barrier, mor)
    del graph
    clocks = sampler.stop()
    if rank == 0:
        step = ms / args.steps
        flops = Bl * Sl * 2 * 2 * D * D  # W_pred s and W_pred^T r per token
        print(json.dumps({
            "metric": "tokens/sec", "value": world * Bl * Sl / (step / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 compute (bf16 x), fp32 state, W_pred products on tcgen05 (TF32 s.G, bf16 hi+lo x.W_pred)",
            "data": "synthetic (seeded)",
            "config": {"workload": "cfg4: W_pred MSE TTT with forget-gated Adam, per GPU B=4 x S=32768, "
                                   "2048-token chunks (16 sequential steps), W_pred 512x512",
                       "global_batch": Bl * world, "seq_len": Sl, "parallelism": f"batch-sharded x{world}"},
            "gemm_tflops": flops / (step / 1e3) / 1e12,
            "timing": "CUDA-graph replay of the public call", "ms_per_step_direct": ms_direct / args.steps,
            "clocks": clocks, "device_status": O.workspace_status(),
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_lion(args):
    """The reference's live op (apply_cheby_rkv_v10 with its Lion TTT) as the
    main line: the `lion` record's workload, per GPU, weak scaling."""
    import torch
    import torch.distributed as dist
    import orthossm_b200 as O
    world, rank, local, dev, mor, barrier = _dist_setup()
    stream = torch.cuda.Stream(dev)
    if args.profile_once:  # 3 warm-up calls + the profiled one, nothing timed
        g = torch.Generator(device=dev).manual_seed(11)
        x = torch.randn(2, 65536, D, generator=g, device=dev).to(torch.bfloat16)
        c0 = O.init_chebyshev_coefficients(2, H, K, HD, dev)
        with torch.cuda.stream(stream):
            for _ in range(4):
                O.apply_cheby_rkv_v10(x, c0.clone(), torch.zeros_like(c0), n_heads=H, chunk_size=256,
                                      seq_threshold=0)
        torch.cuda.synchronize()
        if rank == 0:
            print("profile-once done")
    else:
        rec = lion_record(args, world, dev, stream, barrier, mor)
        if rank == 0:
            print(json.dumps({
                "metric": "tokens/sec", "value": rec["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
                "steps": rec["steps"], "warmup": max(args.warmup, 3), "ms_per_step": rec["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32 compute (bf16 x, fp32 out rounded to bf16 as the reference does)",
                "data": "synthetic (seeded)",
                "config": {"workload": rec["workload"], "global_batch": 2 * world, "seq_len": 65536,
                           "parallelism": f"batch-sharded x{world}"},
                "roofline": dict(rec["hbm"], bound="hbm", unit="GB/s", achieved=rec["hbm"]["achieved_gbs"]),
                "device_status": rec["device_status"]}), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "cfg5":
        run_lm(args)
    elif args.workload == "cfg3":
        run_cfg3(args)
    elif args.workload == "cfg4":
        run_cfg4(args)
    elif args.workload == "lion":
        run_lion(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
