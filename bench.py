#!/usr/bin/env python
"""Headline benchmark: bidirectional Mamba-3 trapezoidal scan, forward + backward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl m3|reference]

One step = the fused bidirectional forward scan (with backward checkpoints) and
the analytic backward of one layer of the config-4 stack (the config-1/2 layer
shape: L=64, d_inner=1536, d_state=32 with 16 rotational + 16 tracking lanes,
bf16 delta/u/B/C/dy, fp32 state) over config 4's global batch of 8192 rows
split evenly across the N GPUs ("strong" scaling), plus -- on more than one GPU
-- one NCCL all-reduce of the scan-parameter gradients (the data-parallel
exchange of config 4).  Inputs (>= 0.6 GB/GPU) exceed the 126 MB L2, so no
flush is needed between steps.

The JSON line also carries the end-to-end leg (host buffers, H2D/D2H copies in
the timed region), the roofline of the dominant kernel (the backward), the CPU
baseline (the oracle port of the reference algorithm on the host cores), the
clocks sampled during the timed region, and the config-3 recurrent-step
rollout measurement.

``--impl reference`` times the reference algorithm (the CPU oracle port; the
reference is pure Python/PyTorch and has no GPU path outside Triton) on the
host cores, on rank 0 only.
"""

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "scan fwd+bwd Gtokens/s (% HBM peak); recurrent-step rollout node-steps/s/GPU"
UNIT = "Gtokens/s"
# config 2 / 4 shape (per GPU)
GLOBAL_B, L, D, N, N_ROT, MIMO_P = 8192, 64, 1536, 32, 16, 4
B_RANK = GLOBAL_B     # rows per GPU; set from the world size in main()
# algorithmic HBM bytes per token at this boundary (bf16 delta/u/B/C/dy, fp32 y)
FWD_BYTES_PER_TOKEN = 2 * 2 * D + 2 * 2 * N + 4 * D            # 12416
BWD_BYTES_PER_TOKEN = 3 * 2 * D + 2 * 2 * N + 2 * 2 * D + 2 * 2 * N  # 15616
FALLBACK_HBM_GBS = 6650.0


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def _profile_value(key):
    """A figure of the committed ncu summary of the backward kernel (or None)."""
    path = os.path.join(REPO, "profiles", "scan_bwd_c2_traffic.txt")
    try:
        for line in open(path):
            if line.startswith(key + ":"):
                return float(line.split(":")[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock/throttle sampling (every 50 ms, timestamped).

    Started before the warm-up so that it is running when the timed region
    begins; ``stop(t0, t1)`` keeps only the samples whose timestamps fall in
    the host wall-clock window [t0, t1] of the timed region.
    """
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "50"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self, t0=None, t1=None):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                if t0 is not None and not (t0 - 0.05 <= ts <= t1 + 0.05):
                    continue
                sm.append(float(parts[2]))
                mx.append(float(parts[3]))
                pw.append(float(parts[4]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[6:10]):
                if v.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "power_w_max": max(pw) if pw else None, "samples": len(sm)}


def cpu_scan_rate(rows, min_seconds, max_reps=None):
    """Reference algorithm (oracle port, fp32 autograd) on the host: tokens/s."""
    import torch
    import oracle as O
    from redpanda_b200.synthetic import ScanShape, make_scan_inputs
    torch.set_num_threads(os.cpu_count() or 1)
    inp = make_scan_inputs(ScanShape(rows, L, D, N, N - N_ROT, MIMO_P), seed=123)
    def once():
        O.scan_with_grads(inp["delta"], inp["u"], inp["Bc"], inp["Cc"], inp["A_real"],
                          inp["A_imag"], inp["track"], inp["dy"], bidir=True)
    once()
    reps, t0 = 0, time.perf_counter()
    while True:
        once()
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or (max_reps and reps >= max_reps):
            break
    return rows * L * reps / el, reps, el


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    from redpanda_b200.synthetic import ScanShape, make_scan_inputs
    import oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    rows = 4
    inp = make_scan_inputs(ScanShape(rows, L, D, N, N - N_ROT, MIMO_P), seed=123)
    def once():
        O.scan_with_grads(inp["delta"], inp["u"], inp["Bc"], inp["Cc"], inp["A_real"],
                          inp["A_imag"], inp["track"], inp["dy"], bidir=True)
    for _ in range(args.warmup):
        once()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        once()
    el = time.perf_counter() - t0
    v = rows * L * args.steps / el / 1e9
    sample = (f"{rows} rows x L={L} of the config-2 shape per step (bidirectional fwd+bwd, "
              f"fp32 PyTorch autograd of the reference chunked scan)")
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "c2/c4: bidirectional scan fwd+bwd of one layer of the "
                                   "config-4 stack (config-2 layer shape), global batch split "
                                   "over the GPUs, scan-parameter grad all-reduce when N>1",
                       "batch_per_gpu": max(1, GLOBAL_B // max(1, world)),
                       "global_batch": GLOBAL_B, "seq_len": L, "d_inner": D, "d_state": N,
                       "n_rot": N_ROT, "mimo_p": MIMO_P,
                       "reference_sample_rows_per_step": rows,
                       "note": "the reference algorithm runs on the host cores on a bounded "
                               "sample of the workload (tokens/s is a rate; rows are "
                               "independent)"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def make_inputs(dev, seed):
    import torch
    import torch.nn.functional as F
    g = torch.Generator(dev).manual_seed(seed)
    bf = torch.bfloat16
    n_tr = N - N_ROT
    x = {
        "delta": F.softplus(torch.randn(B_RANK, L, D, device=dev, generator=g) * 0.5 - 2).to(bf),
        "u": torch.randn(B_RANK, L, D, device=dev, generator=g).to(bf),
    }
    def bc():
        raw = torch.randn(B_RANK, L, N * MIMO_P, device=dev, generator=g) / math.sqrt(N)
        raw = raw * torch.rsqrt(raw.pow(2).mean(-1, keepdim=True) + 1e-5)
        return raw.view(B_RANK, L, N, MIMO_P).sum(-1).to(bf)
    x["Bc"], x["Cc"] = bc(), bc()
    x["dy"] = torch.randn(B_RANK, L, D, device=dev, generator=g).to(bf)
    ar = -torch.exp(torch.randn(D, N_ROT, device=dev, generator=g) * 0.5)
    ai = (torch.rand(D, N_ROT, device=dev, generator=g) * 2 - 1) * math.pi
    tk = torch.tanh(torch.randn(D, n_tr, device=dev, generator=g))
    return x, ar, ai, tk


class MultiRank:
    """Barrier and max-over-ranks timing for the legs that every rank runs."""

    def __init__(self, rank, world, local, dev):
        self.rank, self.world, self.local, self.dev = rank, world, local, dev

    def barrier(self):
        import torch
        import torch.distributed as dist
        if self.world > 1:
            dist.barrier(device_ids=[self.local])
        torch.cuda.synchronize(self.dev)

    def max(self, v):
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return v
        t = torch.tensor([v], device=self.dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, fn):
        """ms of fn() on this rank's stream between barriers, max over ranks."""
        import torch
        stream = torch.cuda.current_stream(self.dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.barrier()
        e0.record(stream)
        fn()
        e1.record(stream)
        self.barrier()
        return self.max(e0.elapsed_time(e1))


def run_m3(args):
    import torch
    import torch.distributed as dist
    from redpanda_b200 import scan as S
    from redpanda_b200.scan import ScanPlan, pad_params

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    global B_RANK
    B_RANK = args.batch if args.batch else max(1, GLOBAL_B // world)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    if not S.HAS_M3:
        raise RuntimeError("m3 library or sm_100 device unavailable")

    x, ar, ai, tk = make_inputs(dev, 1000 + rank)
    Ar_p, Ai_p, Tk_p = (t.contiguous() for t in pad_params(ar, ai, tk, N_ROT, N, D, dev))
    bf = torch.bfloat16
    plan = ScanPlan(B_RANK, L, D, N, N_ROT, bf, bf, S.M3_DIR_BIDIR)
    y = torch.empty(B_RANK, L, D, device=dev)
    ckpt = torch.empty(plan.ckpt_floats(), device=dev)
    ws = torch.empty(plan.workspace_bytes(), device=dev, dtype=torch.uint8)
    gd, gu = torch.empty_like(x["delta"]), torch.empty_like(x["u"])
    gB, gC = torch.empty_like(x["Bc"]), torch.empty_like(x["Cc"])
    gflat = torch.empty(3, D, N, device=dev)   # dA_real, dA_imag, dtrack: one all-reduce
    stream = torch.cuda.current_stream(dev)
    kernel_events = []

    def step(inputs, timed_bwd=False):
        if timed_bwd:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record(stream)
        plan.forward(inputs["delta"], inputs["u"], inputs["Bc"], inputs["Cc"], Ar_p, Ai_p, Tk_p,
                     y, ckpt)
        if timed_bwd:
            ev[1].record(stream)
        plan.backward(inputs["delta"], inputs["u"], inputs["Bc"], inputs["Cc"], Ar_p, Ai_p, Tk_p,
                      inputs["dy"], ckpt, gd, gu, gB, gC, gflat[0], gflat[1], gflat[2], ws)
        if timed_bwd:
            ev[2].record(stream)
            kernel_events.append(ev)
        if world > 1:
            dist.all_reduce(gflat)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident leg
    clk = ClockSampler(local)
    for _ in range(args.warmup):
        step(x)
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    t0.record(stream)
    for _ in range(args.steps):
        step(x, timed_bwd=True)
    t1.record(stream)
    barrier()
    clocks = clk.stop(wall0, time.time())
    ms = max_over_ranks(t0.elapsed_time(t1))
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in kernel_events)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in kernel_events)
    tokens = world * B_RANK * L * args.steps
    value = tokens / (ms / 1e3) / 1e9

    # ---- end-to-end leg: the same calls on host buffers.  Every step copies its
    # inputs in from pinned host memory and ALL of its results out -- y (fp32),
    # d_delta and d_u (bf16), d_Bc and d_Cc (bf16) and the parameter grads --
    # streaming the step's rows in NSUB sub-batches through the same public calls
    # (ScanPlan.forward/backward on row slices).  The host->device copy of
    # sub-batch g+1 runs on one copy stream into the second of two device buffer
    # sets while sub-batch g computes; the device->host copies of sub-batch g's
    # results run on a second copy stream behind its compute (PCIe is full
    # duplex, so both directions overlap the compute and each other).  The
    # parameter grads of the sub-batches are summed on the device and read back
    # once per step.  All copies are inside the timed region.
    nsub = args.e2e_sub if B_RANK % args.e2e_sub == 0 and B_RANK >= 16 * args.e2e_sub else 1
    bsub = B_RANK // nsub
    splan = plan if nsub == 1 else ScanPlan(bsub, L, D, N, N_ROT, bf, bf, S.M3_DIR_BIDIR)
    sckpt = ckpt if nsub == 1 else torch.empty(splan.ckpt_floats(), device=dev)
    sws = ws if nsub == 1 else torch.empty(splan.workspace_bytes(), device=dev, dtype=torch.uint8)
    gsub = torch.empty_like(gflat)
    # the parameter grads of a step are summed into one of two device buffers
    # (alternating steps) and read back on a stream of their own, so the
    # compute stream never queues behind a device->host copy
    gsum = [torch.empty_like(gflat) for _ in range(2)]
    host = {k: v.cpu().pin_memory() for k, v in x.items()}
    dbufs = [{k: torch.empty((bsub,) + tuple(v.shape[1:]), dtype=v.dtype, device=dev)
              for k, v in x.items()} for _ in range(2)]
    outs_dev = {"y": y, "d_delta": gd, "d_u": gu, "d_Bc": gB, "d_Cc": gC}
    outs_host = {k: torch.empty(v.shape, dtype=v.dtype).pin_memory() for k, v in outs_dev.items()}
    gout = [torch.empty(gflat.shape, dtype=gflat.dtype).pin_memory() for _ in range(2)]
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = sum(v.numel() * v.element_size() for v in outs_host.values()) + \
        gout[0].numel() * gout[0].element_size()
    copy_stream = torch.cuda.Stream(dev)
    out_stream = torch.cuda.Stream(dev)
    grad_stream = torch.cuda.Stream(dev)
    summed = [torch.cuda.Event() for _ in range(2)]
    gread = [torch.cuda.Event() for _ in range(2)]
    gread_used = [False, False]
    nstep = [0]
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(nsub)]
    returned = [torch.cuda.Event() for _ in range(nsub)]
    returned_used = [False] * nsub

    def h2d_copy(gi):
        slot, j = gi & 1, gi % nsub
        if gi >= 2:
            copy_stream.wait_event(consumed[slot])   # sub-batch gi-2 is done with this set
        with torch.cuda.stream(copy_stream):
            for k in host:
                dbufs[slot][k].copy_(host[k][j * bsub:(j + 1) * bsub], non_blocking=True)
            copied[slot].record(copy_stream)

    def d2h_copy(j):
        rows = slice(j * bsub, (j + 1) * bsub)
        out_stream.wait_event(computed[j])
        with torch.cuda.stream(out_stream):
            for k, v in outs_dev.items():
                outs_host[k][rows].copy_(v[rows], non_blocking=True)
            returned[j].record(out_stream)
        returned_used[j] = True

    def sub_step(inp, j):
        rows = slice(j * bsub, (j + 1) * bsub)
        if returned_used[j]:
            stream.wait_event(returned[j])   # the previous step's rows j are on the host
        splan.forward(inp["delta"], inp["u"], inp["Bc"], inp["Cc"], Ar_p, Ai_p, Tk_p, y[rows],
                      sckpt)
        splan.backward(inp["delta"], inp["u"], inp["Bc"], inp["Cc"], Ar_p, Ai_p, Tk_p,
                       inp["dy"], sckpt, gd[rows], gu[rows], gB[rows], gC[rows],
                       gsub[0], gsub[1], gsub[2], sws)
        computed[j].record(stream)
        par = nstep[0] & 1
        acc = gsum[par]
        if j == 0:
            if gread_used[par]:
                stream.wait_event(gread[par])   # read back two steps ago
            acc.copy_(gsub)
        else:
            acc.add_(gsub)
        if j == nsub - 1:
            if world > 1:
                dist.all_reduce(acc)
            summed[par].record(stream)
            grad_stream.wait_event(summed[par])
            with torch.cuda.stream(grad_stream):
                gout[par].copy_(acc, non_blocking=True)
                gread[par].record(grad_stream)
            gread_used[par] = True
            nstep[0] += 1

    def e2e_run(k_steps, start_event=None):
        if start_event is not None:
            copy_stream.wait_event(start_event)
            out_stream.wait_event(start_event)
        total = k_steps * nsub
        h2d_copy(0)
        for gi in range(total):
            slot, j = gi & 1, gi % nsub
            if gi + 1 < total:
                h2d_copy(gi + 1)
            stream.wait_event(copied[slot])
            sub_step(dbufs[slot], j)
            consumed[slot].record(stream)
            d2h_copy(j)
        for j in range(nsub):   # the timed region ends when every result is on the host
            stream.wait_event(returned[j])
        for par in range(2):
            if gread_used[par]:
                stream.wait_event(gread[par])

    e2e_run(max(1, args.warmup))
    barrier()
    t0.record(stream)
    e2e_run(args.steps, start_event=t0)
    t1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1))
    e2e_value = tokens / (e2e_ms / 1e3) / 1e9
    # the host copies hold the device results bit for bit (last step's rows)
    last = (nstep[0] - 1) & 1
    e2e_check = (all(torch.equal(outs_host[k], v.cpu()) for k, v in outs_dev.items())
                 and torch.equal(gout[last], gsum[last].cpu()))

    # every rank runs the config-3 rollouts on its share of the rows and the
    # config-4 model-level training step on its share of the global batch (in
    # the same order, so their barriers and collectives pair up); the
    # one-GPU configurations (the sequence-length sweep, the per-config lines)
    # run on rank 0 alone afterwards, with no collective
    mp = MultiRank(rank, world, local, dev)
    step_info = run_step_rollout(dev, args, mp) if args.rollout else None
    model_info = run_model_rollout(dev, args, mp) if args.rollout else None
    train_info = run_model_train(dev, args, mp) if args.model_train else None
    sweep_info = run_l_sweep(dev, args) if (args.sweep and rank == 0) else None
    configs_info = run_configs(dev, args, clocks) if (args.configs and rank == 0) else None
    eval_info = run_model_eval(dev, args) if (args.model_train and rank == 0) else None
    node_info = (run_search_nodes(dev, args) if (args.rollout and args.search and rank == 0)
                 else None)

    if rank == 0:
        peak, peak_kind = _peaks()
        bwd_bytes = BWD_BYTES_PER_TOKEN * B_RANK * L
        achieved = bwd_bytes / (bwd_ms / 1e3) / 1e9
        tpt = _profile_value("dram_bytes_per_token")
        ipt = _inst_per_token().get("c2_bwd_bidir")
        mhz = clocks.get("sm_mhz") or 1965.0
        issue_frac = (ipt * B_RANK * L / (bwd_ms / 1e3) / (SMS * SCHEDULERS * mhz * 1e6)
                      if ipt else None)
        fma = _profile_value("fma_pipe_active_pct")
        cpu = None
        if world == 1 and not args.no_cpu:
            rate, reps, el = cpu_scan_rate(4, args.cpu_seconds)
            cpu = {"value": rate / 1e9, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                   "sample": f"{reps} x 4 rows x L={L} of the config-2 shape, bidirectional "
                             f"fwd+bwd, fp32 reference algorithm (oracle port), {el:.1f} s"}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if not args.batch else "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "c2/c4: bidirectional scan fwd+bwd of one layer of the "
                                   "config-4 stack (config-2 layer shape), global batch split "
                                   "over the GPUs, scan-parameter grad all-reduce when N>1",
                       "batch_per_gpu": B_RANK, "global_batch": B_RANK * world, "seq_len": L,
                       "d_inner": D, "d_state": N, "n_rot": N_ROT, "mimo_p": MIMO_P,
                       "parallelism": f"dp{world}", "l2": "inputs larger than L2 (no flush)",
                       "compute": "fp32 state/accumulation, bf16 inputs and input grads"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms / args.steps,
                    "sub_batches": nsub,
                    "returned": "y (fp32), d_delta, d_u, d_Bc, d_Cc (bf16), parameter grads",
                    "host_results_equal_device": e2e_check},
            "gpu_launches": 4 * args.steps,
            "roofline": {"bound": "hbm", "kernel": "scan_bwd (m3_scan_bwd)",
                         "achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": achieved / peak,
                         "traffic": (tpt * B_RANK * L) if tpt else None,
                         "algorithmic_bytes": bwd_bytes, "ms_per_launch": bwd_ms,
                         "fma_pipe_active_frac": (fma / 100.0) if fma is not None else None,
                         "issue_frac": issue_frac,
                         "note": "compute-bound: instruction issue, not HBM, limits the scan; "
                                 "issue_frac = the backward's warp instructions per token (ncu, "
                                 "profiles/scan_inst_per_token.txt) x tokens / its event time / "
                                 "(148 SMs x 4 schedulers x the sampled SM clock)"},
            "kernels_ms": {"scan_fwd_bidir": fwd_ms, "scan_bwd_bidir": bwd_ms,
                           "tokens_per_launch": B_RANK * L},
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        if step_info is not None:
            line["step_rollout"] = step_info
        if model_info is not None:
            line["model_rollout"] = model_info
        if train_info is not None:
            line["model_train"] = train_info
        if configs_info is not None:
            line["configs"] = configs_info
        if eval_info is not None:
            line["model_eval"] = eval_info
        if node_info is not None:
            line["search_nodes"] = node_info
        if sweep_info is not None:
            line["l_sweep"] = {"workload": "c4 sequence-length sweep: bidirectional scan "
                                           "fwd+bwd, c2 layer shape, bf16, 1 GPU",
                               "points": sweep_info}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_step_rollout(dev, args, mp):
    """Config 3: 12-layer lockstep rollout of B=8192 states, 32 steps, re-anchored
    every 8 steps by a full L=64 scan with return_state (recurrence kernels only;
    per-layer token inputs are synthetic).  The rows are split evenly over the
    ranks (independent rollouts, no communication); times are max over ranks."""
    import torch
    from redpanda_b200 import scan as S
    from redpanda_b200.scan import ScanPlan, pad_params
    layers, Ds, Ns, nr = args.rollout_layers, 1024, 32, 24
    Bg = args.rollout_batch
    Bs = max(1, Bg // mp.world)
    g = torch.Generator(dev).manual_seed(7 + mp.rank)
    params = []
    for _ in range(layers):
        ar = -torch.exp(torch.randn(Ds, nr, device=dev, generator=g) * 0.5)
        ai = (torch.rand(Ds, nr, device=dev, generator=g) * 2 - 1) * math.pi
        tk = torch.tanh(torch.randn(Ds, Ns - nr, device=dev, generator=g))
        params.append(tuple(t.contiguous() for t in pad_params(ar, ai, tk, nr, Ns, Ds, dev)))
    h = [torch.zeros(Bs, Ds, Ns, device=dev) for _ in range(layers)]
    db = [torch.zeros(Bs, Ds, Ns, device=dev) for _ in range(layers)]
    bf = torch.bfloat16
    seq = {"delta": torch.nn.functional.softplus(
               torch.randn(Bs, 64, Ds, device=dev, generator=g) * 0.5 - 2).to(bf),
           "u": torch.randn(Bs, 64, Ds, device=dev, generator=g).to(bf),
           "Bc": torch.randn(Bs, 64, Ns, device=dev, generator=g).to(bf),
           "Cc": torch.randn(Bs, 64, Ns, device=dev, generator=g).to(bf)}
    yseq = torch.empty(Bs, 64, Ds, device=dev)
    tok = {k: v[:, 0].float().contiguous() for k, v in seq.items()}
    ystep = torch.empty(Bs, Ds, device=dev)
    plan = ScanPlan(Bs, 64, Ds, Ns, nr, bf, bf, S.M3_DIR_FWD)
    lib = S._lib.load()
    sdesc = S.StepDesc(Bs, Ds, Ns, nr, S.M3_F32, S.M3_F32)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    def anchor():
        for li in range(layers):
            plan.forward(seq["delta"], seq["u"], seq["Bc"], seq["Cc"], *params[li], yseq,
                         None, h[li], db[li])

    def one_step():
        for li in range(layers):
            ar, ai, tk = params[li]
            S._lib.check(lib.m3_step(sdesc, h[li].data_ptr(), db[li].data_ptr(),
                                     tok["delta"].data_ptr(), tok["u"].data_ptr(),
                                     tok["Bc"].data_ptr(), tok["Cc"].data_ptr(), ar.data_ptr(),
                                     ai.data_ptr(), tk.data_ptr(), ystep.data_ptr(), sh))

    def rollout():
        for s in range(32):
            if s % 8 == 0:
                anchor()
            one_step()

    # factored state: h in place, [delta*u | B] factors ping-ponged per layer
    fac = [[torch.zeros(Bs, Ds + Ns, device=dev) for _ in range(2)] for _ in range(layers)]
    fdesc = S.StepDesc(Bs, Ds, Ns, nr, S.M3_F32, S.M3_F32)

    def one_step_factored(parity):
        for li in range(layers):
            ar, ai, tk = params[li]
            S._lib.check(lib.m3_step_factored(
                fdesc, h[li].data_ptr(), fac[li][parity].data_ptr(),
                fac[li][parity ^ 1].data_ptr(), tok["delta"].data_ptr(), tok["u"].data_ptr(),
                tok["Bc"].data_ptr(), tok["Cc"].data_ptr(), ar.data_ptr(), ai.data_ptr(),
                tk.data_ptr(), ystep.data_ptr(), sh))

    def steps32():
        for _ in range(32):
            one_step()

    def fsteps32():
        for s_ in range(32):
            one_step_factored(s_ & 1)

    rollout()
    fsteps32()
    total_ms = mp.timed(rollout)
    steps_ms = mp.timed(steps32)
    fsteps_ms = mp.timed(fsteps32)
    peak, kind = _peaks()
    rows = Bs * mp.world
    state_bytes = layers * Bs * Ds * Ns * 16          # per rank and node-step batch
    gbs = state_bytes / (steps_ms / 32 / 1e3) / 1e9
    fgbs = state_bytes / 2 / (fsteps_ms / 32 / 1e3) / 1e9
    return {
        "workload": f"c3: {layers} layers, B={rows} ({Bs} per GPU), D=1024, N=32 (24 rot + 8 "
                    "track), 32 steps, re-anchor every 8 steps by an L=64 scan with return_state",
        "n_gpus": mp.world,
        "node_steps_per_s": rows * 32 / (total_ms / 1e3),
        "ms_per_rollout": total_ms,
        "step_only_node_steps_per_s": rows * 32 / (steps_ms / 1e3),
        "step_ms_per_node_step_batch": steps_ms / 32,
        "step_hbm_gbs_per_gpu": gbs,
        "step_hbm_frac": gbs / peak,
        "step_algorithmic_bytes_per_gpu": state_bytes,
        "factored_step_node_steps_per_s": rows * 32 / (fsteps_ms / 1e3),
        "factored_step_hbm_gbs_per_gpu": fgbs,
        "factored_step_hbm_frac": fgbs / peak,
        "gpu_launches": 32 * layers + 4 * layers,
        "note": "recurrence kernels only; the projection GEMMs of Mamba.step are not included; "
                "times are max over ranks",
    }


# Issue roofline of the scan kernels: 148 SMs x 4 warp schedulers, one warp
# instruction per scheduler and clock.  The per-token warp-instruction counts
# come from the committed ncu summary (smsp__inst_executed.sum of each kernel
# variant / tokens of its launch).
SMS, SCHEDULERS = 148, 4


def _inst_per_token():
    out = {}
    path = os.path.join(REPO, "profiles", "scan_inst_per_token.txt")
    try:
        for line in open(path):
            if ":" in line and not line.startswith("#"):
                k, v = line.split(":", 1)
                out[k.strip()] = float(v)
    except OSError:
        pass
    return out


def run_configs(dev, args, clocks):
    """One line per BASELINE configuration on one GPU (device-resident inputs,
    CUDA events, a few warm-up launches):
      c0         causal fwd+bwd, fp32, B=8, L=64, D=256, N=16 (12 rot + 4 track),
                 with the reference algorithm on the host cores on the same
                 inputs (config 0 is the reference's CPU-runnable case)
      c1_fwd     bidirectional forward only (inference, no checkpoints), bf16,
                 B=1024, L=64, D=1536, N=32 (16 rot + 16 track)
      c2_bidir   bidirectional fwd (with checkpoints) + bwd + reductions, c1 shape
      c2_causal  causal fwd + bwd + reductions, c1 shape
    Each line: tokens/s, ms per step, the HBM fraction of its algorithmic bytes
    and, where the ncu instruction counts are committed, the fraction of the
    issue roofline (148 SMs x 4 schedulers x the median SM clock sampled in
    the timed region of the headline)."""
    import torch
    from redpanda_b200 import scan as S
    from redpanda_b200.scan import ScanPlan, pad_params
    from redpanda_b200.synthetic import ScanShape, make_scan_inputs
    peak, _ = _peaks()
    ipt = _inst_per_token()
    mhz = (clocks or {}).get("sm_mhz") or 1965.0
    issue_peak = SMS * SCHEDULERS * mhz * 1e6
    stream = torch.cuda.current_stream(dev)
    out = {}

    def bench(fn, reps):
        fn()
        fn()
        fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps

    def setup(sh, dtype, direction, seed):
        inp = make_scan_inputs(sh, seed=seed, dtype=dtype)
        g = {k: (None if v is None else v.to(dev)) for k, v in inp.items()}
        D_, N_ = sh.d_inner, sh.d_state
        P = [t.contiguous() for t in pad_params(g["A_real"], g["A_imag"], g["track"], sh.n_rot,
                                                N_, D_, dev)]
        plan = ScanPlan(sh.batch, sh.seqlen, D_, N_, sh.n_rot, dtype, dtype, direction)
        bufs = {"y": torch.empty(sh.batch, sh.seqlen, D_, device=dev),
                "ckpt": torch.empty(max(1, plan.ckpt_floats()), device=dev),
                "ws": torch.empty(max(1, plan.workspace_bytes()), device=dev, dtype=torch.uint8),
                "gd": torch.empty_like(g["delta"]), "gu": torch.empty_like(g["u"]),
                "gB": torch.empty_like(g["Bc"]), "gC": torch.empty_like(g["Cc"]),
                "gA": torch.empty(3, D_, N_, device=dev), "dy": g["dy"].to(dtype).contiguous()}
        return inp, g, P, plan, bufs

    def fwd_bwd(g, P, plan, b):
        ck = b["ckpt"] if plan.ckpt_floats() else None
        plan.forward(g["delta"], g["u"], g["Bc"], g["Cc"], *P, b["y"], ck)
        plan.backward(g["delta"], g["u"], g["Bc"], g["Cc"], *P, b["dy"], ck, b["gd"], b["gu"],
                      b["gB"], b["gC"], b["gA"][0], b["gA"][1], b["gA"][2], b["ws"])

    def line(name, sh, ms, bytes_per_token, kernels, extra=None):
        tok = sh.batch * sh.seqlen
        gbs = bytes_per_token * tok / (ms / 1e3) / 1e9
        d = {"tokens_per_s": tok / (ms / 1e3), "ms_per_step": ms, "tokens_per_step": tok,
             "hbm_gbs": gbs, "hbm_frac": gbs / peak, "algorithmic_bytes_per_token": bytes_per_token}
        if kernels and all(k in ipt for k in kernels):
            inst = sum(ipt[k] for k in kernels) * tok
            d["issue_frac"] = inst / (ms / 1e3) / issue_peak
            d["warp_inst_per_token"] = sum(ipt[k] for k in kernels)
        if extra:
            d.update(extra)
        out[name] = d

    # c0: the reference's CPU-runnable case, fp32
    sh0 = ScanShape(8, 64, 256, 16, 4, 4)
    inp0, g0, P0, plan0, b0 = setup(sh0, torch.float32, S.M3_DIR_FWD, 0)
    ms0 = bench(lambda: fwd_bwd(g0, P0, plan0, b0), 200)
    c0_bytes = (2 * 4 * 256 + 2 * 4 * 16 + 4 * 256) + (3 * 4 * 256 + 2 * 4 * 16 + 2 * 4 * 256
                                                      + 2 * 4 * 16)
    cpu0 = None
    if not args.no_cpu:
        import oracle as O
        torch.set_num_threads(os.cpu_count() or 1)
        def ref0():
            O.scan_with_grads(inp0["delta"], inp0["u"], inp0["Bc"], inp0["Cc"], inp0["A_real"],
                              inp0["A_imag"], inp0["track"], inp0["dy"])
        ref0()
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 3.0:
            ref0()
            reps += 1
        el = time.perf_counter() - t0
        cpu0 = {"tokens_per_s": sh0.batch * sh0.seqlen * reps / el, "cores": os.cpu_count(),
                "kind": "port", "sample": f"the full config-0 batch, {reps} fwd+bwd in {el:.1f} s"}
    line("c0", sh0, ms0, c0_bytes, ["c0_fwd", "c0_bwd"],
         {"workload": "c0: causal scan fwd+bwd, fp32, B=8, L=64, D=256, N=16 (12 rot + 4 "
                      "track); launch-bound (512 tokens)",
          "reference_cpu": cpu0})
    del g0, b0

    cb = args.config_batch
    sh1 = ScanShape(cb, 64, 1536, 32, 16, 4)
    bf = torch.bfloat16
    # c1: bidirectional forward, inference (no checkpoints)
    _, g1, P1, plan1, b1 = setup(sh1, bf, S.M3_DIR_BIDIR, 1)
    ms1 = bench(lambda: plan1.forward(g1["delta"], g1["u"], g1["Bc"], g1["Cc"], *P1, b1["y"]), 10)
    line("c1_fwd", sh1, ms1, FWD_BYTES_PER_TOKEN, ["c1_fwd_bidir"],
         {"workload": f"c1: bidirectional forward scan (inference), bf16 inputs, fp32 state and "
                      f"y, B={cb}, L=64, D=1536, N=32 (16 rot + 16 track)"})
    # c2: fwd (with checkpoints) + bwd, bidirectional and causal
    ms2 = bench(lambda: fwd_bwd(g1, P1, plan1, b1), 5)
    line("c2_bidir", sh1, ms2, FWD_BYTES_PER_TOKEN + BWD_BYTES_PER_TOKEN,
         ["c2_fwd_bidir", "c2_bwd_bidir"],
         {"workload": f"c2: bidirectional scan fwd + analytic bwd + reductions, bf16, B={cb}"})
    del g1, b1
    torch.cuda.empty_cache()
    _, g2, P2, plan2, b2 = setup(sh1, bf, S.M3_DIR_FWD, 2)
    ms3 = bench(lambda: fwd_bwd(g2, P2, plan2, b2), 5)
    line("c2_causal", sh1, ms3, FWD_BYTES_PER_TOKEN + BWD_BYTES_PER_TOKEN,
         ["c2_fwd_causal", "c2_bwd_causal"],
         {"workload": f"c2: causal scan fwd + analytic bwd + reductions, bf16, B={cb}"})
    del g2, b2
    torch.cuda.empty_cache()
    # c2 from the raw projections -- bf16 dt before softplus and the x_proj rows
    # holding B_raw/C_raw, the 12 800 (fwd) and 29 184 (fwd+bwd) B/token
    # boundary -- two ways, both through autograd with the same dy: (a) the
    # prologue fused into both scan kernels (m3_fused_scan), (b) the prologue as
    # its own launch (m3_step_inputs, fp32) + casts to bf16 + the scan (the
    # layer's default).  Both give the same bits (tests/test_fused_prologue_gpu.py).
    g3 = torch.Generator(dev).manual_seed(3)
    dt_rank, p4 = 48, 4
    ld_x = dt_rank + 2 * N * p4
    fx = {"dt": (torch.randn(cb, 64, 1536, device=dev, generator=g3) * 0.5 - 4.0).to(bf),
          "x": torch.randn(cb, 64, ld_x, device=dev, generator=g3).to(bf),
          "u": torch.randn(cb, 64, 1536, device=dev, generator=g3).to(bf),
          "dy": torch.randn(cb, 64, 1536, device=dev, generator=g3).to(bf)}
    wbc = [1 + 0.1 * torch.randn(N * p4, device=dev, generator=g3) for _ in range(2)]
    ar_f = -torch.exp(torch.randn(1536, N_ROT, device=dev, generator=g3) * 0.5)
    ai_f = (torch.rand(1536, N_ROT, device=dev, generator=g3) * 2 - 1) * math.pi
    tk_f = torch.tanh(torch.randn(1536, N - N_ROT, device=dev, generator=g3))
    leaves = {k: v.requires_grad_(True) for k, v in fx.items() if k != "dy"}
    rows = cb * 64

    def chain(fused):
        def run():
            for v in leaves.values():
                v.grad = None
            if fused:
                y = S.m3_fused_scan(leaves["dt"], leaves["x"], wbc[0], wbc[1], 1e-5, leaves["u"],
                                    ar_f, ai_f, tk_f, N_ROT, N, p4, dt_rank, dt_rank + N * p4,
                                    S.M3_DIR_BIDIR, y_dtype=torch.float32)
            else:
                dl, bc_, cc_ = S.step_inputs(leaves["dt"].float().reshape(rows, 1536),
                                             leaves["x"].float().reshape(rows, ld_x), dt_rank,
                                             dt_rank + N * p4, wbc[0], wbc[1], 1e-5, N, p4)
                y = S.m3_bidir_scan(dl.view(cb, 64, 1536).to(bf), leaves["u"],
                                    bc_.view(cb, 64, N).to(bf), cc_.view(cb, 64, N).to(bf),
                                    ar_f, ai_f, tk_f, N_ROT, N)
            y.backward(fx["dy"].float())
        return run
    msf = bench(chain(True), 5)
    msu = bench(chain(False), 5)
    raw_bc = 2 * N * p4 * 2
    pro_bytes = (2 * 2 * 1536 + raw_bc + 4 * 1536) + (3 * 2 * 1536 + raw_bc + 2 * 2 * 1536 + raw_bc)
    line("c2_fused_prologue_bidir", sh1, msf, pro_bytes, [],
         {"workload": f"c2 from the raw projections with the prologue fused into the scan "
                      f"kernels: bidirectional fwd + bwd from raw bf16 dt and x_proj rows "
                      f"(softplus, BCNorm, MIMO fold and their backward inside the kernels), "
                      f"B={cb}, y fp32, through autograd"})
    line("c2_unfused_prologue_bidir", sh1, msu, pro_bytes, [],
         {"workload": f"the same computation with the prologue as its own launch "
                      f"(m3_step_inputs, fp32) + casts to bf16 + the scan, B={cb}, through "
                      f"autograd (the bf16 layer's default)"})
    del fx, leaves
    torch.cuda.empty_cache()
    out["issue_peak_warp_inst_per_s"] = issue_peak
    out["sm_mhz_assumed"] = mhz
    return out


def run_l_sweep(dev, args):
    """Config 4's sequence-length sweep on one GPU: the bidirectional scan fwd+bwd
    (config-2 layer shape, bf16 inputs) at B=256 rows and L = 64 .. 4096;
    tokens/s per length from CUDA events over a few steps."""
    import torch
    from redpanda_b200 import scan as S
    from redpanda_b200.scan import ScanPlan, pad_params
    out = []
    Bs = args.sweep_batch
    torch.cuda.empty_cache()
    for Ls in (64, 256, 1024, 4096):
        g = torch.Generator(dev).manual_seed(Ls)
        bf = torch.bfloat16
        x = {"delta": torch.nn.functional.softplus(
                 torch.randn(Bs, Ls, D, device=dev, generator=g) * 0.5 - 2).to(bf),
             "u": torch.randn(Bs, Ls, D, device=dev, generator=g).to(bf),
             "Bc": torch.randn(Bs, Ls, N, device=dev, generator=g).to(bf),
             "Cc": torch.randn(Bs, Ls, N, device=dev, generator=g).to(bf),
             "dy": torch.randn(Bs, Ls, D, device=dev, generator=g).to(bf)}
        ar = -torch.exp(torch.randn(D, N_ROT, device=dev, generator=g) * 0.5)
        ai = (torch.rand(D, N_ROT, device=dev, generator=g) * 2 - 1) * math.pi
        tk = torch.tanh(torch.randn(D, N - N_ROT, device=dev, generator=g))
        P = [t.contiguous() for t in pad_params(ar, ai, tk, N_ROT, N, D, dev)]
        plan = ScanPlan(Bs, Ls, D, N, N_ROT, bf, bf, S.M3_DIR_BIDIR)
        y = torch.empty(Bs, Ls, D, device=dev)
        ckpt = torch.empty(plan.ckpt_floats(), device=dev)
        ws = torch.empty(plan.workspace_bytes(), device=dev, dtype=torch.uint8)
        gd, gu = torch.empty_like(x["delta"]), torch.empty_like(x["u"])
        gB, gC = torch.empty_like(x["Bc"]), torch.empty_like(x["Cc"])
        ga = torch.empty(3, D, N, device=dev)

        def once():
            plan.forward(x["delta"], x["u"], x["Bc"], x["Cc"], *P, y, ckpt)
            plan.backward(x["delta"], x["u"], x["Bc"], x["Cc"], *P, x["dy"], ckpt, gd, gu, gB,
                          gC, ga[0], ga[1], ga[2], ws)
        reps = max(2, 4096 // Ls)
        once()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            once()
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / reps
        out.append({"seq_len": Ls, "batch": Bs, "ms_per_step": ms,
                    "gtokens_per_s": Bs * Ls / (ms / 1e3) / 1e9})
        del x, y, ckpt, ws, gd, gu, gB, gC
        torch.cuda.empty_cache()
    return out


def run_model_train(dev, args, mp):
    """Config 4 at model level: the 16-layer bidirectional Eval-Mamba stack of
    config 1 (d_model=768, d_inner=1536, d_state=32 with 16 tracking lanes,
    mimo_p=4, vocab 8192, the reference initialisation), one training step =
    forward, loss y.pow(2).mean() (the reference's verify-gate loss), backward
    through the kernels (scan, prologue) and torch (GEMMs), and a fused AdamW
    step.  The global batch (``args.train_global`` rows of L=64 random token
    ids) is split evenly over the ranks and run in micro-batches of
    ``args.train_batch`` rows with gradient accumulation; on more than one GPU
    every parameter gradient (the scan parameters A, theta, dt bias and BCNorm
    weights among them) is all-reduced over NCCL in buckets started from the
    backward of the last micro-batch, overlapping the rest of it.  GEMMs in
    TF32, scan state and gradients in fp32."""
    import torch
    from redpanda_b200.distributed import OverlappedGradAllReducer
    from redpanda_b200.mamba import Mamba, MambaConfig
    mb = args.train_batch
    per_rank = max(mb, args.train_global // mp.world)
    accum = max(1, per_rank // mb)
    old_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        torch.manual_seed(17)   # the same initial weights on every rank
        cfg = MambaConfig(d_model=768, n_layer=16, d_state=32, n_track_state=16, mimo_p=4,
                          vocab_size=8192, bidirectional=True)
        model = Mamba(cfg).to(dev).train()
        opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True)
        red = OverlappedGradAllReducer(model) if mp.world > 1 else None
        g = torch.Generator(dev).manual_seed(19 + mp.rank)
        ids = [torch.randint(0, 8192, (mb, 64), device=dev, generator=g) for _ in range(accum)]
        last = {}

        def step():
            opt.zero_grad(set_to_none=True)
            for i in range(accum):
                if red is not None and i == accum - 1:
                    red.arm()
                # bf16 mixed precision, as the reference trains (train.py:268)
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    loss = model(ids[i]).float().pow(2).mean() / accum
                loss.backward()
            if red is not None:
                red.finish()
            opt.step()
            last["loss"] = loss

        def steps(n):
            def run():
                for _ in range(n):
                    step()
            return run
        steps(2)()
        n = 3
        ms = mp.timed(steps(n)) / n
        rows = per_rank * mp.world
        return {"workload": f"c4 model level: 16-layer bidirectional Mamba (d_model=768, "
                            f"d_inner=1536, d_state=32 with 16 tracking lanes, mimo_p=4), global "
                            f"B={rows} x L=64 per step ({per_rank} rows per GPU in {accum} "
                            f"micro-batches of {mb}), fwd + bwd + fused AdamW",
                "n_gpus": mp.world, "ms_per_step": ms, "tokens_per_s": rows * 64 / (ms / 1e3),
                "loss": float(last["loss"].item()) * accum,
                "allreduce": ("every parameter gradient, NCCL, buckets of ~8 MB started during "
                              "the last micro-batch's backward" if mp.world > 1 else "none (1 GPU)"),
                "precision": "torch.autocast bf16 (the reference's mixed precision): bf16 "
                             "projections on the tensor cores, the kernels' bf16 configuration "
                             "(bf16 delta/u/Bc/Cc and y, fp32 state and accumulation), fp32 "
                             "parameters, residual stream and optimizer"}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old_tf32


def run_search_nodes(dev, args):
    """Search node evaluation at batch 1 (SearchMamba.eval_step,
    search_mamba.py:275-291, as MARS calls it per node): a config-3-shaped
    SearchMamba (12 layers, d_model=512, d_inner=1024, d_state=32 with 8
    tracking lanes, mimo_p=2, vocab 8192) primed on a 64-token board, then a
    chain of single-move evaluations, each returning the value as a Python
    float (a host sync per node, as the reference's ``.item()``).  Eager
    (``eval_step``: the stack's launches one by one) against the stack and both
    heads replayed as one CUDA graph (``eval_step_graphed``).  TF32 projections."""
    import torch
    from redpanda_b200.search_mamba import SearchMamba, SearchMambaConfig
    old_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        torch.manual_seed(31)
        scfg = SearchMambaConfig(d_model=512, n_layer=12, d_state=32, n_track_state=8,
                                 mimo_p=2, vocab_size=8192)
        sm = SearchMamba(scfg, vocab_size=8192).to(dev).eval()
        g = torch.Generator(dev).manual_seed(37)
        board = torch.randint(0, 8192, (64,), device=dev, generator=g)
        moves = torch.randint(0, 8192, (64,), generator=torch.Generator().manual_seed(41)).tolist()
        out = {}
        with torch.no_grad():
            _, cache0 = sm.prime_board(board)
            for name, fn in (("eager", sm.eval_step), ("graph", sm.eval_step_graphed)):
                cache = cache0
                for mv in moves[:8]:   # warm-up (captures the graph)
                    _, _, cache = fn(cache, mv)
                torch.cuda.synchronize(dev)
                t0 = time.perf_counter()
                cache = cache0
                for mv in moves:
                    _, _, cache = fn(cache, mv)
                torch.cuda.synchronize(dev)
                dt = time.perf_counter() - t0
                out[name] = {"us_per_node": dt / len(moves) * 1e6,
                             "nodes_per_s": len(moves) / dt}
            # evaluate_lines_fast: 32 candidate lines of 8 moves from the board
            # (search_mamba.py:178-219), eager vs stepping a captured graph
            lines = torch.randint(0, 8192, (32, 8), device=dev, generator=g)
            for name, graphed in (("lines_eager", False), ("lines_graph", True)):
                sm.evaluate_lines_fast(board, lines, graphed=graphed)   # warm-up / capture
                torch.cuda.synchronize(dev)
                t0 = time.perf_counter()
                for _ in range(5):
                    sm.evaluate_lines_fast(board, lines, graphed=graphed)
                torch.cuda.synchronize(dev)
                out[name] = {"ms_per_call": (time.perf_counter() - t0) / 5 * 1e3,
                             "lines": 32, "moves": 8}
        sm.release_graphs()
        # the backbone's step graph alone by batch, with the prologue inside the
        # step kernel and as its own launch (Mamba3Block.fuse_step)
        from redpanda_b200.graphs import StepGraph
        from redpanda_b200.mamba import Mamba3Block
        sweep = {}
        old_small = Mamba3Block.small_step_max_batch
        try:
            for B in (1, 8, 64, 256, 1024, 4096):
                ids = torch.randint(0, 8192, (B, 16), device=dev, generator=g)
                mv = torch.randint(0, 8192, (B,), device=dev, generator=g)
                variants = ([("small", True, old_small)] if B <= old_small else []) + \
                    [("fused", True, 0), ("two_launch", False, 0)]
                for vname, fuse, small in variants:
                    Mamba3Block.fuse_step = fuse
                    Mamba3Block.small_step_max_batch = small
                    old_max = Mamba3Block.fuse_step_max_batch
                    Mamba3Block.fuse_step_max_batch = 1 << 30
                    with torch.no_grad():
                        gr = StepGraph(sm.backbone, B)
                        sm.backbone.prime_cache(ids, out=gr.cache)
                        for _ in range(3):
                            gr.step(mv)
                        torch.cuda.synchronize(dev)
                        e0 = torch.cuda.Event(enable_timing=True)
                        e1 = torch.cuda.Event(enable_timing=True)
                        n = 30 if B <= 1024 else 10
                        e0.record()
                        for _ in range(n):
                            gr.step(mv)
                        e1.record()
                        torch.cuda.synchronize(dev)
                    Mamba3Block.fuse_step_max_batch = old_max
                    sweep[f"B{B}_{vname}"] = e0.elapsed_time(e1) / n * 1e3
                    del gr
        finally:
            Mamba3Block.fuse_step = True
            Mamba3Block.small_step_max_batch = old_small
        del sm
        torch.cuda.empty_cache()
        out["workload"] = ("a10 search node evaluation: 12-layer SearchMamba (d_model=512, "
                           "d_inner=1024, d_state=32 with 8 tracking lanes, mimo_p=2), batch 1, "
                           "64 chained eval_step calls after a 64-token prime, value read "
                           "back per node; host wall clock (each node ends in a host sync)")
        out["speedup"] = out["eager"]["us_per_node"] / out["graph"]["us_per_node"]
        out["graph_step_us_by_batch"] = sweep
        out["graph_step_note"] = ("the backbone's 12-layer step as one CUDA graph, us per step "
                                  "(CUDA events): small = the small-batch layer (norm + "
                                  "projections + step + residual in four launches per layer, "
                                  "step_fused_'s path up to Mamba3Block.small_step_max_batch "
                                  "rows); fused = cuBLAS projections with the prologue inside "
                                  "the step kernel (up to Mamba3Block.fuse_step_max_batch rows); "
                                  "two_launch = cuBLAS projections, prologue as its own launch")
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old_tf32


def run_model_eval(dev, args):
    """The Eval-Mamba stack forward in bf16 (model.py:110-132 / mamba.py:231-267 at
    config 1): the 16-layer bidirectional Mamba of config 4 (d_model=768,
    d_inner=1536, d_state=32 with 16 tracking lanes, mimo_p=4), inference
    (no grad) under torch.autocast bf16, B=``args.config_batch`` rows x L=64:
    bf16 projections, softplus/BCNorm/MIMO fold in one launch, the fused
    bidirectional scan writing bf16 y, the gate (y + 2uD)*silu(z) in bf16, the
    bf16 out_proj.  One GPU."""
    import torch
    from redpanda_b200.mamba import Mamba, MambaConfig
    Bs = args.config_batch
    torch.manual_seed(23)
    cfg = MambaConfig(d_model=768, n_layer=16, d_state=32, n_track_state=16, mimo_p=4,
                      vocab_size=8192, bidirectional=True)
    model = Mamba(cfg).to(dev).eval()
    g = torch.Generator(dev).manual_seed(29)
    ids = torch.randint(0, 8192, (Bs, 64), device=dev, generator=g)
    stream = torch.cuda.current_stream(dev)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        for _ in range(2):
            model(ids)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 5
        e0.record(stream)
        for _ in range(n):
            out = model(ids)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / n
    del model, out
    torch.cuda.empty_cache()
    return {"workload": f"c1 model level: 16-layer bidirectional Mamba forward (d_model=768, "
                        f"d_inner=1536, d_state=32 with 16 tracking lanes, mimo_p=4), inference, "
                        f"B={Bs} x L=64",
            "ms_per_forward": ms, "tokens_per_s": Bs * 64 / (ms / 1e3),
            "precision": "torch.autocast bf16; scan state and accumulation fp32"}


def run_model_rollout(dev, args, mp):
    """Config 3 at model level: a 12-layer Search-Mamba-shaped ``Mamba``
    (d_model=512, d_inner=1024, d_state=32 with 8 tracking lanes, mimo_p=2,
    vocab 8192, the reference initialisation), B rollout rows (split evenly
    over the ranks, no communication) advanced 32 steps by the fused step layer
    (embedding, RMSNorm, cuBLAS projections, one launch for softplus/BCNorm/MIMO
    fold, one for the recurrence with the gated output, out_proj fused with the
    residual add), re-anchored every 8 steps by ``prime_cache`` over a fresh
    L=64 token sequence (scan with return_state).  Token ids are uniform over
    the 8192-move space.  GEMMs run in TF32; state and recurrence in fp32."""
    import torch
    from redpanda_b200.mamba import Mamba, MambaConfig
    layers = args.rollout_layers
    Bs = max(1, args.rollout_batch // mp.world)
    old_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        torch.manual_seed(11)
        cfg = MambaConfig(d_model=512, n_layer=layers, d_state=32, n_track_state=8, mimo_p=2,
                          vocab_size=8192)
        model = Mamba(cfg).to(dev).eval()
        g = torch.Generator(dev).manual_seed(13 + mp.rank)
        boards = [torch.randint(0, 8192, (Bs, 64), device=dev, generator=g) for _ in range(4)]
        moves = torch.randint(0, 8192, (32, Bs), device=dev, generator=g)
        stream = torch.cuda.current_stream(dev)
        ev = []

        def rollout(record=False):
            cache = None
            for s_ in range(32):
                if s_ % 8 == 0:
                    if record:
                        ev.append(torch.cuda.Event(enable_timing=True))
                        ev[-1].record(stream)
                    _, cache = model.prime_cache(boards[s_ // 8])
                    if record:
                        ev.append(torch.cuda.Event(enable_timing=True))
                        ev[-1].record(stream)
                x, cache = model.step_fused_(token_id=moves[s_], cache=cache)
            return x

        with torch.no_grad():
            rollout()
            total = mp.timed(lambda: rollout(record=True))
        anchor = mp.max(sum(ev[i].elapsed_time(ev[i + 1]) for i in range(0, len(ev), 2)))
        steps_ms = total - anchor

        # the same eager rollout with the step prologue fused into the step
        # kernel (m3_step_gated_fused; by default only batches of at most
        # Mamba3Block.fuse_step_max_batch rows take it)
        from redpanda_b200.mamba import Mamba3Block
        ev.clear()
        old_max = Mamba3Block.fuse_step_max_batch
        Mamba3Block.fuse_step_max_batch = 1 << 30
        try:
            with torch.no_grad():
                rollout()
                total_u = mp.timed(lambda: rollout(record=True))
        finally:
            Mamba3Block.fuse_step_max_batch = old_max
        anchor_u = mp.max(sum(ev[i].elapsed_time(ev[i + 1]) for i in range(0, len(ev), 2)))
        steps_u = total_u - anchor_u

        # the same rollout with the 12-layer step replayed as one CUDA graph
        # (redpanda_b200.graphs.StepGraph) and each re-anchor primed straight
        # into the graph's static state
        from redpanda_b200.graphs import StepGraph
        ev.clear()
        torch.cuda.empty_cache()
        with torch.no_grad():
            graph = StepGraph(model, Bs)

            def rollout_graph(record=False):
                for s_ in range(32):
                    if s_ % 8 == 0:
                        if record:
                            ev.append(torch.cuda.Event(enable_timing=True))
                            ev[-1].record(stream)
                        model.prime_cache(boards[s_ // 8], out=graph.cache)
                        if record:
                            ev.append(torch.cuda.Event(enable_timing=True))
                            ev[-1].record(stream)
                    x = graph.step(moves[s_])[0]
                return x

            rollout_graph()
            total_g = mp.timed(lambda: rollout_graph(record=True))
        anchor_g = mp.max(sum(ev[i].elapsed_time(ev[i + 1]) for i in range(0, len(ev), 2)))
        steps_g = total_g - anchor_g
        del graph
        torch.cuda.empty_cache()
        rows = Bs * mp.world
        return {
            "workload": f"c3 model level: {layers}-layer Mamba (d_model=512, d_inner=1024, "
                        f"d_state=32 with 8 tracking lanes, mimo_p=2, vocab 8192), B={rows} "
                        f"({Bs} per GPU), 32 lockstep steps, prime_cache re-anchor over L=64 "
                        "every 8 steps",
            "n_gpus": mp.world,
            "node_steps_per_s": rows * 32 / (total / 1e3),
            "ms_per_rollout": total,
            "anchor_ms": anchor,
            "step_ms_per_node_step_batch": steps_ms / 32,
            "step_only_node_steps_per_s": rows * 32 / (steps_ms / 1e3),
            "precision": "TF32 projections, fp32 state and recurrence",
            "state": "reference (h, dBu) cache pair",
            "step_ms_fused_prologue": steps_u / 32,
            "graph": {
                "node_steps_per_s": rows * 32 / (total_g / 1e3),
                "ms_per_rollout": total_g,
                "anchor_ms": anchor_g,
                "step_ms_per_node_step_batch": steps_g / 32,
                "launches_per_step": 1,
                "note": "the 12-layer fused step captured once as a CUDA graph; re-anchors "
                        "prime into the graph's static state",
            },
        }
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old_tf32


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["m3", "reference"], default="m3")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-rollout", dest="rollout", action="store_false",
                    help="skip the config-3 step rollout measurement")
    ap.add_argument("--no-model-train", dest="model_train", action="store_false",
                    help="skip the config-4 model-level training step")
    ap.add_argument("--train-batch", type=int, default=256,
                    help="micro-batch rows of the config-4 model-level training step")
    ap.add_argument("--train-global", type=int, default=2048,
                    help="global rows per training step, split over the GPUs")
    ap.add_argument("--no-sweep", dest="sweep", action="store_false",
                    help="skip the config-4 sequence-length sweep")
    ap.add_argument("--sweep-batch", type=int, default=256)
    ap.add_argument("--no-configs", dest="configs", action="store_false",
                    help="skip the per-configuration lines (c0, c1 forward, c2 causal/bidir)")
    ap.add_argument("--config-batch", type=int, default=1024,
                    help="rows of the c1/c2 lines (default 1024, the configs' batch)")
    ap.add_argument("--rollout-layers", type=int, default=12,
                    help="layers of the config-3 rollout (default 12; fewer for profiler captures)")
    ap.add_argument("--rollout-batch", type=int, default=8192,
                    help="rollout rows (default 8192; fewer for profiler captures)")
    ap.add_argument("--e2e-sub", type=int, default=16,
                    help="sub-batches the end-to-end leg streams each step's rows in "
                         "(default 16: measured 130 ms/step at 8192 rows against 147 with 4 "
                         "and 137 with 8; the copies then run near the PCIe limit)")
    ap.add_argument("--no-search", dest="search", action="store_false",
                    help="skip the batch-1 search-node line")
    ap.add_argument("--batch", type=int, default=0,
                    help="rows per GPU (default: config 4's global 8192 rows split over "
                         "the GPUs; smaller values are for profiler captures only)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_m3(args)


if __name__ == "__main__":
    main()
