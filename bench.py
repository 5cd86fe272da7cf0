"""Benchmark of the decode-shaped quantized matmul path on B200.

One step = every 4-bit g64 quantized projection of one Qwen2.5-7B decode token
at M=1: 28 layers x (q 3584x3584, k 512x3584, v 512x3584, o 3584x3584,
gate 18944x3584, up 18944x3584, down 3584x18944) + lm_head 152064x3584.
Weights ~ N(0, 0.02) -> bf16 -> quantized on device; x ~ N(0, 1) bf16 (synthetic,
seeded). The step streams 3.98 GB of packed weights, far larger than L2, so
no L2 flush is needed between steps.

  value  device-resident throughput: algorithmic bytes / step time, the step
         replayed from a CUDA graph of the public-API calls (HBM GB/s).
  e2e    same metric with, every step, the H2D copy of all inputs from pinned
         host memory, the graph replay, and the D2H copy of all outputs.
  fused_projections  the same weights with each layer's q/k/v and gate/up
         stacked along N (concat_quantized): 113 launches per step instead of 197.

With --gpus N (torchrun), every projection is N-sharded by output rows; each
rank streams its shard and the step ends with one NCCL all-gather of all
outputs; value = all ranks' algorithmic bytes / max-over-ranks step time.

--impl reference runs the CPU restatement of MLX's algorithm (the oracle, all
host threads) on a bounded sample of the same workload (one decoder layer).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, INTER, VOCAB, LAYERS = 3584, 18944, 152064, 28
KV = 512
PROJ = [("q", HIDDEN, HIDDEN), ("k", KV, HIDDEN), ("v", KV, HIDDEN), ("o", HIDDEN, HIDDEN),
        ("gate", INTER, HIDDEN), ("up", INTER, HIDDEN), ("down", HIDDEN, INTER)]
BITS, GS = 4, 64
METRIC = "W4 qmm HBM GB/s at M=1 (Qwen2.5-7B decode-token projections)"


def load_package():
    name = "mlx_server_runtime_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = os.path.join(ROOT, "mlx-server-runtime_b200")
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(pkg, "__init__.py"), submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def qmm_bytes(M, N, K, bits=BITS, gs=GS):
    """Algorithmic bytes of one quantized_matmul: packed weights + bf16 scales and
    biases + bf16 activations in + bf16 outputs."""
    return N * K * bits // 8 + 4 * N * K // gs + 2 * M * K + 2 * M * N


def shapes(world=1, rank=0):
    """(name, N_shard, K) of every projection of the step, N-sharded over ranks."""
    out = []
    for layer in range(LAYERS):
        for name, N, K in PROJ:
            out.append((f"L{layer}.{name}", N, K))
    out.append(("lm_head", VOCAB, HIDDEN))
    res = []
    for name, N, K in out:
        per = (N + world - 1) // world
        lo, hi = rank * per, min(N, (rank + 1) * per)
        res.append((name, max(0, hi - lo), K))
    return res


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                r = subprocess.run(["nvidia-smi", "-i", str(self.index),
                                    f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits"],
                                   capture_output=True, text=True, timeout=5)
                if r.returncode == 0 and r.stdout.strip():
                    self.samples.append([v.strip() for v in r.stdout.strip().split(",")])
            except Exception:
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 3 + i and s[3 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class CpuLayer:
    """One Qwen2.5-7B decoder layer's quantized projections in host memory, for
    the C oracle (CPU restatement of MLX's algorithm)."""

    def __init__(self, threads: int | None = None):
        import numpy as np

        from oracle import coracle, oracle_np

        coracle.build()
        if threads:
            coracle.set_num_threads(threads)
        self.coracle = coracle
        rng = np.random.default_rng(0)
        self.layer = []
        for name, N, K in PROJ:
            w = oracle_np.from_f32(rng.standard_normal((N, K), dtype=np.float32) * 0.02,
                                   "bfloat16")
            wq, s, b = coracle.quantize(w, "bfloat16", GS, BITS)
            x = oracle_np.from_f32(rng.standard_normal((1, K), dtype=np.float32), "bfloat16")
            self.layer.append((x, wq, s, b))
        self.bytes = sum(qmm_bytes(1, N, K) for _, N, K in PROJ)
        self.threads = coracle.num_threads()

    def run(self, seconds: float):
        """Whole-layer passes until `seconds` elapse; returns (GB/s, passes, seconds)."""
        t0 = time.perf_counter()
        passes = 0
        while True:
            for x, wq, s, b in self.layer:
                self.coracle.quantized_matmul(x, wq, s, b, "bfloat16", GS, BITS)
            passes += 1
            if time.perf_counter() - t0 > seconds:
                break
        dt = time.perf_counter() - t0
        return self.bytes * passes / dt / 1e9, passes, dt


def cpu_baseline(seconds: float = 12.0, threads: int | None = None):
    """Time the C oracle on one decoder layer's projections at M=1 (bounded sample)."""
    lay = CpuLayer(threads)
    lay.run(0.0)  # warm-up pass
    gbs, passes, dt = lay.run(seconds)
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": lay.threads, "kind": "port",
            "sample": f"{passes} pass(es) over one Qwen2.5-7B layer's 7 projections at M=1 "
                      f"({lay.bytes / 1e6:.1f} MB each), C oracle -O3 OpenMP, "
                      f"{dt:.1f} s of CPU work",
            "seconds": round(dt, 2)}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    import numpy as np  # noqa: F401

    lay = CpuLayer()
    nthreads = lay.threads
    per_step = min(10.0, max(0.5, 90.0 / max(1, args.steps + args.warmup)))
    vals = []
    for i in range(args.warmup + args.steps):
        gbs, _, _ = lay.run(per_step)
        if i >= args.warmup:
            vals.append(gbs)
    value = round(statistics.median(vals), 3)
    step_bytes = sum(qmm_bytes(1, N, K) for _, N, K in shapes())
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_bytes / (value * 1e9) * 1e3, 3),
        "higher_is_better": True, "scaling": "strong" if args.gpus > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded numpy, W~N(0,0.02) bf16 -> 4-bit g64, x~N(0,1))",
        "config": {"workload": "qwen2.5-7b decode-token projections, M=1, 4-bit g64 "
                               "(CPU sample: one layer per step)", "global_batch": 1,
                   "parallelism": "cpu"},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": nthreads, "kind": "port",
                         "sample": "one Qwen2.5-7B layer's 7 projections at M=1 per step "
                                   "(C restatement of MLX's CPU algorithm; MLX itself is not "
                                   "installable here)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    mxq = load_package()
    mxq.load_library()

    shp = shapes(world, rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    weights, xs, outs = [], [], []
    x_flat = torch.empty(sum(K for _, N, K in shp if N), dtype=torch.bfloat16, device=dev)
    out_flat = torch.empty(sum(N for _, N, K in shp if N), dtype=torch.bfloat16, device=dev)
    off = 0
    for name, N, K in shp:
        if N == 0:
            weights.append(None)
            xs.append(None)
            outs.append(None)
            continue
        w = (torch.randn(N, K, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        weights.append(mxq.quantize(w, GS, BITS))
        del w
        x = x_flat[off:off + K].view(1, K)
        x.copy_(torch.randn(1, K, device=dev, generator=gen))
        off += K
        xs.append(x)
        outs.append(None)
    torch.cuda.synchronize()

    def step_eager():
        for i, wt in enumerate(weights):
            if wt is not None:
                outs[i] = mxq.quantized_matmul(xs[i], *wt, group_size=GS, bits=BITS)
        # one flat result buffer (feeds the all-gather and the single D2H copy)
        torch.cat([o.reshape(-1) for o in outs if o is not None], out=out_flat)

    # Launch overlap: the projections' weights are static, so each matmul may start
    # streaming them while the previous one finishes.
    overlap = mxq.launch_overlap(not args.no_overlap)

    # warm-up eagerly (sets kernel attributes, allocates workspaces), then capture
    for _ in range(2):
        step_eager()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        step_eager()  # workspaces for this stream
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            step_eager()
    torch.cuda.synchronize()
    launches_per_step = sum(1 for w in weights if w is not None)

    # The same projections with q/k/v and gate/up stacked along N (concat_quantized):
    # 4 launches per layer instead of 7, the same weight bytes.
    fused_ops = []
    for layer in range(LAYERS + 1):
        if layer == LAYERS:
            groups = [[len(weights) - 1]]
        else:
            b0 = layer * len(PROJ)
            groups = [[b0, b0 + 1, b0 + 2], [b0 + 3], [b0 + 4, b0 + 5], [b0 + 6]]
        for g in groups:
            g = [i for i in g if weights[i] is not None]
            if not g:
                continue
            wt = weights[g[0]] if len(g) == 1 else mxq.concat_quantized(
                [weights[i] for i in g], GS, BITS)
            fused_ops.append((xs[g[0]], wt))
    fused_bytes = sum(qmm_bytes(1, wt[0].shape[0], x.shape[-1]) for x, wt in fused_ops)

    def step_fused_eager():
        for x, wt in fused_ops:
            mxq.quantized_matmul(x, *wt, group_size=GS, bits=BITS)

    for _ in range(2):
        step_fused_eager()
    torch.cuda.synchronize()
    graph_fused = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        step_fused_eager()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph_fused, stream=stream):
            step_fused_eager()
    torch.cuda.synchronize()

    gathered = None
    if world > 1:
        gathered = torch.empty(world * out_flat.numel(), dtype=torch.bfloat16, device=dev)

    def step():
        graph.replay()
        if world > 1:
            dist.all_gather_into_tensor(gathered, out_flat)

    step_bytes = sum(qmm_bytes(1, N, K) for _, N, K in shp if N)
    total_bytes = step_bytes
    if world > 1:
        t = torch.tensor([step_bytes], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        total_bytes = int(t.item())

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    cur = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        barrier()
        ev0.record(cur)
        for _ in range(args.steps):
            step()
        ev1.record(cur)
        barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = total_bytes / (ms * 1e-3) / 1e9

    # ---- fused projections (device-resident, like value) --------------------------
    for _ in range(3):
        graph_fused.replay()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(cur)
    for _ in range(args.steps):
        graph_fused.replay()
    f1.record(cur)
    barrier()
    ms_fused = f0.elapsed_time(f1) / args.steps
    if world > 1:
        t = torch.tensor([ms_fused, float(fused_bytes)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_fused = float(t[0].item())
        tb = torch.tensor([float(fused_bytes)], dtype=torch.float64, device=dev)
        dist.all_reduce(tb)
        fused_total = float(tb.item())
    else:
        fused_total = float(fused_bytes)
    del graph_fused

    # ---- end to end: pinned H2D of inputs, replay, D2H of outputs ---------------
    x_host = x_flat.cpu().pin_memory()
    res = gathered if world > 1 else out_flat
    o_host = torch.empty(res.shape, dtype=res.dtype).pin_memory()
    h2d = x_host.numel() * 2
    d2h = o_host.numel() * 2

    def step_e2e():
        x_flat.copy_(x_host, non_blocking=True)
        step()
        o_host.copy_(res, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()

    for _ in range(3):
        step_e2e()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(cur)
    for _ in range(args.steps):
        step_e2e()
    t1.record(cur)
    barrier()
    ms_e2e = t0.elapsed_time(t1) / args.steps
    if world > 1:
        t = torch.tensor([ms_e2e], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e = total_bytes / (ms_e2e * 1e-3) / 1e9

    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            tr = json.load(f)
        traffic = tr.get("qmv_decode_step_bytes")
    except Exception:
        pass

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            cpu = cpu_baseline(seconds=args.cpu_seconds)
        except Exception as e:  # reported, never fatal to the GPU numbers
            cpu = {"value": None, "error": str(e)[:200]}

    if world > 1:
        graph.reset() if hasattr(graph, "reset") else None
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded torch RNG: W~N(0,0.02) bf16 -> 4-bit g64 on device, "
                    "x~N(0,1) bf16)",
            "config": {"workload": "qwen2.5-7b decode-token quantized projections at M=1: "
                                   "28 layers x q/k/v/o/gate/up/down + lm_head, 4-bit g64",
                       "global_batch": 1, "parallelism": f"n-shard{world}",
                       "step_bytes": total_bytes, "l2": "inputs exceed L2 (3.98 GB/step)",
                       "replay": "cuda graph of public-API calls",
                       "launch_overlap": not args.no_overlap,
                       "allgather": "one NCCL all-gather of all outputs per step" if world > 1
                       else None,
                       "qmm_only_tok_per_s": round(1000.0 / ms, 1)},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": peak * world,
                         "unit": "GB/s", "frac": round(value / (peak * world), 4),
                         "peak_source": peak_src + (f" (per GPU x {world})" if world > 1 else ""),
                         "frac_of_8TBs_nominal": round(value / (8000.0 * world), 4),
                         "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e, 4)},
            "clocks": clk.summary(),
            "fused_projections": {
                "value": round(fused_total / (ms_fused * 1e-3) / 1e9, 1), "unit": "GB/s",
                "ms_per_step": round(ms_fused, 4),
                "launches_per_step": len(fused_ops),
                "qmm_only_tok_per_s": round(1000.0 / ms_fused, 1),
                "what": "same projections with q/k/v and gate/up stacked along N "
                        "(concat_quantized): one launch each, same weight bytes"},
        }
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.destroy_process_group()


CASES = {"q": (HIDDEN, HIDDEN), "kv": (KV, HIDDEN), "gate": (INTER, HIDDEN),
         "down": (HIDDEN, INTER), "lm_head": (VOCAB, HIDDEN)}


def run_case(args):
    """A few launches of one projection (small, for ncu captures and sweeps):
    rotates over enough weight copies that their total exceeds L2."""
    import torch

    mxq = load_package()
    dev = torch.device("cuda", 0)
    N, K = CASES[args.case]
    M = args.m
    per = qmm_bytes(M, N, K)
    copies = max(2, min(16, -(-400_000_000 // (N * K // 2))))
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    ws = []
    for _ in range(copies):
        w = (torch.randn(N, K, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        ws.append(mxq.quantize(w, GS, BITS))
        del w
    x = torch.randn(M, K, device=dev, generator=gen).to(torch.bfloat16)
    mxq.launch_overlap(not args.no_overlap)
    for i in range(max(3, args.warmup)):
        mxq.quantized_matmul(x, *ws[i % copies], group_size=GS, bits=BITS)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.eager:
        e0.record()
        for i in range(args.steps):
            mxq.quantized_matmul(x, *ws[i % copies], group_size=GS, bits=BITS)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.steps
    else:
        # one graph of `copies` launches (each weight copy once), replayed
        st = torch.cuda.Stream(device=dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(st):
            for i in range(copies):
                mxq.quantized_matmul(x, *ws[i], group_size=GS, bits=BITS)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for i in range(copies):
                mxq.quantized_matmul(x, *ws[i], group_size=GS, bits=BITS)
        for _ in range(3):
            g.replay()
        reps = max(1, args.steps // copies)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
    flops = 2.0 * M * N * K
    print(json.dumps({"case": args.case, "M": M, "N": N, "K": K, "copies": copies,
                      "overlap": not args.no_overlap,
                      "us_per_launch": round(us, 3), "bytes": per,
                      "GB/s": round(per / (us * 1e-6) / 1e9, 1),
                      "TFLOP/s": round(flops / (us * 1e-6) / 1e12, 1)}), flush=True)


MOE_CASES = {"moe_gate": (768, 2048), "moe_down": (2048, 768)}  # (N, K), 128 experts
MOE_E, MOE_TOPK = 128, 8


def run_moe_case(args):
    """Sorted gather_qmm of one Qwen3-30B-A3B-shaped MoE projection: T tokens x top-8
    of 128 experts (uniform random routing, seeded), rows sorted by expert."""
    import torch

    mxq = load_package()
    dev = torch.device("cuda", 0)
    N, K = MOE_CASES[args.case]
    T = args.m
    rows = T * MOE_TOPK
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    w = (torch.randn(MOE_E, N, K, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    wq, s, b = mxq.quantize(w, GS, BITS)
    del w
    x = torch.randn(rows, 1, K, device=dev, generator=gen).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(MOE_E, device=dev, generator=gen)[:MOE_TOPK]
                       for _ in range(T)]).reshape(-1).to(torch.int32)
    rhs = torch.sort(idx).values

    def call():
        return mxq.gather_qmm(x, wq, s, b, rhs_indices=rhs, group_size=GS, bits=BITS,
                              sorted_indices=True)

    for _ in range(max(3, args.warmup)):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    used = int(torch.unique(rhs).numel())
    wbytes = used * (N * K * BITS // 8 + 4 * N * K // GS)
    byts = wbytes + 2 * rows * K + 2 * rows * N
    flops = 2.0 * rows * N * K
    print(json.dumps({"case": args.case, "T": T, "rows": rows, "N": N, "K": K, "experts": MOE_E,
                      "experts_used": used, "us_per_call": round(us, 3), "bytes": byts,
                      "GB/s": round(byts / (us * 1e-6) / 1e9, 1),
                      "TFLOP/s": round(flops / (us * 1e-6) / 1e12, 2)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=sorted(CASES) + sorted(MOE_CASES), default=None,
                    help="time one projection only (eager launches, for profiling)")
    ap.add_argument("--m", type=int, default=1, help="tokens for --case")
    ap.add_argument("--eager", action="store_true", help="--case: plain launches, no graph")
    ap.add_argument("--no-overlap", action="store_true",
                    help="launch matmuls without programmatic launch overlap")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.case in MOE_CASES:
        run_moe_case(args)
    elif args.case:
        run_case(args)
    else:
        run(args)


if __name__ == "__main__":
    main()
