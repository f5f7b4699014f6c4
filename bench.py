#!/usr/bin/env python
"""Benchmark of the int4 MatMulNBits path on B200 (one JSON line on rank 0).

Workload ("decode GEMV sweep"): M in {1, 2, 4, 8} tokens x the four fused
projection shapes (K, N) = qkvz|ab (2048, 8224), attn qkv (2048, 3072), gate|up (2048, 12288),
down (6144, 2048). One step = the 16 matmuls of the sweep. Weights are synthetic with the
configs' distribution (seeded), replicated on every GPU (data-parallel, no collective: each rank
runs the same per-GPU work, weak scaling). Each call uses the next of 8 distinct device copies of
its weight, 272 MB in total, so weights stream from HBM, not from the 126 MB L2.

Metric: algorithmic bytes / second, bytes = N*K/2 (int4) + N*K/16 (fp16 scales) + 2*M*K + 2*M*N
(the weight bytes of gemmbench/bench.js:53 plus activations in and out). ``value`` is the
device-timed aggregate with inputs resident; ``e2e`` is the same sweep through the C ABI's
host-buffer entry point (pinned host x -> device -> matmul -> pinned host y, every call).

``--impl reference`` times the reference's CPU path (fp32 dequantise-then-matmul, the fake-quant
route of convert/export_engine.py:88-103, restated in ``oracle/``) on the host cores instead.
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
PKG_DIR = os.path.join(ROOT, "strands-decider-web_b200")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

SHAPES = [("qkvz_ab", 2048, 8224), ("attn_qkv", 2048, 3072), ("gate_up", 2048, 12288), ("down", 6144, 2048)]
MS = [1, 2, 4, 8]
COPIES = 8
NSETS = 4           # bound input/output buffer sets (and end-to-end streams), used round robin
L2_BYTES = 126 << 20
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def load_pkg():
    name = "strands_decider_web_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def upload_graph(g, stream) -> bool:
    """Upload an instantiated CUDA graph to the device before it is first replayed (cuGraphUpload:
    executes nothing), so the first replay's upload does not land inside a timed region."""
    try:
        from cuda.bindings import driver as cu
        exec_ = g.raw_cuda_graph_exec()
        err, = cu.cuGraphUpload(cu.CUgraphExec(int(exec_)), cu.CUstream(int(stream.cuda_stream)))
        return int(err) == 0
    except Exception:
        return False


def bench_config():
    """The workload both arms report (the same dict, so the two lines' configs compare equal)."""
    return {"workload": "decode_gemv_sweep_config2", "M": MS, "shapes_KN": [[K, N] for _, K, N in SHAPES]}


# device-side delay queued before a start event (about 1 ms at 1965 MHz), longer than the host's
# event record + graph launch
LAUNCH_SHIELD_CYCLES = 2_000_000


def alg_bytes(M, K, N):
    return N * K // 2 + N * K // 16 + 2 * M * K + 2 * M * N


def sweep_bytes():
    return sum(alg_bytes(M, K, N) for M in MS for _, K, N in SHAPES)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def profile_traffic():
    """DRAM bytes per launch of the chained decode kernel from the committed ncu summary (or None)."""
    p = os.path.join(ROOT, "profiles", "chain_decode_sweep.md")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 20 ms while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.lines = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxes.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms)}


# ------------------------------------------------------------------------------------------------
# CPU side: the reference's fp32 path (oracle), used for cpu_baseline and --impl reference
# ------------------------------------------------------------------------------------------------
def cpu_setup():
    import numpy as np
    import torch
    from oracle import s4ref
    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(0)
    deqs, packs, xs = {}, {}, {}
    for name, K, N in SHAPES:
        packed, scales = s4ref.config_weights(rng, K, N)
        deqs[name] = torch.from_numpy(s4ref.dequant(packed, scales))   # dequantised once (fake-quant)
        packs[name] = (torch.from_numpy(packed), torch.from_numpy(scales))
    for M in MS:
        for name, K, N in SHAPES:
            xs[(M, name)] = torch.from_numpy(s4ref.config_x(rng, M, K).astype(np.float32))
    return deqs, packs, xs


def cpu_sweep_once(deqs, xs):
    import torch
    with torch.inference_mode():
        for M in MS:
            for name, K, N in SHAPES:
                (xs[(M, name)] @ deqs[name].T).to(torch.float16)


def cpu_sweep_dequant_once(packs, xs):
    """The same sweep dequantising every weight inside each call (int4 bytes in, fp32 math)."""
    import torch
    from oracle import s4ref
    with torch.inference_mode():
        for M in MS:
            for name, K, N in SHAPES:
                (xs[(M, name)] @ s4ref.dequant_torch(*packs[name]).T).to(torch.float16)


def cpu_time(deqs, xs, seconds: float, sweep=cpu_sweep_once):
    sweep(deqs, xs)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        sweep(deqs, xs)
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            return n, dt


def cpu_prefill_baseline(seconds: float):
    """Configs 1 and 3 on the host cores: gate|up at M = 64 and gate|up / down at M = 2048, torch fp32
    on weights dequantised once (fake-quant route), each timed for a third of ``seconds``; TFLOP/s."""
    import numpy as np
    import torch
    from oracle import s4ref
    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(0)
    w = {}
    for name, K, N in (("gate_up", 2048, 12288), ("down", 6144, 2048)):
        packed, scales = s4ref.config_weights(rng, K, N)
        w[name] = s4ref.dequant_torch(packed, scales)
    out = {}
    with torch.inference_mode():
        for name, M in (("gate_up", 64), ("gate_up", 2048), ("down", 2048)):
            N, K = w[name].shape
            x = torch.from_numpy(s4ref.config_x(rng, M, K).astype(np.float32))
            (x @ w[name].T).half()  # warm
            n, t0 = 0, time.perf_counter()
            while True:
                (x @ w[name].T).half()
                n += 1
                dt = time.perf_counter() - t0
                if dt >= seconds / 3:
                    break
            out[f"{name}/M{M}"] = {"TFLOPs": round(2.0 * M * N * K * n / dt / 1e12, 3), "calls": n}
    return out


def cpu_stack_baseline(serve, seconds: float):
    """Configs 4/5 on the host cores, on a bounded sample: the stack's repeating 4-layer unit (three
    linear-attention layers sharing one set of weights, then an attention layer) over a 2048-token
    prompt, torch fp32 on weights dequantised once (fake-quant route, export_engine.py:88-103), with
    the residual add + RMSNorm (wgsl.js:55-78) and SiLU*mul (wgsl.js:81-90) in fp32 and fp16
    activations between ops, wired like ``serve.stack_forward``. The 24-layer stack repeats the unit
    six times, so its tokens/s is the unit's divided by six."""
    import torch
    from oracle import s4ref
    torch.set_num_threads(os.cpu_count() or 1)
    T, D = 2048, serve.HIDDEN
    weights = {}
    for kind, layer_idx in (("linear", 0), ("attn", 3)):
        weights[kind] = {}
        for name, K, N in serve.projection_shapes(kind):
            packed, scales = serve.synthetic_projection(serve.projection_seed(layer_idx, name), K, N)
            weights[kind][name] = s4ref.dequant_torch(packed, scales)  # [N, K] fp32

    def norm(x):
        return (x * torch.rsqrt((x * x).mean(1, keepdim=True) + 1e-6)).half()

    def layer(x, w):
        a = (norm(x).float() @ w["in_proj"].T).half()
        x = x + (a[:, :D].float() @ w["out_proj"].T).half().float()
        gu = (norm(x).float() @ w["gate_up"].T).half().float()
        g, u = gu[:, :gu.shape[1] // 2], gu[:, gu.shape[1] // 2:]
        return x + ((g / (1.0 + torch.exp(-g)) * u).half().float() @ w["down"].T).half().float()

    def unit(x):
        for kind in ("linear", "linear", "linear", "attn"):
            x = layer(x, weights[kind])
        return x

    x0 = torch.randn((T, D), generator=torch.Generator().manual_seed(0)).half().float()
    with torch.inference_mode():
        unit(x0)  # warm
        n, t0 = 0, time.perf_counter()
        while True:
            unit(x0)
            n += 1
            dt = time.perf_counter() - t0
            if dt >= seconds:
                break
    units = serve.N_LAYERS // 4
    return {"value": T * n / dt / units, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{n} passes of the stack's 4-layer unit (3 linear-attention + 1 attention layer) over a "
                      f"{T}-token prompt in {dt:.1f} s, torch fp32 on weights dequantised once (fake-quant route, "
                      f"export_engine.py:88-103); the 24-layer stack = {units} units"}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    deqs, _, xs = cpu_setup()
    for _ in range(args.warmup):
        cpu_sweep_once(deqs, xs)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_sweep_once(deqs, xs)
    dt = time.perf_counter() - t0
    gbs = sweep_bytes() * args.steps / dt / 1e9
    cores = os.cpu_count() or 1
    line = {
        "impl": "reference", "metric": "int4 GEMM GB/s (decode sweep M=1..8, algorithmic bytes)", "value": gbs,
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": bench_config(),
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} full sweeps (16 matmuls each), torch fp32 on dequantised weights"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------------
# GPU side
# ------------------------------------------------------------------------------------------------
def linear_stack_extras(args, ctx, rank, world, dev, barrier, max_over_ranks):
    """BASELINE configs 4 and 5 beside the decode headline, on the same ranks.

    * ``stack`` (config 4): one 2048-token prompt through the 24-layer linear stack, the whole
      forward replayed as one CUDA graph; on one GPU the plain stack, on N GPUs column-sharded with
      the all-gathers fused into the GEMM / SiLU*mul epilogues (peer stores over NVLink) and a flag
      barrier per projection (strong scaling: the same prompt whatever N is).
    * ``serve`` (config 5): the first ``--requests`` of the seeded 4096 requests, assigned to ranks
      longest-first (LPT), weights replicated, no collective (weak scaling of work per GPU); each
      rank runs its requests packed into chunks of at most 8192 tokens.
    Both are device-timed (CUDA events, max over ranks) after three warm-up steps."""
    import importlib

    import numpy as np
    import torch

    serve = importlib.import_module("strands_decider_web_b200.serve")
    stream = torch.cuda.current_stream(dev)
    flops_tok = serve.stack_flops_per_token()
    _, tc_peak, peak_kind = peaks()
    out = {}

    def timed(step, n_steps):
        for _ in range(3):
            step()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n_steps):
            step()
        b.record(stream)
        barrier()
        return max_over_ranks(a.elapsed_time(b))

    # ---- config 4: the 2048-token prompt ----
    x = torch.from_numpy(np.random.default_rng(0).standard_normal((2048, serve.HIDDEN)).astype(np.float16)).to(dev)
    fused, graph = None, None
    full = serve.CudaStack(ctx, fuse_silu=True)  # replicated weights: the one-GPU stack and config 5
    if world == 1:
        full.forward(x)
        torch.cuda.synchronize(dev)
        l0 = ctx.launch_count
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            full.forward(x)
        launches = ctx.launch_count - l0
        step = graph.replay
    else:
        fused = serve.FusedColshardStack(ctx, None, rank, world, fuse_silu=True)
        fused.forward(x)
        torch.cuda.synchronize(dev)
        l0 = ctx.launch_count
        fused.capture(x)
        launches = ctx.launch_count - l0
        step = fused.replay
    n_stack = max(1, min(args.steps, 20))
    ms = timed(step, n_stack)
    tok_s = 2048 * n_stack / (ms / 1e3)
    out["stack"] = {"workload": "config4_stack_2048_prompt", "value": tok_s, "unit": "tokens/s",
                    "ms_per_step": ms / n_stack, "steps": n_stack, "warmup": 3, "scaling": "strong",
                    "parallelism": "one GPU" if world == 1 else
                    f"colshard{world} (all-gathers fused into the GEMM / SiLU*mul epilogues, NVLink peer stores)",
                    "tflops": tok_s * flops_tok / 1e12, "tensor_frac": tok_s * flops_tok / 1e12 / tc_peak,
                    "peak_kind": peak_kind, "gpu_launches_per_step": launches, "cuda_graph": True}
    step = graph = None
    if fused is not None:
        fused.close()
        fused = None
    torch.cuda.synchronize(dev)

    # ---- config 5: batched data-parallel serving ----
    lengths = serve.request_lengths(4096)[: args.requests]
    mine = serve.lpt_shard(lengths, world)[rank]
    chunks = serve.pack_chunks(lengths[mine], 8192)
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    xs = [torch.randn((int(lengths[mine][c].sum()), serve.HIDDEN), generator=g, device=dev).to(torch.float16)
          for c in chunks]

    def serve_step():
        for xc in xs:
            full.forward(xc)
    n_serve = max(1, min(args.steps, 3))
    ms = timed(serve_step, n_serve)
    tokens = int(lengths.sum())
    tok_s = tokens * n_serve / (ms / 1e3)
    out["serve"] = {"workload": f"config5_serve_{args.requests}_requests_lpt", "value": tok_s, "unit": "tokens/s",
                    "ms_per_step": ms / n_serve, "steps": n_serve, "warmup": 3, "scaling": "weak",
                    "tokens_per_step": tokens, "parallelism": f"dp{world} (LPT request shards, no collective)",
                    "tflops": tok_s * flops_tok / 1e12, "tensor_frac": tok_s * flops_tok / 1e12 / (tc_peak * world),
                    "peak_kind": peak_kind}
    if ctx.check_errors():
        raise RuntimeError("device error word set during the stack / serving runs")
    del xs, full
    torch.cuda.synchronize(dev)
    return out


def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist
    from oracle import s4ref  # input generator only (same seeded synthetic data as the tests)

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    pkg = load_pkg()
    ctx = pkg.Context(local_rank)
    if args.family != "auto":
        ctx.force(args.family)
    stream = torch.cuda.current_stream(dev)

    rng = np.random.default_rng(0)
    Ws = {}
    for name, K, N in SHAPES:
        packed, scales = s4ref.config_weights(rng, K, N)
        Ws[name] = [ctx.upload(packed, scales, N, K) for _ in range(COPIES)]
    # all inputs of a sweep in one device buffer and all outputs in another (one copy each way for
    # the host-buffer run); every slice starts on a 16-byte boundary (K, N multiples of 8)
    keys = [(M, name, K, N) for M in MS for name, K, N in SHAPES]
    xbuf = torch.empty(sum(M * K for M, _, K, _ in keys), dtype=torch.float16, device=dev)
    ybuf = torch.empty(sum(M * N for M, _, _, N in keys), dtype=torch.float16, device=dev)
    xs, ys = {}, {}
    xo = yo = 0
    for M, name, K, N in keys:
        xs[(M, name)] = xbuf[xo:xo + M * K].view(M, K)
        xs[(M, name)].copy_(torch.from_numpy(s4ref.config_x(rng, M, K)))
        ys[(M, name)] = ybuf[yo:yo + M * N].view(M, N)
        xo += M * K
        yo += M * N
    counter = [0]

    def weight_for(name, rot, mi):
        return Ws[name][(rot * len(MS) + mi) % COPIES]

    # The engine submits a decode step's recorded matmul steps at once (engine.js:236-282); the
    # chained GEMV runs the 16 matmuls of one sweep step (on the step's weight copies) as ONE
    # persistent launch. One chain per weight rotation; consecutive steps alternate between two
    # bound buffer sets (inputs and outputs). The device-timed steps follow one another on one
    # stream as programmatic dependent launches: a step's CTAs start, and stream their first
    # weights, as the previous step's CTAs exit.
    sets = [(xbuf, ybuf)]
    for _ in range(NSETS - 1):
        sets.append((xbuf.clone(), torch.empty_like(ybuf)))
    chains = []
    for rot in range(COPIES):
        xb_, yb_ = sets[rot % NSETS]
        ops, xo, yo = [], 0, 0
        for mi, M in enumerate(MS):   # the slice order of xbuf / ybuf (M-major, then shape)
            for name, K, N in SHAPES:
                ops.append((xb_[xo:xo + M * K].view(M, K), weight_for(name, rot, mi), yb_[yo:yo + M * N].view(M, N)))
                xo += M * K
                yo += M * N
        chains.append(ctx.chain(ops))
    step_streams = [stream] + [torch.cuda.Stream(dev) for _ in range(NSETS - 1)]

    def sweep(rot: int, st):
        # the same 16 matmuls as one launch each (the per-call path, s4_matmul)
        for mi, M in enumerate(MS):
            for name, K, N in SHAPES:
                ctx.matmul(xs[(M, name)], weight_for(name, rot, mi), M, ys[(M, name)], st)

    # Steps are replayed from CUDA graphs so the host does not pace the GPU. The warm-up steps and
    # the timed steps are one graph each, holding exactly that many chained launches over the weight
    # rotations back to back, so consecutive steps overlap (programmatic dependent launch) across the
    # whole timed region whatever --steps is; call_graphs hold the 16 per-call launches of each
    # rotation for comparison.
    call_graphs = []
    cap_stream = torch.cuda.Stream(dev)
    cap_stream.wait_stream(stream)
    with torch.cuda.stream(cap_stream):
        for rot in range(COPIES):
            chains[rot].run(cap_stream)      # eager warm-up
            sweep(rot, cap_stream)
        cap_stream.synchronize()
        n0 = ctx.launch_count
        chains[0].run(cap_stream)
        launches_per_step = ctx.launch_count - n0
        cap_stream.synchronize()
        # the timed steps continue the warm-up's rotation, so the first timed step's weight copies are
        # not the ones the last warm-up step left in L2
        step_graphs = {}
        for n, start in ((args.warmup, 0), (args.steps, args.warmup)):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap_stream):
                for i in range(n):
                    chains[(start + i) % COPIES].run(cap_stream)
            step_graphs[(n, start)] = g
        for rot in range(COPIES):
            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2, stream=cap_stream):
                sweep(rot, cap_stream)
            call_graphs.append(g2)
    stream.wait_stream(cap_stream)
    graphs_uploaded = all([upload_graph(g, stream) for g in step_graphs.values()])
    torch.cuda.synchronize(dev)

    def steps_on_stream(k: int, start: int):
        with torch.cuda.stream(stream):
            step_graphs[(k, start)].replay()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the clock sampler starts (it waits for its first reading) before the warm-up, so the GPU is not
    # left idle, and clocking down, right before the timed steps
    with ClockSampler(local_rank) as clocks:
        steps_on_stream(args.warmup, 0)
        barrier()
        # A short device-side delay ahead of the start event keeps the GPU busy while the host submits
        # the event and the graph: the start timestamp is then taken when the GPU reaches the timed
        # steps, not while it sits idle waiting for the host's launch (tens of microseconds, which
        # would otherwise land inside the device-timed region).
        with torch.cuda.stream(stream):
            torch.cuda._sleep(LAUNCH_SHIELD_CYCLES)
        e0.record(stream)
        steps_on_stream(args.steps, args.warmup)
        e1.record(stream)
        barrier()
    launches = launches_per_step * args.steps   # kernels inside the replayed graphs
    ms = max_over_ranks(e0.elapsed_time(e1))
    errs = ctx.check_errors()
    if errs:
        raise RuntimeError(f"device error word 0x{errs:x} after the timed region")
    total_bytes = sweep_bytes() * args.steps * world
    value = total_bytes / (ms / 1e3) / 1e9

    # the same sweep as 16 separate launches (outside the timed region above)
    for r in range(args.warmup):
        call_graphs[r % COPIES].replay()
    barrier()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    for r in range(args.steps):
        call_graphs[r % COPIES].replay()
    c1.record(stream)
    barrier()
    per_launch_value = total_bytes / (max_over_ranks(c0.elapsed_time(c1)) / 1e3) / 1e9

    # ---- e2e: the same sweep through the host-buffer C-ABI entry point ------------------------------
    # Every step: its inputs from pinned host memory, one chained launch, its outputs back to pinned
    # host memory (s4_chain_run_host), on the stream of its buffer set (NSETS round robin), so a step's
    # copies overlap the following steps' launches and have NSETS - 1 steps to finish before their
    # buffers are reused. Each rotation's call is captured once in a CUDA graph (copies included) and
    # replayed, so the host's call rate does not pace the steps.
    hx = [xbuf.cpu().pin_memory() for _ in range(NSETS)]
    hy = [torch.empty(ybuf.shape, dtype=torch.float16).pin_memory() for _ in range(NSETS)]
    e2e_streams = step_streams
    e2e_graphs = []
    with torch.cuda.stream(cap_stream):
        for rot in range(COPIES):
            k = rot % NSETS
            chains[rot].run_host(hx[k], sets[k][0], hy[k], sets[k][1], cap_stream)  # eager once
            cap_stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap_stream):
                chains[rot].run_host(hx[k], sets[k][0], hy[k], sets[k][1], cap_stream)
            e2e_graphs.append(g)
    for g in e2e_graphs:
        upload_graph(g, stream)
    torch.cuda.synchronize(dev)

    def e2e_step():
        r = counter[0]
        with torch.cuda.stream(e2e_streams[r % NSETS]):
            e2e_graphs[r % COPIES].replay()
        counter[0] += 1

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    counter[0] = 0
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(LAUNCH_SHIELD_CYCLES)  # as for the device-timed steps
    e2.record(stream)
    for st_ in e2e_streams[1:]:
        st_.wait_event(e2)
    for _ in range(args.steps):
        e2e_step()
    for st_ in e2e_streams[1:]:
        stream.wait_stream(st_)
    e3.record(stream)
    barrier()
    ms_e2e = max_over_ranks(e2.elapsed_time(e3))
    e2e_value = total_bytes / (ms_e2e / 1e3) / 1e9
    h2d = hx[0].numel() * 2
    d2h = hy[0].numel() * 2

    # ---- parity of the timed configuration (outside the timed region): a chained run whose ops all
    # use copy 0 of their weight, every output against the oracle --------------------------------------
    rng2 = np.random.default_rng(0)
    wref = {name: s4ref.config_weights(rng2, K, N) for name, K, N in SHAPES}
    pchain = ctx.chain([(xs[(M, name)], Ws[name][0], ys[(M, name)]) for M in MS for name, _, _ in SHAPES])
    pchain.run(stream)
    torch.cuda.synchronize(dev)
    ok_all = True
    worst = 0.0
    for M in MS:
        for name, K, N in SHAPES:
            _, ref = s4ref.matmul(xs[(M, name)].cpu().numpy(), *wref[name])
            ok, mr, _ = s4ref.check(ys[(M, name)].cpu().numpy(), ref)
            ok_all &= ok
            worst = max(worst, mr)
    pchain.free()

    # ---- per-(shape, M) breakdown on this rank (device time, 8 rotating copies) -------------------------
    per = {}
    if rank == 0 and not args.quick:
        # each (shape, M) alone: a graph of 64 back-to-back calls over the 8 rotating copies
        for name, K, N in SHAPES:
            for M in MS:
                reps = 64
                g = torch.cuda.CUDAGraph()
                with torch.cuda.stream(cap_stream):
                    with torch.cuda.graph(g, stream=cap_stream):
                        for r in range(reps):
                            ctx.matmul(xs[(M, name)], Ws[name][r % COPIES], M, ys[(M, name)], cap_stream)
                torch.cuda.synchronize(dev)
                for _ in range(3):
                    g.replay()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(5):
                    g.replay()
                b.record(stream)
                torch.cuda.synchronize(dev)
                us = a.elapsed_time(b) * 1e3 / (5 * reps)
                gbs = alg_bytes(M, K, N) / (us * 1e-6) / 1e9
                per[f"{name}/M{M}"] = {"us": round(us, 3), "GBps": round(gbs, 1), "frac": round(gbs / peaks()[0], 3)}

    # ---- prefill / mid-M GEMMs (BASELINE configs 1 and 3), rank 0 ------------------------------------
    prefill = {}
    if rank == 0 and not args.quick:
        hbm_pk, tc_pk, _ = peaks()
        pre_shapes = {"down": (6144, 2048), "gate_up": (2048, 12288)}
        pre_w = {}
        rng_p = np.random.default_rng(0)
        for name, (K, N) in pre_shapes.items():
            # weights rotate over >= 8 device copies whose bytes exceed twice the L2, so every call
            # streams its weight from HBM (a weight of these shapes alone fits in the L2)
            packed, scales = s4ref.config_weights(rng_p, K, N)
            n_copies = max(8, -(-2 * L2_BYTES // (N * K // 2 + N * K // 16)))
            pd, sd = torch.from_numpy(packed).to(dev), torch.from_numpy(scales).to(dev)
            pre_w[name] = [ctx.upload(pd, sd, N, K) for _ in range(n_copies)]
            del pd, sd
        prefill_copies = {name: len(v) for name, v in pre_w.items()}
        for name, (K, N) in pre_shapes.items():
            nw = len(pre_w[name])
            for M in (16, 64, 128, 512, 2048):
                x = torch.from_numpy(s4ref.config_x(np.random.default_rng(M), M, K)).to(dev)
                y = torch.empty((M, N), dtype=torch.float16, device=dev)
                reps = max(nw, 8 if M >= 512 else 32)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.stream(cap_stream):
                    for r in range(2):
                        ctx.matmul(x, pre_w[name][r % nw], M, y, cap_stream)
                    cap_stream.synchronize()
                    with torch.cuda.graph(g, stream=cap_stream):
                        for r in range(reps):
                            ctx.matmul(x, pre_w[name][r % nw], M, y, cap_stream)
                torch.cuda.synchronize(dev)
                g.replay()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(3):
                    g.replay()
                b.record(stream)
                torch.cuda.synchronize(dev)
                us = a.elapsed_time(b) * 1e3 / (3 * reps)
                flops = 2.0 * M * N * K
                tfs = flops / (us * 1e-6) / 1e12
                gbs = alg_bytes(M, K, N) / (us * 1e-6) / 1e9
                fam, tile, split = ctx.plan(M, N, K)
                prefill[f"{name}/M{M}"] = {"us": round(us, 2), "TFLOPs": round(tfs, 1), "GBps": round(gbs, 1),
                                           "tensor_frac": round(tfs / tc_pk, 3), "hbm_frac": round(gbs / hbm_pk, 3),
                                           "family": fam, "tile": tile, "split": split}
                del g
        for ws_ in pre_w.values():
            for W in ws_:
                W.free()
        prefill["weight_copies"] = prefill_copies
        prefill["l2"] = "each call streams its weight from HBM: rotation over device copies totalling > 2x L2"

    # ---- BASELINE configs 4 and 5 on the same ranks (extra keys of the line) ---------------------------
    extras = {}
    if not args.quick and not args.no_stack:
        extras = linear_stack_extras(args, ctx, rank, world, dev, barrier, max_over_ranks)

    # ---- CPU baseline (rank 0, N = 1 only) ------------------------------------------------------------
    hbm, bf16, peak_kind = peaks()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        deqs, packs, cxs = cpu_setup()
        n, dt = cpu_time(deqs, cxs, args.cpu_seconds)
        n2, dt2 = cpu_time(packs, cxs, args.cpu_seconds / 2, cpu_sweep_dequant_once)
        cpu = {"value": sweep_bytes() * n / dt / 1e9, "unit": "GB/s", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"{n} full sweeps (16 matmuls each) in {dt:.1f} s, torch fp32 on weights dequantised once "
                         f"(fake-quant route, export_engine.py:88-103)",
               "dequant_per_call": {"value": sweep_bytes() * n2 / dt2 / 1e9, "unit": "GB/s",
                                    "sample": f"{n2} full sweeps in {dt2:.1f} s, every weight dequantised from its "
                                              f"int4 bytes inside each call, then the same fp32 matmul"},
               "prefill": cpu_prefill_baseline(args.cpu_seconds / 2)}

    if rank == 0:
        per_launch_bytes = sweep_bytes()  # one chained launch moves the whole sweep
        avg_launch_us = ms / args.steps * 1e3
        achieved = per_launch_bytes / (avg_launch_us * 1e-6) / 1e9
        line = {
            "metric": "int4 GEMM GB/s (decode sweep M=1..8, algorithmic bytes)",
            "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16", "data": "synthetic",
            "config": bench_config(),
            "setup": {"launch": "the 16 matmuls of a step as one chained launch; the timed steps are one CUDA "
                                "graph of that many launches back to back on one stream (programmatic dependent "
                                "launch), uploaded to the device before the timed region",
                      "graph_uploaded": graphs_uploaded,
                      "weight_copies": COPIES,
                      "l2": "inputs larger than L2: 8 rotating weight copies (272 MB) per step sequence",
                      "parallelism": f"dp{world} (weights replicated, no collective)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": profile_traffic(), "peak_kind": peak_kind,
                         "kernel": "chain_kernel", "launch_us_avg": avg_launch_us},
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "s4_chain_run_host every step (pinned host x -> device, one chained launch, device -> "
                           "pinned host y), each rotation's call replayed from a CUDA graph; steps round robin over "
                           "four streams with four bound buffer sets"},
            "per_launch_sweep": {"value": per_launch_value, "unit": "GB/s",
                                 "note": "the same 16 matmuls as 16 s4_matmul launches (decode GEMV kernel)"},
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "parity": {"ok": bool(ok_all), "max_rel": worst, "tol": s4ref.TOL_MAX_REL},
            "per_call": per,
            "prefill": prefill,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    del step_graphs, call_graphs, e2e_graphs
    for ch in chains:
        ch.free()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_stack(args, rank, world, local_rank):
    """Configs 4 and 5 on the 24-layer linear stack (strands-decider-web_b200/serve.py)."""
    import datetime
    import importlib

    import numpy as np
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    pkg = load_pkg()
    serve = importlib.import_module("strands_decider_web_b200.serve")
    ctx = pkg.Context(local_rank)
    stream = torch.cuda.current_stream(dev)
    flops_tok = serve.stack_flops_per_token()
    _, tc_peak, peak_kind = peaks()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    gather_ms = [0.0]
    fused = None
    if args.workload == "stack":
        if args.gather == "fused":
            fused = serve.FusedColshardStack(ctx, None, rank, world, fuse_silu=bool(args.fuse_silu))
            stack = fused.stack
        else:
            stack = serve.CudaStack(ctx, rank=rank, world=world, fuse_silu=bool(args.fuse_silu),
                                    fuse_norm=bool(args.fuse_norm))
        x = torch.from_numpy(np.random.default_rng(0).standard_normal((2048, serve.HIDDEN)).astype(np.float16)).to(dev)
        timing = {"on": False}

        def timers(kind, fn):
            if not timing["on"]:
                return fn()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            out = fn()
            b.record(stream)
            timing["events"].append((a, b))
            return out

        def eager():
            if fused is not None:
                return fused.forward(x)
            return stack.forward(x, timers=timers)
        step = eager
        tokens_per_step = 2048 * 1  # the prompt, whatever the number of ranks (strong scaling)
        label = f"config4_stack_2048_prompt_colshard_{args.gather}"
    else:
        # weights replicated on every rank
        stack = serve.CudaStack(ctx, fuse_silu=bool(args.fuse_silu), fuse_norm=bool(args.fuse_norm))
        lengths = serve.request_lengths(4096)[: args.requests]
        mine = serve.lpt_shard(lengths, world)[rank]
        chunks = serve.pack_chunks(lengths[mine], 8192)
        xs = []
        g = torch.Generator(device=dev)
        g.manual_seed(1234 + rank)
        for c in chunks:
            n = int(lengths[mine][c].sum())
            xs.append(torch.randn((n, serve.HIDDEN), generator=g, device=dev).to(torch.float16))

        def step():
            for xc in xs:
                stack.forward(xc)
        tokens_per_step = int(lengths.sum())
        label = f"config5_serve_{args.requests}_requests_lpt"
        timers = None

    for _ in range(args.warmup):
        step()
    barrier()
    graph = None
    launches_per_step = None
    if args.workload == "stack" and args.graph:
        # the whole forward (GEMMs, norms, SiLU*mul, barriers or NCCL all-gathers) as one CUDA graph
        l0 = ctx.launch_count
        if fused is not None:
            fused.capture(x)
            step = fused.replay
        else:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                stack.forward(x)
            step = graph.replay
        launches_per_step = ctx.launch_count - l0
        for _ in range(args.warmup):
            step()
        barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ctx.launch_count
    with ClockSampler(local_rank) as clocks:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        barrier()
    launches = ctx.launch_count - launches0
    if launches_per_step is not None:
        launches = launches_per_step * args.steps
    ms = max_over_ranks(e0.elapsed_time(e1))
    comm_share = None
    if args.workload == "stack" and world > 1 and fused is None:
        # NCCL all-gather share of one eager step (events around each all-gather), outside the timed region
        timing.update(on=True, events=[])
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        a.record(stream)
        eager()
        b.record(stream)
        barrier()
        timing["on"] = False
        gather_ms = sum(p.elapsed_time(q) for p, q in timing["events"])
        comm_share = max_over_ranks(gather_ms / a.elapsed_time(b))
    tok_s = tokens_per_step * args.steps / (ms / 1e3)
    tflops = tok_s * flops_tok / 1e12
    if ctx.check_errors():
        raise RuntimeError("device error word set during the stack run")
    if rank == 0:
        line = {
            "metric": "prefill tokens/s through the 24-layer int4 linear stack",
            "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16", "data": "synthetic",
            "config": {"workload": label, "layers": 24, "hidden": serve.HIDDEN, "intermediate": serve.INTER,
                       "parallelism": ((f"colshard{world} (all-gathers fused into the GEMM/SiLU epilogues, NVLink peer stores)"
                                        if args.gather == "fused" else f"colshard{world} (NCCL all-gather after every projection)")
                                       if args.workload == "stack" else f"dp{world} (LPT request sharding, no collective)"),
                       "l2": "weights 758 MB > L2"},
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": tflops / tc_peak, "traffic": None, "peak_kind": peak_kind,
                         "note": "whole-stack FLOP rate (2 x weight parameters per token), all kernels included"},
            "gather_share": comm_share,
            "cuda_graph": bool(args.workload == "stack" and args.graph),
            "silu_mul": "in the gate|up GEMM epilogue" if args.fuse_silu else "separate kernel",
            "add_norm": ("residual add in the out_proj / down GEMM epilogue, one row pass"
                         if args.fuse_norm and not (args.workload == "stack" and args.gather == "fused")
                         else "separate kernel"),
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_stack_baseline(serve, args.cpu_seconds / 2)
        print(json.dumps(line), flush=True)
    # a graph that holds NCCL calls must be gone before destroy_process_group (the bound replay
    # method in `step` keeps it alive too)
    step = graph = None
    torch.cuda.synchronize(dev)
    if fused is not None:
        fused.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


GEMM_SHAPES = {"qkvz_ab": (2048, 8224), "attn_qkv": (2048, 3072), "gate_up": (2048, 12288), "down": (6144, 2048),
               "out_proj": (2048, 2048)}


def run_gemm(args, rank, world, local_rank):
    """One (shape, M) matmul through s4_matmul (BASELINE configs 1 and 3), back to back over rotating
    device copies of the weight whose bytes exceed twice the L2, replayed from one CUDA graph per
    step of 64 calls: GB/s and TFLOP/s of the algorithmic work. The small, single-kernel command the
    ncu captures of the mid-M and prefill kernels run."""
    import numpy as np
    import torch
    from oracle import s4ref

    if world > 1:
        print(json.dumps({"workload": "gemm", "skipped": "single-GPU measurement"}) if rank == 0 else "")
        return 0
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pkg = load_pkg()
    ctx = pkg.Context(local_rank)
    K, N = GEMM_SHAPES[args.shape]
    M = args.m
    rng = np.random.default_rng(0)
    packed, scales = s4ref.config_weights(rng, K, N)
    copies = max(8, -(-2 * L2_BYTES // (N * K // 2 + N * K // 16)))
    pd, sd = torch.from_numpy(packed).to(dev), torch.from_numpy(scales).to(dev)
    Ws = [ctx.upload(pd, sd, N, K) for _ in range(copies)]
    x = torch.from_numpy(s4ref.config_x(rng, M, K)).to(dev)
    y = torch.empty((M, N), dtype=torch.float16, device=dev)
    reps = 64
    lib = pkg.load_library()

    def call(r):
        if args.noalloc:  # the allocation-free entry point (static scratch, no context)
            rc = lib.s4_matmul_noalloc(Ws[r % copies].handle, x.data_ptr(), M, y.data_ptr(),
                                       torch.cuda.current_stream(dev).cuda_stream)
            if rc:
                raise RuntimeError(lib.s4_last_error().decode())
        else:
            ctx.matmul(x, Ws[r % copies], M, y)
    call(0)  # the allocation-free entry point's first call looks up its scratch (outside capture)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for r in range(reps):
            call(r)
    stream = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize(dev)
        a.record(stream)
        for _ in range(args.steps):
            g.replay()
        b.record(stream)
        torch.cuda.synchronize(dev)
    us = a.elapsed_time(b) * 1e3 / (args.steps * reps)
    _, ref = s4ref.matmul(x.cpu().numpy(), packed, scales)
    ok, mr, mc = s4ref.check(y.cpu().numpy(), ref)
    hbm, tc_peak, peak_kind = peaks()
    alg = N * K // 2 + N * K // 16 + 2 * M * K + 2 * M * N
    fam, tile, split = ctx.plan(M, N, K)
    print(json.dumps({"workload": "gemm", "entry": "s4_matmul_noalloc" if args.noalloc else "s4_matmul",
                      "shape": args.shape, "K": K, "N": N, "M": M, "us": us,
                      "GBps": alg / us / 1e3, "TFLOPs": 2.0 * M * N * K / us / 1e6,
                      "hbm_frac": alg / us / 1e3 / hbm, "tensor_frac": 2.0 * M * N * K / us / 1e6 / tc_peak,
                      "peak_kind": peak_kind, "family": fam, "tile": tile, "split": split, "weight_copies": copies,
                      "calls_per_step": reps, "steps": args.steps, "warmup": args.warmup,
                      "parity": {"ok": bool(ok), "max_rel": mr, "min_cos": mc}, "clocks": clk.summary()}))
    if ctx.check_errors():
        raise RuntimeError("device error word set")
    del g
    ctx.close()
    return 0


# formats: the non-default weight formats, the online FWHT and the wire scale decode, measured
FORMATS = [(4, 32, False), (2, 32, False), (3, 32, False), (4, 64, False), (2, 64, True), (4, 32, True),
           (3, 64, True)]


def format_bytes(K, N, bits, group, asym):
    """Bytes of one weight in its own format (q words + fp16 scales [+ fp16 biases])."""
    return N * K * bits // 8 + (N * K // group) * 2 * (2 if asym else 1)


def run_formats(args, rank, world, local_rank):
    """Decode (M = 1, GEMV) and prefill (M = 2048, tcgen05) matmuls of the gate|up shape for every
    weight format, the FWHT of a 2048 x 2048 activation in 256-blocks, and the device decode of
    wire-format scales for that weight. Weights rotate over 16 copies (> L2) for the decode calls."""
    import numpy as np
    import torch
    from oracle import s4ref

    if world > 1:
        print(json.dumps({"workload": "formats", "skipped": "single-GPU measurement"}) if rank == 0 else "")
        return 0
    torch.cuda.set_device(local_rank)
    pkg = load_pkg()
    ctx = pkg.Context(local_rank)
    hbm, tc_peak, peak_kind = peaks()
    stream = torch.cuda.current_stream()
    K, N = 2048, 12288
    rng = np.random.default_rng(5)
    copies = 16

    def timed(fn, reps):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps  # us per call

    rows = []
    x1 = torch.from_numpy(s4ref.config_x(rng, 1, K)).cuda()
    xp = torch.from_numpy(s4ref.config_x(rng, 2048, K)).cuda()
    y1 = torch.empty((1, N), dtype=torch.float16, device="cuda")
    yp = torch.empty((2048, N), dtype=torch.float16, device="cuda")
    with ClockSampler(local_rank) as clk:
        for bits, group, asym in FORMATS:
            words = s4ref.pack_format(rng.integers(0, 2 ** bits, (N, K)), bits)
            sc = (np.abs(rng.standard_normal((N, K // group))) * 0.02 / 2 ** (bits - 1)).astype(np.float16)
            bi = (-(2 ** bits - 1) / 2 * sc).astype(np.float16) if asym else None
            # symmetric 2-bit: with the native 2-bit decode layout, so decode streams 2-bit bytes
            Ws = [ctx.upload_format(words, sc, N, K, bits, group, bias=bi, decode_layout=bits == 2 and not asym)
                  for _ in range(copies)]
            it = {"i": 0}

            def dec():
                ctx.matmul(x1, Ws[it["i"] % copies], y=y1, stream=stream)
                it["i"] += 1

            us_dec = timed(dec, 20 * copies)
            us_pre = timed(lambda: ctx.matmul(xp, Ws[0], y=yp, stream=stream), 20)
            fb = format_bytes(K, N, bits, group, asym)
            # bytes a decode call streams: the native 2-bit layout for symmetric 2-bit weights, the
            # int4 layout otherwise (+ the scales, + the biases of an asymmetric format)
            chunks = -(-N // 128) * -(-K // 64)
            streamed = chunks * ((2048 if bits == 2 and not asym else 4096) + 512 * (2 if asym else 1))
            rows.append({"format": f"{bits}b g{group} {'asym' if asym else 'sym'}",
                         "decode_us": round(us_dec, 2),
                         "decode_format_GBps": round((fb + 2 * K + 2 * N) / us_dec / 1e3, 1),
                         "decode_device_GBps": round((streamed + 2 * K + 2 * N) / us_dec / 1e3, 1),
                         "prefill_us": round(us_pre, 1),
                         "prefill_TFLOPs": round(2.0 * 2048 * K * N / us_pre / 1e6, 1)})
            for W in Ws:
                W.free()
        a = torch.from_numpy(s4ref.config_x(rng, 2048, 2048)).cuda()
        us_fwht = timed(lambda: ctx.fwht(a, 256, stream=stream), 50)
        G = K // 32
        wire = torch.frombuffer(bytearray(s4ref.encode_wire_scales(
            (rng.standard_normal((N, G)) * 0.01).astype(np.float16))), dtype=torch.uint8).cuda()
        out = torch.empty((N, G), dtype=torch.float16, device="cuda")
        us_wire = timed(lambda: ctx.decode_wire_scales(wire, N, G, out=out, stream=stream), 50)
    line = {"workload": "formats", "shape": {"K": K, "N": N, "decode_M": 1, "prefill_M": 2048},
            "weight_copies": copies, "rows": rows,
            "fwht": {"M": 2048, "K": 2048, "n": 256, "us": round(us_fwht, 2),
                     "GBps": round(2 * 2 * 2048 * 2048 / us_fwht / 1e3, 1)},
            "wire_decode": {"N": N, "G": G, "us": round(us_wire, 2),
                            "GBps": round((4 * N + 3 * N * G) / us_wire / 1e3, 1)},
            "peaks": {"hbm_GBps": hbm, "bf16_TFLOPs": tc_peak, "kind": peak_kind},
            "clocks": clk.summary()}
    print(json.dumps(line))
    ctx.close()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--quick", action="store_true", help="skip the per-call breakdown, prefill, stack and serving")
    ap.add_argument("--no-stack", action="store_true", help="skip the stack and serving keys of the decode line")
    ap.add_argument("--family", choices=["auto", "gemv", "tc"], default="auto",
                    help="pin the kernel family instead of the dispatch table")
    ap.add_argument("--workload", choices=["decode", "stack", "serve", "formats", "gemm"], default="decode",
                    help="decode: configs[1] GEMV sweep (default); stack: config 4, one 2048-token prompt "
                         "through the 24-layer linear stack, column-sharded over the ranks; serve: config 5, "
                         "requests sharded over the ranks (weights replicated); formats: the non-default weight "
                         "formats, FWHT and wire scale decode (one GPU); gemm: one (--shape, --m) matmul back to "
                         "back (one GPU)")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="stack: fuse the all-gathers into the producing kernels (peer stores over NVLink) or "
                         "call NCCL all-gather after every projection")
    ap.add_argument("--graph", type=int, default=1,
                    help="stack: replay the whole forward as one CUDA graph (1, default) or launch eagerly (0)")
    ap.add_argument("--fuse-silu", type=int, default=1,
                    help="stack/serve: SiLU*mul in the gate|up GEMM epilogue (1, default) or as its own kernel (0)")
    ap.add_argument("--fuse-norm", type=int, default=0,
                    help="stack/serve on one GPU: the residual add of out_proj / down in the GEMM epilogue "
                         "(s4_matmul_add_rmsnorm, 1) or the separate ADD_NORM kernel (0, default)")
    ap.add_argument("--shape", choices=sorted(GEMM_SHAPES), default="gate_up", help="gemm: the projection shape")
    ap.add_argument("--m", type=int, default=64, help="gemm: tokens per call")
    ap.add_argument("--noalloc", action="store_true", help="gemm: time s4_matmul_noalloc instead of s4_matmul")
    ap.add_argument("--requests", type=int, default=512,
                    help="serve: number of config-5 requests timed per step (the first n of the seeded 4096)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # timing rules: at least 3 untimed warm-up steps
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world == 1 and args.gpus > 1:
        print(f"--gpus {args.gpus} needs torchrun with {args.gpus} processes", file=sys.stderr)
        return 2
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.workload in ("stack", "serve"):
        return run_stack(args, rank, world, local_rank)
    if args.workload == "formats":
        return run_formats(args, rank, world, local_rank)
    if args.workload == "gemm":
        return run_gemm(args, rank, world, local_rank)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
