"""Benchmark of basal's quantised-linear hot path on B200: BASELINE config 2, one decoder layer's projection set with
FP8-block W8A8 over 64 varlen-packed requests (lengths uniform in [128, 2048], seed 0), hidden 2048:
qkv [2048 -> 5120], o [2048 -> 2048], gate/up [2048 -> 12288], down [6144 -> 2048].

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step = the four projections (activation quantiser + tcgen05 block GEMM each) over the packed rows. Metric:
TFLOP/s (2 M N K summed over the projections), whole job: with N GPUs every rank serves its own 64 requests (row
shards of independent requests, no collective; "weak" scaling) and the value is all ranks' FLOPs over the slowest
rank's device time. One JSON line on rank 0 with, besides the contract keys:
  roofline      the FP8 block GEMM (the dominant kernel): achieved TFLOP/s from CUDA events around its launches in
                the timed steps, against 2 x the measured dense bf16 peak (FP8 is twice bf16 on B200): the burst
                figure, unless the clock samples of the timed region show the power cap holding the median SM clock
                below its maximum (then the sustained figure, the one measured under that cap); the fraction of the
                other figure is reported beside it
  e2e           the same metric through the public API (BlockFP8Linear modules) from pinned host memory: the H2D copy
                of the step's activations and the D2H copy of its four outputs inside the timed region, on their
                own streams so that the two PCIe directions and the GPU work of neighbouring steps overlap
  cpu_baseline  the reference's CPU maths (oracle/, numpy + BLAS on all host threads) on a bounded sample of rows
  clocks        nvidia-smi samples taken during the timed region
  decisions     the metric's second half: a random-init 32-layer Gated DeltaNet / attention hybrid
                (hidden 2560, every linear FP8-block, basal_b200.hybrid) answering 4096 decision requests, each a
                shared 1024-token prefix + 256 random suffix tokens, read out over 8 options; the requests are
                row-sharded across the ranks (strong scaling: 4096 in all), each GPU computes the prefix once;
                decisions/s = 4096 / the slowest rank's time, with the suffix ids copied in from pinned host memory and
                the probabilities copied back inside the timed region
--impl reference times the reference's CPU implementation of the path (the oracle port) on this box's host cores
(the reference has no native code, and its only B200 GPU path is a Triton kernel), rank 0 only.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "block-scaled GEMM TFLOP/s (% tcgen05 peak); decisions/s at 1/2/4/8 B200"
PROJ = (("qkv", 5120, 2048), ("o", 2048, 2048), ("gate_up", 12288, 2048), ("down", 2048, 6144))
HIDDEN, INTER = 2048, 6144
WORKLOAD = ("C2: one decoder layer's projection set, FP8-block W8A8, 64 varlen-packed requests (lengths U[128,2048], "
            "seed 0), qkv 2048->5120, o 2048->2048, gate/up 2048->12288, down 6144->2048")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
PROFILE = os.path.join(ROOT, "profiles", "fp8_block_gemm_c2.txt")


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS, source="fallback")


def profiled_traffic():
    """DRAM bytes per GEMM launch of the committed ncu summary (its 'traffic_bytes_per_launch:' line), or None."""
    try:
        with open(PROFILE) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].split()[0])
    except (OSError, ValueError):
        pass
    return None


def workload_rows():
    from basal_b200.shard import varlen_lengths
    return int(varlen_lengths(64, 128, 2048, seed=0).sum())


def flops_per_row():
    return sum(2 * n * k for _, n, k in PROJ)


class ClockSampler:
    """nvidia-smi clock / throttle samples every 20 ms while running (started before, stopped after the timed
    region)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc = index, None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = [r.split(", ") for r in self.out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(rows[0][2]),
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------------------------------------------
# CPU: the reference's maths (oracle port), a bounded sample of rows
# ------------------------------------------------------------------------------------------------------------------
def cpu_sample(rows, seed=0):
    """Seeded bf16-valued activations of `rows` tokens and the four quantised weights, as numpy (oracle inputs)."""
    import numpy as np
    from oracle import blockquant as obq
    rng = np.random.default_rng(seed)
    bf = lambda a: (a.astype(np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)  # noqa: E731 (truncate)
    xs = {HIDDEN: bf(rng.standard_normal((rows, HIDDEN))), INTER: bf(rng.standard_normal((rows, INTER)))}
    ws = {name: obq.quantize(rng.standard_normal((n, k)).astype(np.float32) * np.float32(0.02), "fp8")
          for name, n, k in PROJ}
    return xs, ws


def cpu_step(xs, ws):
    """One step of the reference's CPU path: per projection, act_quant_ops + reference() (both operands dequantised
    every call, an fp32 matmul), as fp8block.linear runs on CPU tensors (basal/fp8block.py:74-85)."""
    from oracle import blockquant as obq
    out = []
    for name, n, k in PROJ:
        q, s = ws[name]
        out.append(obq.linear(xs[k], q, s, "fp8"))
    return out


def blas_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else os.cpu_count()
    except Exception:
        return os.cpu_count()


def cpu_baseline(rows=1024, reps=3):
    xs, ws = cpu_sample(rows)
    cpu_step(xs, ws)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        cpu_step(xs, ws)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(rows * flops_per_row() / t / 1e12, 4), "unit": "TFLOP/s", "cores": blas_threads(),
            "kind": "port", "sample": f"{rows} rows of the C2 workload through the 4 projections, median of {reps} "
                                      f"steps ({t:.2f} s a step)"}


def run_reference(args, rank):
    if rank != 0:
        return
    rows = 256
    xs, ws = cpu_sample(rows)
    for _ in range(args.warmup):
        cpu_step(xs, ws)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(xs, ws)
    dt = (time.perf_counter() - t0) / args.steps
    value = rows * flops_per_row() / dt / 1e12
    cores = blas_threads()
    line = {"metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e4m3 (dequantised to fp32 on the CPU)", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "rows_per_step": rows, "parallelism": "rank 0 only, host cores"},
            "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                             "sample": f"{rows} rows of the C2 workload through the 4 projections each step"},
            "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------------------------
# GPU
# ------------------------------------------------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import basal_b200 as b2
    from basal_b200 import shard

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    M = workload_rows()
    g = torch.Generator(device=dev).manual_seed(1000 + rank)  # each rank serves its own requests
    xs = {HIDDEN: torch.randn(M, HIDDEN, device=dev, generator=g).bfloat16(),
          INTER: torch.randn(M, INTER, device=dev, generator=g).bfloat16()}
    mods = {}
    for name, n, k in PROJ:
        lin = torch.nn.Linear(k, n, bias=False, device=dev)
        with torch.no_grad():
            lin.weight.normal_(0.0, 0.02, generator=g)
        mods[name] = b2.fp8block.BlockFP8Linear.of(lin)
        del lin
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()

    def step(ev=None):
        outs = []
        for i, (name, n, k) in enumerate(PROJ):
            m = mods[name]
            q, s = b2.ops.fp8_act_quant(xs[k])
            if ev is not None:
                ev[i][0].record(stream)
            outs.append(b2.ops.fp8_block_gemm(q, s, m.weight, m.weight_scale, torch.bfloat16))
            if ev is not None:
                ev[i][1].record(stream)
        return outs

    for _ in range(args.warmup):
        step()
    K = args.steps
    evs = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in PROJ]
           for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    shard.check_peers(tag="timed")
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        start.record(stream)
        for i in range(K):
            step(evs[i])
        end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end) / K
    ms_max = shard.max_over_ranks(ms)
    gemm_ms = [sum(evs[i][j][0].elapsed_time(evs[i][j][1]) for i in range(K)) / K for j in range(len(PROJ))]
    total_rows = shard.sum_over_ranks(M)
    value = total_rows * flops_per_row() / (ms_max * 1e-3) / 1e12

    # end to end through the public API: pinned host activations in, the four outputs back to pinned host memory,
    # pipelined as a server would run it: step i + 1's inputs go up on one stream (two device buffers) while step i
    # computes on the compute stream, and each projection's output goes down on a third stream as soon as it is
    # written, so the two PCIe directions and the GPU work overlap. Every copy of every step is in the timed region.
    hx = {k: v.cpu().pin_memory() for k, v in xs.items()}
    hy = {name: torch.empty(M, n, dtype=torch.bfloat16).pin_memory() for name, n, _ in PROJ}
    h2d = sum(t.numel() * t.element_size() for t in hx.values())
    d2h = sum(t.numel() * t.element_size() for t in hy.values())
    dx = [{k: torch.empty_like(v, device=dev) for k, v in hx.items()} for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    freed = [torch.cuda.Event(), torch.cuda.Event()]  # the compute stream is done reading dx[b]
    for ev in freed:
        ev.record(stream)

    def e2e_step(i):
        b = i % 2
        landed = torch.cuda.Event()
        with torch.cuda.stream(s_in):
            s_in.wait_event(freed[b])
            for k in hx:
                dx[b][k].copy_(hx[k], non_blocking=True)
            landed.record(s_in)
        stream.wait_event(landed)
        for name, n, k in PROJ:
            y = mods[name](dx[b][k])
            done = torch.cuda.Event()
            done.record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                hy[name].copy_(y, non_blocking=True)
                y.record_stream(s_out)
        freed[b].record(stream)

    e2e_steps = max(1, min(K, 20))
    for i in range(2):
        e2e_step(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(s_in)
    for i in range(e2e_steps):
        e2e_step(i)
    s_out.wait_stream(stream)
    s_out.wait_stream(s_in)
    e2.record(s_out)
    torch.cuda.synchronize()
    e2e_ms = shard.max_over_ranks(s2.elapsed_time(e2) / e2e_steps)
    e2e_value = total_rows * flops_per_row() / (e2e_ms * 1e-3) / 1e12

    clocks = clk.summary()
    pk = peaks()
    # the O projection with the attention width as its K (32 heads x 128 = 4096; the config states K = 2048 and the
    # step above uses that): 20 GEMM launches on the same rows after 3 untimed ones, outside the timed step
    x4 = torch.randn(M, 4096, device=dev, generator=g).bfloat16()
    lin4 = torch.nn.Linear(4096, HIDDEN, bias=False, device=dev)
    with torch.no_grad():
        lin4.weight.normal_(0.0, 0.02, generator=g)
    o4 = b2.fp8block.BlockFP8Linear.of(lin4)
    q4, s4 = b2.ops.fp8_act_quant(x4)
    for _ in range(3):
        b2.ops.fp8_block_gemm(q4, s4, o4.weight, o4.weight_scale, torch.bfloat16)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(20):
        b2.ops.fp8_block_gemm(q4, s4, o4.weight, o4.weight_scale, torch.bfloat16)
    e1.record(stream)
    torch.cuda.synchronize()
    o4_tflops = 2 * M * HIDDEN * 4096 / (e0.elapsed_time(e1) / 20 * 1e-3) / 1e12
    del x4, q4, s4, o4, lin4

    del xs, mods, hx, hy, dx
    torch.cuda.empty_cache()
    decisions = run_decisions(rank, world, local_rank) if not args.no_decisions else None

    gemm_flops = sum(2 * M * n * k for _, n, k in PROJ)
    achieved = gemm_flops / (sum(gemm_ms) * 1e-3) / 1e12
    # the denominator follows the clocks sampled in the timed region: the sustained peak was measured under the
    # power cap, the burst peak at full clock; a region the cap did not touch is held to the burst figure
    capped = ("sw_power_cap" in clocks.get("reasons", []) and clocks.get("sm_mhz") is not None
              and clocks["sm_mhz"] < 0.97 * clocks["sm_max_mhz"])  # the cap active AND holding the clock down
    peak_burst, peak_sust = 2.0 * pk["bf16_tflops"], 2.0 * pk["bf16_tflops_sustained"]
    peak = peak_sust if capped else peak_burst
    traffic = profiled_traffic()
    if rank == 0:
        cpu = cpu_baseline() if world == 1 else None
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e4m3", "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights)",
            "config": {"workload": WORKLOAD, "rows_per_rank": M, "total_rows": int(total_rows),
                       "parallelism": f"{world} row-sharded replicas, no collective",
                       "l2": "inputs larger than L2 (285 MB + 855 MB activations a step), no flush"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": "basal200 fp8 block GEMM (tcgen05 kind::f8f6f4)",
                         "peak_source": (f"2 x {'bf16_tflops_sustained' if capped else 'bf16_tflops'} of "
                                         f"{pk['source']} peaks (FP8 dense = 2 x bf16 dense; "
                                         f"{'the power cap held the median SM clock down' if capped else 'median SM clock at its maximum'} "
                                         "in the clock samples of the timed region)"),
                         "frac_of_burst_peak": round(achieved / peak_burst, 4),
                         "frac_of_sustained_peak": round(achieved / peak_sust, 4),
                         "per_projection_tflops": {name: round(2 * M * n * k / (t * 1e-3) / 1e12, 1)
                                                   for (name, n, k), t in zip(PROJ, gemm_ms)},
                         "o_k4096_tflops": round(o4_tflops, 1)},
            "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "path": "BlockFP8Linear.forward on pinned host activations, outputs copied back; input, "
                            "compute and output copies on three streams, overlapped across steps"},
            "gpu_launches": 2 * len(PROJ) * K,
            "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if decisions is not None:
            if world == 1:
                decisions["cpu_baseline"] = c5_cpu_baseline()
            line["decisions"] = decisions
        print(json.dumps(line), flush=True)


CASES = {
    # name: (format, M, N, K) -- the small cases the committed ncu summaries were captured on (inputs > L2, a few
    # GB on the device): 2 untimed launches, then 3 launches of the kernel under study
    "fp8_gemm": ("fp8", 65536, 5120, 2048),
    "fp8_gemm_few": ("fp8", 16, 12288, 2048),  # the few-rows (weight-streaming) kernel; ncu flushes L2 per pass
    "fp8_gemm_split": ("fp8", 16, 2048, 6144),  # the few-rows GEMM split over the SMs (products + ordered sum)
    "int8_gemm": ("int8", 65536, 5120, 2048),
    "fp8_act_quant": ("fp8", 65536, 0, 2048),
    "nvfp4_gemm": ("nvfp4", 65536, 5120, 2048),
    "nvfp4_act_quant": ("nvfp4", 8192, 0, 6144),
    "readout": ("readout", 256, 255, 2048),  # C4's readout: R prompts, k option ids (N), D features (K)
    # the C5 hybrid's steps at one micro-batch of 32 requests x 256 tokens (M = 8192 rows): (kind, rows, T, D)
    "rms_quant": ("c5", 32, 256, 2560),
    "gdn_prep": ("c5", 32, 256, 2560),
    "gdn_chunk": ("c5", 32, 256, 2560),
    "gdn_gate": ("c5", 32, 256, 2560),
    # the same steps at one full C5 micro-batch (128 requests x 256 tokens, M = 32768 rows: inputs larger than L2),
    # and the quantiser of the MLP's down-projection input (D = 9728)
    "rms_quant_mb": ("c5", 128, 256, 2560),
    "gdn_prep_mb": ("c5", 128, 256, 2560),
    "gdn_gate_mb": ("c5", 128, 256, 2560),
    "act_quant_mb": ("c5", 128, 256, 9728),
}


def run_case(name):
    import torch

    import basal_b200 as b2
    fmt, M, N, K = CASES[name]
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    if fmt == "c5":
        run_c5_case(b2, name, M, N, K, dev, g)
        return
    x = torch.randn(M, K, device=dev, generator=g).bfloat16()
    if fmt == "readout":
        head = torch.nn.Linear(K, 151936, bias=False, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            head.weight.normal_(0.0, 0.02, generator=g)
        ro = b2.readout.CodeReadout(head)
        rows, idx, pad = ro.rows([torch.randperm(151936, device=dev, generator=g)[:N].tolist()] * M)
        for _ in range(5):
            ro.device_probs(x, rows, idx, pad)
    elif N == 0 and fmt == "nvfp4":
        inv_g = torch.tensor([0.5], device=dev)
        for _ in range(5):
            b2.nvfp4.act_quant(x, inv_g)
    elif N == 0:
        for _ in range(5):
            b2.fp8block.act_quant(x)
    elif fmt == "nvfp4":
        lin = torch.nn.Linear(K, N, bias=False, device=dev)
        f = b2.nvfp4.NVFP4Linear.of(lin, float(x.abs().max()))
        q, s = b2.nvfp4.act_quant(x, f.inv_g)
        for _ in range(5):
            torch.ops.basal.nvfp4_gemm(q, s, f.weight, f.weight_scale.view(torch.uint8), f.alpha, M, torch.bfloat16)
    else:
        mod = b2.fp8block if fmt == "fp8" else b2.int8block
        q, s = mod.quantize(torch.randn(N, K, device=dev, generator=g) * 0.02)
        qa, sa = mod.act_quant(x)
        for _ in range(5):
            if name == "fp8_gemm_few":  # the unsplit kernel, one CTA on each weight tile
                unsplit_gemm(b2, fmt, qa, sa, q, s)
            else:
                mod.gemm(qa, sa, q, s, torch.bfloat16)
    torch.cuda.synchronize()
    print(json.dumps({"case": name, "M": M, "N": N, "K": K, "faults": b2._lib.device_faults(0)}))


def run_c5_case(b2, name, rows, T, D, dev, g):
    """One C5 step on its own (C5's sizes: 16 key / 32 value heads of 128, convolution 4) over rows x T tokens: 2
    untimed launches, then 3 of the kernel under study; inputs drawn as the model makes them."""
    import torch
    from basal_b200 import hybrid
    cfg = hybrid.C5
    M = rows * T
    name = name.removesuffix("_mb")
    if name == "act_quant":
        x = torch.randn(M, D, device=dev, generator=g).bfloat16()
        for _ in range(5):
            b2.ops.fp8_act_quant(x)
    elif name == "rms_quant":
        x = torch.randn(M, D, device=dev, generator=g).bfloat16()
        w = (torch.randn(D, device=dev, generator=g) * 0.02).bfloat16()
        for _ in range(5):
            b2.ops.rms_norm_fp8_quant(x, w, cfg.eps)
    else:
        ld = sum(cfg.in_sizes)
        proj = torch.randn(M, ld, device=dev, generator=g).bfloat16()
        conv = (torch.rand(cfg.conv_dim, cfg.conv, device=dev, generator=g) - 0.5).bfloat16()
        A_log = torch.log(1 + 15 * torch.rand(cfg.lin_v_heads, device=dev, generator=g))
        dt_bias = torch.ones(cfg.lin_v_heads, device=dev).bfloat16()
        tail = torch.randn(1, cfg.conv - 1, cfg.conv_dim, device=dev, generator=g).bfloat16()
        b_off = cfg.conv_dim + cfg.value_dim
        args = (proj, tail, conv, A_log, dt_bias, rows, T, cfg.lin_k_heads, cfg.lin_v_heads, b_off,
                b_off + cfg.lin_v_heads)
        q, k, v, beta, gg = b2.ops.gdn_prep(*args)
        s0 = torch.randn(1, cfg.lin_v_heads, 128, 128, device=dev, generator=g) * 0.05
        o, _ = b2.ops.gdn_chunk_rule(q, k, v, gg, beta, s0, True)
        for _ in range(5):
            if name == "gdn_prep":
                b2.ops.gdn_prep(*args)
            elif name == "gdn_chunk":
                b2.ops.gdn_chunk_rule(q, k, v, gg, beta, s0, True)
            else:
                b2.ops.gdn_gate_fp8_quant(o, proj, cfg.conv_dim, torch.ones(128, device=dev).bfloat16(), cfg.eps,
                                          rows, T)
    torch.cuda.synchronize()
    print(json.dumps({"case": name, "rows": rows, "T": T, "D": D, "faults": b2._lib.device_faults(0)}))


def unsplit_gemm(b2, fmt, qa, sa, q, s):
    """The block GEMM through the C ABI with no workspace (bf16 out): for M <= 64, one CTA on each weight tile."""
    import torch
    M, K = qa.shape
    c = torch.empty(M, q.shape[0], dtype=torch.bfloat16, device=qa.device)
    name = "basal200_int8_block_gemm" if fmt == "int8" else "basal200_fp8_block_gemm"
    b2._lib.call(name, qa.device, qa.data_ptr(), sa.data_ptr(), q.data_ptr(), s.data_ptr(), None, c.data_ptr(),
                 b2._lib.BF16, M, q.shape[0], K, None, 0)
    return c


def run_sweep(fmts):
    """The C3 / C4 linear sweeps (BASELINE configs 3 and 4): M in {16, 128, 1024, 8192} x (N, K) in {(2048, 2048),
    (12288, 2048), (2048, 6144)}, per format. One JSON line per point: the GEMM alone (codes and scales already
    quantised) and the linear (activation quantiser + GEMM), each timed as 4 launches on 4 different weights inside
    one CUDA graph that first reads a 256 MB buffer (L2 holds no operand, and stays clean), minus that read alone;
    bytes = weight codes + scales + activation codes + scales + bf16 output (the algorithmic bytes), against the
    measured HBM copy bandwidth. Synthetic inputs: X ~ N(0, 1) (NVFP4: 1% of values x 20), W ~ N(0, 0.02), seed 0."""
    import torch

    import basal_b200 as b2
    dev = torch.device("cuda", 0)
    pk = peaks()
    flush = torch.ones(64 << 20, device=dev)
    reps = 4

    graph_us = graph_timer(torch, flush)

    base = graph_us(lambda: flush.sum())
    gen = torch.Generator(device=dev).manual_seed(0)
    if "glu" in fmts:
        # C2's gate/up projection (2048 -> 2 x 6144) with the SwiGLU that follows it: the gated linear in one GEMM
        # (basal::fp8_block_linear_glu) against the merged linear and torch's silu and product
        K, I = 2048, 6144
        qg, sg = b2.fp8block.quantize(torch.randn(2 * I, K, device=dev, generator=gen) * 0.02)
        for M in (16, 1024, 8192, 77431):
            x = torch.randn(M, K, device=dev, generator=gen).bfloat16()

            def unfused():
                y = b2.fp8block.linear(x, qg, sg)
                return torch.nn.functional.silu(y[:, :I]) * y[:, I:]
            tf = graph_us(lambda: (flush.sum(), b2.fp8block.linear_glu(x, qg, sg, "silu"))) - base
            tu = graph_us(lambda: (flush.sum(), unfused())) - base
            print(json.dumps({"sweep": "gated linear (C2 gate/up + SwiGLU)", "M": M, "I": I, "K": K,
                              "fused_us": round(tf, 2), "unfused_us": round(tu, 2),
                              "fused_tflops": round(2 * M * 2 * I * K / tf / 1e6, 1)}), flush=True)
        fmts = [f for f in fmts if f != "glu"]
    if "res" in fmts:
        # C2's o projection (2048 -> 2048) added to the residual stream: the addition in the GEMM's epilogue
        # (basal::fp8_block_linear_residual) against the linear and torch's addition, and the plain linear alone
        K, N = 2048, 2048
        qr, sr = b2.fp8block.quantize(torch.randn(N, K, device=dev, generator=gen) * 0.02)
        for M in (16, 1024, 8192, 77431):
            x = torch.randn(M, K, device=dev, generator=gen).bfloat16()
            hres = torch.randn(M, N, device=dev, generator=gen).bfloat16()
            tf = graph_us(lambda: (flush.sum(), b2.fp8block.FORMAT.linear_residual(x, qr, sr, None, hres))) - base
            tu = graph_us(lambda: (flush.sum(), hres + b2.fp8block.linear(x, qr, sr))) - base
            tl = graph_us(lambda: (flush.sum(), b2.fp8block.linear(x, qr, sr))) - base
            print(json.dumps({"sweep": "residual linear (C2 o projection + residual)", "M": M, "N": N, "K": K,
                              "fused_us": round(tf, 2), "unfused_us": round(tu, 2), "linear_alone_us": round(tl, 2)}),
                  flush=True)
        fmts = [f for f in fmts if f != "res"]
    if "c5" in fmts:
        # one C5 micro-batch (128 requests of 256 suffix tokens after the shared 1024-token prefix, 8 options): its time
        # (CUDA events, after a warm-up call) and the device time of each kernel in it (torch profiler, one call)
        from basal_b200 import hybrid, readout
        model = hybrid.HybridClassifier(hybrid.C5, device=dev, seed=0)
        prefix, suffix, options = c5_inputs(hybrid.C5.vocab)
        ro = readout.CodeReadout(model.head)
        rows, idx, pad = ro.rows([options] * C5_MICRO)
        st = model.prefix(prefix.to(dev))
        ids = suffix[:C5_MICRO].to(dev)
        model.decide(ids, st, ro, rows, idx, pad)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        model.decide(ids, st, ro, rows, idx, pad)
        e1.record()
        torch.cuda.synchronize()
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            model.decide(ids, st, ro, rows, idx, pad)
            torch.cuda.synchronize()
        ev = [e for e in prof.key_averages() if e.device_time_total > 0]
        total = sum(e.device_time_total for e in ev)
        print(json.dumps({"sweep": "C5 micro-batch", "requests": C5_MICRO, "ms": round(e0.elapsed_time(e1), 2),
                          "kernels_ms": round(total / 1e3, 2)}), flush=True)
        for e in sorted(ev, key=lambda e: -e.device_time_total)[:16]:
            print(json.dumps({"kernel": e.key[:90], "calls": e.count, "ms": round(e.device_time_total / 1e3, 3),
                              "share": round(e.device_time_total / total, 4)}), flush=True)
        fmts = [f for f in fmts if f != "c5"]
    if "readout" in fmts:
        # C4's readout: h [256, 2048] bf16 ~ N(0, 1) at the answer positions, a 151,936-row bf16 head ~ N(0, 0.02),
        # one code set of k ids shared by all rows; the device part of CodeReadout.probs per call (basal::code_logits +
        # basal::code_probs)
        R, D, V = 256, 2048, 151936
        head = torch.nn.Linear(D, V, bias=False, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            head.weight.normal_(0.0, 0.02, generator=gen)
        h = torch.randn(R, D, device=dev, generator=gen).bfloat16()
        for softcap in (None, 30.0):
            ro = b2.readout.CodeReadout(head, softcap=softcap)
            for k in (2, 8, 64, 255):
                ids = torch.randperm(V, device=dev, generator=gen)[:k].tolist()
                rows, idx, pad = ro.rows([ids] * R)
                t = graph_us(lambda: (flush.sum(), ro.device_probs(h, rows, idx, pad))) - base
                byts = 2 * R * D + 2 * k * D + 4 * R * k * 2 + 8 * k
                print(json.dumps({"sweep": "C4 readout", "R": R, "D": D, "k": k, "softcap": softcap,
                                  "us": round(t, 2), "gbs": round(byts / t / 1e3, 1),
                                  "gflops": round(2 * R * k * D / t / 1e3, 1)}), flush=True)
        del head
        fmts = [f for f in fmts if f != "readout"]
    for fmt in fmts:
        for N, K in ((2048, 2048), (12288, 2048), (2048, 6144)):
            ws = [torch.randn(N, K, device=dev, generator=gen) * 0.02 for _ in range(reps)]
            if fmt == "nvfp4":
                lins = []
                for w in ws:
                    lin = torch.nn.Linear(K, N, bias=False, device=dev)
                    with torch.no_grad():
                        lin.weight.copy_(w)
                    lins.append(lin)
            else:
                mod = b2.fp8block if fmt == "fp8" else b2.int8block
                qw = [mod.quantize(w) for w in ws]
            del ws
            for M in (16, 128, 1024, 8192):
                x = torch.randn(M, K, device=dev, generator=gen)
                if fmt == "nvfp4":
                    x = torch.where(torch.rand(M, K, device=dev, generator=gen) < 0.01, x * 20, x).bfloat16()
                    fs = [b2.nvfp4.NVFP4Linear.of(lin, float(x.abs().max())) for lin in lins]
                    qa, sa = b2.nvfp4.act_quant(x, fs[0].inv_g)
                    gemm = [lambda f=f: torch.ops.basal.nvfp4_gemm(qa, sa, f.weight, f.weight_scale.view(torch.uint8),
                                                                  f.alpha, M, torch.bfloat16) for f in fs]
                    linear = [lambda f=f: f(x) for f in fs]
                    wbytes, abytes = N * K // 2 + N * K // 16, M * K // 2 + M * K // 16
                else:
                    x = x.bfloat16()
                    qa, sa = mod.act_quant(x)
                    gemm = [lambda q=q, s=s: mod.gemm(qa, sa, q, s, torch.bfloat16) for q, s in qw]
                    linear = [lambda q=q, s=s: mod.linear(x, q, s) for q, s in qw]
                    wbytes, abytes = N * K + 4 * (N // 128) * (K // 128), M * K + 4 * M * (K // 128)
                    split = b2._lib.lib().basal200_block_gemm_workspace_bytes(M, N, K) > 0
                    # the same GEMM without a workspace: the few-rows kernel that puts one CTA on each weight tile
                    whole = [lambda q=q, s=s: unsplit_gemm(b2, fmt, qa, sa, q, s) for q, s in qw] if split else None

                def body(fns):
                    flush.sum()
                    for fn in fns:
                        fn()
                tg = (graph_us(lambda: body(gemm)) - base) / reps
                tl = (graph_us(lambda: body(linear)) - base) / reps
                byts = wbytes + abytes + 2 * M * N
                line = {
                    "sweep": "C3" if fmt == "nvfp4" else ("C4" if fmt == "int8" else "C3/C4 shapes, FP8"),
                    "format": fmt, "M": M, "N": N, "K": K, "gemm_us": round(tg, 2),
                    "gemm_tflops": round(2 * M * N * K / tg / 1e6, 1), "gemm_gbs": round(byts / tg / 1e3, 1),
                    "gemm_hbm_frac": round(byts / tg / 1e3 / pk["hbm_gbs"], 3), "linear_us": round(tl, 2),
                    "kernel": ("nvfp4" if fmt == "nvfp4" else
                               ("few-rows split" if M <= 64 and split else ("few-rows" if M <= 64 else "block")))}
                if fmt != "nvfp4" and whole:
                    tw = (graph_us(lambda: body(whole)) - base) / reps
                    line["unsplit_gemm_us"] = round(tw, 2)
                    line["unsplit_hbm_frac"] = round(byts / tw / 1e3 / pk["hbm_gbs"], 3)
                print(json.dumps(line), flush=True)
    print(json.dumps({"faults": b2._lib.device_faults(0), "hbm_peak_gbs": pk["hbm_gbs"], "peak_source": pk["source"]}))


# ------------------------------------------------------------------------------------------------------------------
# decisions/s
# ------------------------------------------------------------------------------------------------------------------
C5_REQUESTS, C5_PREFIX, C5_SUFFIX, C5_OPTIONS, C5_MICRO = 4096, 1024, 256, 8, 128


def c5_inputs(vocab):
    """The seeded prefix ids, every request's suffix ids [4096, 256] (host) and the 8 option ids."""
    import torch
    g = torch.Generator().manual_seed(5)
    prefix = torch.randint(0, vocab, (C5_PREFIX,), generator=g)
    options = torch.randperm(vocab, generator=g)[:C5_OPTIONS].tolist()
    suffix = torch.randint(0, vocab, (C5_REQUESTS, C5_SUFFIX), generator=torch.Generator().manual_seed(6))
    return prefix, suffix, options


def run_decisions(rank, world, local_rank):
    """Decisions/s of C5 over `world` ranks (each its row shard of the 4096 requests); returns a dict on rank 0."""
    import torch
    import torch.distributed as dist

    from basal_b200 import hybrid, readout, shard
    dev = torch.device("cuda", local_rank)
    model = hybrid.HybridClassifier(hybrid.C5, device=dev, seed=0)  # the same weights on every rank
    prefix, suffix, options = c5_inputs(hybrid.C5.vocab)
    lo, hi = shard.shard_range(C5_REQUESTS, world, rank)
    mine = suffix[lo:hi].pin_memory()
    out = torch.empty(hi - lo, C5_OPTIONS, dtype=torch.float32).pin_memory()
    ro = readout.CodeReadout(model.head)
    rows, idx, pad = ro.rows([options] * C5_MICRO)
    ids = torch.empty(C5_MICRO, C5_SUFFIX, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)

    def job(n_requests):
        st = model.prefix(prefix.to(dev, non_blocking=True))
        for a in range(0, n_requests, C5_MICRO):
            b = min(a + C5_MICRO, n_requests)
            ids[: b - a].copy_(mine[a:b], non_blocking=True)
            r, i, p = (rows, idx, pad) if b - a == C5_MICRO else ro.rows([options] * (b - a))
            out[a:b].copy_(model.decide(ids[: b - a], st, ro, r, i, p), non_blocking=True)

    job(min(C5_MICRO, hi - lo))  # warm-up: the prefix and one micro-batch
    torch.cuda.synchronize(dev)
    shard.check_peers(tag="decisions")
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    job(hi - lo)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = shard.max_over_ranks(e0.elapsed_time(e1))
    if world > 1:
        dist.barrier()
    tokens = world * C5_PREFIX + C5_REQUESTS * C5_SUFFIX
    ok = bool(torch.isfinite(out).all()) and float((out.sum(-1) - 1).abs().max()) < 1e-4
    if rank != 0:
        return None
    return {"value": round(C5_REQUESTS / (ms * 1e-3), 1), "unit": "decisions/s", "n_gpus": world,
            "ms": round(ms, 1), "requests": C5_REQUESTS, "prefix_tokens": C5_PREFIX, "suffix_tokens": C5_SUFFIX,
            "options": C5_OPTIONS, "micro_batch": C5_MICRO, "scaling": "strong (4096 requests in all)",
            "linear_tflops": round(model.flops_per_token() * tokens / (ms * 1e-3) / 1e12, 1),
            "probabilities_ok": ok,
            "h2d_bytes": int(C5_REQUESTS * C5_SUFFIX * 8 + world * C5_PREFIX * 8),
            "d2h_bytes": int(C5_REQUESTS * C5_OPTIONS * 4),
            "model": "random-init 32-layer hybrid, 24 Gated DeltaNet + 8 attention layers, hidden 2560, SwiGLU 9728, "
                     "vocab 151936, every linear FP8-block (GPT-2 scaled init)",
            "timed": "the prefix on every GPU, then the rank's requests in micro-batches of 128 (suffix ids copied in "
                     "from pinned host memory, probabilities copied out), CUDA events, max over ranks"}


def c5_cpu_baseline():
    """The oracle (numpy, all host threads) on one request of the C5 layer sizes, on one 3 : 1 period of layers
    (4 of 32), a 64-token prefix and 32 suffix tokens; per-token time x 8 periods x 256 tokens = seconds a decision."""
    import numpy as np
    from oracle import hybrid as ohy

    class Cfg:  # C5's sizes (basal_b200.hybrid.C5), 4 layers
        layers, hidden, heads, kv_heads, head_dim, inter, vocab = 4, 2560, 16, 4, 128, 9728, 151936
        lin_k_heads, lin_v_heads, lin_k_dim, lin_v_dim, conv, eps, rotary_dims, rope_theta = 16, 32, 128, 128, 4, \
            1e-6, 32, 10000.0
        key_dim, value_dim = 2048, 4096
        conv_dim = 8192
        in_sizes = (8192, 4096, 32, 32, 64)
        qkv_sizes = (4096, 512, 512)
        kinds = ["linear_attention"] * 3 + ["full_attention"]
    cfg = Cfg()
    rng = np.random.default_rng(0)
    n = lambda *sh, std=0.02: (rng.standard_normal(sh, dtype=np.float32) * np.float32(std))  # noqa: E731

    def q(a):  # random finite e4m3 codes (sign | 0x00..0x7e) and 128 x 128 block scales of a weight's shape
        codes = rng.integers(0, 0x7F, a.shape, dtype=np.uint8) | (rng.integers(0, 2, a.shape, dtype=np.uint8) << 7)
        return codes, np.full((a.shape[0] // 128, a.shape[1] // 128), 0.02 / 448 * 3, np.float32)
    D = cfg.hidden
    W = {"embed": n(512, D, std=1.0), "head": n(8, D), "final_norm": n(D), "layers": []}
    for kind in cfg.kinds:
        L = dict(kind=kind, nw=n(D), mlp_nw=n(D), gate_up=q(n(2 * cfg.inter, D)), down=q(n(D, cfg.inter)))
        if kind == "linear_attention":
            L.update(w_in=q(n(sum(cfg.in_sizes), D)), conv=n(cfg.conv_dim, 4, std=0.3), A_log=np.zeros(32, np.float32),
                     dt_bias=np.ones(32, np.float32), gnorm=np.ones(128, np.float32), out=q(n(D, cfg.value_dim)))
        else:
            L.update(w_qkv=q(n(sum(cfg.qkv_sizes), D)), q_norm=n(128), k_norm=n(128), o=q(n(D, 2048)))
        W["layers"].append(L)
    _, st = ohy.prefix(W, cfg, rng.integers(0, 512, 64))
    sfx = rng.integers(0, 512, 32)
    t0 = time.perf_counter()
    ohy.decide(W, cfg, st, sfx, np.arange(8))
    dt = time.perf_counter() - t0
    sec = dt / 32 * (32 / 4) * C5_SUFFIX
    return {"value": round(1.0 / sec, 4), "unit": "decisions/s", "cores": blas_threads(), "kind": "port",
            "sample": f"1 request: 32 suffix tokens through 4 of the 32 layers in {dt:.1f} s (after a 64-token prefix), "
                      "scaled to 32 layers and 256 tokens; the FP8 weights dequantised on every call, as the "
                      "reference's CPU linear does (basal/blockquant.py:54-60)"}


# ------------------------------------------------------------------------------------------------------------------
# the reference's own GPU paths on this box (its package installed unmodified under baseline/_ref)
# ------------------------------------------------------------------------------------------------------------------
def graph_timer(torch, flush):
    """us of fn() captured in a CUDA graph after a read of `flush` (L2 holds no operand), minus the read alone; median
    of n replays."""
    def graph_us(fn, n=15):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(n):
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        del g
        return statistics.median(ts)
    return graph_us


def run_ref_sweep(fmts):
    """The reference's GPU paths (basal 2.8.1 from baseline/_ref, through its own public functions) on the inputs
    run_sweep draws (the same seeds and draw order, so the same operands): FP8 / INT8 the Triton block GEMM
    (blockquant.py:63-106, what runs on B200: fp8block.sm90() is false off Hopper) and the linear (its
    torch.compile'd act_quant + that GEMM); NVFP4 cuBLAS through F.scaled_mm (nvfp4._mm) and the linear (its Triton
    quantiser + cuBLAS); "c2": C2's projection set. Run in a process of its own: the reference registers the same
    basal:: op names as basal_b200. One JSON line per point, "impl": "reference"."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "basal")):
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref holds no reference install"}))
        return
    sys.path.insert(0, ref)
    import torch

    from basal import fp8block, int8block, nvfp4
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pk = peaks()
    flush = torch.ones(64 << 20, device=dev)
    graph_us = graph_timer(torch, flush)
    base = graph_us(lambda: flush.sum())
    reps = 4
    gen = torch.Generator(device=dev).manual_seed(0)
    if "c2" in fmts:
        run_ref_c2(fp8block, graph_us, base, flush, dev)
    for fmt in [f for f in fmts if f in ("fp8", "int8", "nvfp4")]:
        mod = {"fp8": fp8block, "int8": int8block}.get(fmt)
        for N, K in ((2048, 2048), (12288, 2048), (2048, 6144)):
            ws = [torch.randn(N, K, device=dev, generator=gen) * 0.02 for _ in range(reps)]
            if fmt == "nvfp4":
                lins = []
                for w in ws:
                    lin = torch.nn.Linear(K, N, bias=False, device=dev)
                    with torch.no_grad():
                        lin.weight.copy_(w)
                    lins.append(lin)
            else:
                qw = [mod.quantize(w) for w in ws]
            del ws
            for M in (16, 128, 1024, 8192):
                x = torch.randn(M, K, device=dev, generator=gen)
                if fmt == "nvfp4":
                    x = torch.where(torch.rand(M, K, device=dev, generator=gen) < 0.01, x * 20, x).bfloat16()
                    fs = [nvfp4.NVFP4Linear.of(lin, float(x.abs().max())) for lin in lins]
                    qa, sa = nvfp4.act_quant(x, fs[0].inv_g)
                    gemm = [lambda f=f: nvfp4._mm(qa, sa, f.weight, f.weight_scale, f.alpha, M, torch.bfloat16)
                            for f in fs]
                    linear = [lambda f=f: f(x) for f in fs]
                else:
                    x = x.bfloat16()
                    qa, sa = mod.act_quant(x)
                    gemm = [lambda q=q, s=s: mod.gemm(qa, sa, q, s, torch.bfloat16) for q, s in qw]
                    linear = [lambda q=q, s=s: mod.linear(x, q, s) for q, s in qw]

                def body(fns):
                    flush.sum()
                    for fn in fns:
                        fn()
                tg = (graph_us(lambda: body(gemm)) - base) / reps
                tl = (graph_us(lambda: body(linear)) - base) / reps
                print(json.dumps({"impl": "reference", "format": fmt, "M": M, "N": N, "K": K, "gemm_us": round(tg, 2),
                                  "gemm_tflops": round(2 * M * N * K / tg / 1e6, 1), "linear_us": round(tl, 2),
                                  "kernel": "cuBLAS block-scaled FP4 (F.scaled_mm)" if fmt == "nvfp4" else
                                  "Triton block GEMM"}), flush=True)
    print(json.dumps({"impl": "reference", "peak_source": pk["source"], "torch": torch.__version__}))


def run_ref_c2(fp8block, graph_us, base, flush, dev):
    """C2's projection set through the reference's FP8 linear (its act_quant + Triton block GEMM), one step captured
    in a CUDA graph after an L2-clean read: TFLOP/s beside this build's bench value."""
    import torch
    g = torch.Generator().manual_seed(0)
    M = int(torch.randint(128, 2049, (64,), generator=g).sum())  # C2's packed rows (shard.varlen_lengths, seed 0)
    gen = torch.Generator(device=dev).manual_seed(1000)
    xs = {HIDDEN: torch.randn(M, HIDDEN, device=dev, generator=gen).bfloat16(),
          INTER: torch.randn(M, INTER, device=dev, generator=gen).bfloat16()}
    ws = {name: fp8block.quantize(torch.randn(n, k, device=dev, generator=gen) * 0.02) for name, n, k in PROJ}

    def step():
        flush.sum()
        for name, n, k in PROJ:
            fp8block.linear(xs[k], *ws[name])
    t = graph_us(step, n=5) - base
    gemm_t = {}
    for name, n, k in PROJ:
        qa, sa = fp8block.act_quant(xs[k])
        gemm_t[name] = graph_us(lambda: (flush.sum(), fp8block.gemm(qa, sa, *ws[name], torch.bfloat16)), n=5) - base
    print(json.dumps({"impl": "reference", "workload": "C2", "rows": M, "step_us": round(t, 1),
                      "tflops": round(M * flops_per_row() / t / 1e6, 1),
                      "gemm_tflops": {name: round(2 * M * n * k / gemm_t[name] / 1e6, 1) for name, n, k in PROJ},
                      "path": "fp8block.linear: torch.compile'd act_quant + the Triton block GEMM"}), flush=True)


# C5's projections (hidden 2560; 16 query and 4 key/value heads of 128; SwiGLU 9728), as (name, N, K)
C5_PROJ = (("qkv", 3072, 2560), ("o", 2560, 2048), ("gate_up", 19456, 2560), ("down", 2560, 9728))


def run_sweep_tp(rank, world, local_rank, steps=20):
    """The column-parallel FP8 linears of C5's projections split over the `world` GPUs of a torchrun (every rank the
    same rows): the GEMM whose epilogue stores each rank's columns into every rank's output (fused all-gather)
    against the shard's GEMM + NCCL all-gather + interleave copy. One JSON line per (projection, rows) on rank 0:
    us per forward (CUDA events over `steps` forwards, max over ranks), TFLOP/s of the whole linear, and the bound
    = max(shard FLOPs / FP8 peak, bytes a rank sends over NVLink / 770 GB/s measured per direction)."""
    import torch

    import basal_b200 as b2
    from basal_b200 import shard
    dev = torch.device("cuda", local_rank)
    pk = peaks()
    fp8_peak = 2.0 * pk["bf16_tflops"] * 1e12
    g = torch.Generator(device=dev).manual_seed(7)
    for name, N, K in C5_PROJ:
        lin = torch.nn.Linear(K, N, bias=False, device=dev)
        with torch.no_grad():
            lin.weight.normal_(0.0, 0.02, generator=g)
        full = b2.fp8block.BlockFP8Linear.of(lin)
        del lin
        m = shard.ColumnShardedFP8Linear(full, timeout_ms=30000)
        n_local = m.shard.out_features
        for M in (256, 4096):
            x = torch.randn(M, K, device=dev, generator=g).bfloat16()
            times, how = {}, {}
            for mode, fn in (("fused", m.forward), ("nccl", m.forward_nccl)):
                for _ in range(3):
                    fn(x)
                torch.cuda.synchronize()
                # `steps` forwards captured in one CUDA graph (the device time, not Python's); eager if capture fails
                graph = None
                try:
                    side = torch.cuda.Stream()
                    side.wait_stream(torch.cuda.current_stream())
                    with torch.cuda.stream(side):
                        graph = torch.cuda.CUDAGraph()
                        with torch.cuda.graph(graph, stream=side):
                            for _ in range(steps):
                                fn(x)
                    torch.cuda.current_stream().wait_stream(side)
                    torch.cuda.synchronize()
                except Exception:  # noqa: BLE001 - a library that cannot be captured: time it eagerly
                    graph = None
                    torch.cuda.synchronize()
                ok = shard.max_over_ranks(0.0 if graph is not None else 1.0) == 0.0  # every rank captured
                shard.check_peers(tag=f"tp-{name}-{M}-{mode}")
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                if ok:
                    graph.replay()
                else:
                    for _ in range(steps):
                        fn(x)
                e1.record()
                torch.cuda.synchronize()
                del graph
                times[mode] = shard.max_over_ranks(e0.elapsed_time(e1) / steps * 1e3)
                how[mode] = "graph" if ok else "eager"
            flops = 2 * M * N * K
            bound_us = max(2 * M * n_local * K / fp8_peak, M * n_local * 2 * (world - 1) / 770e9) * 1e6
            if rank == 0:
                print(json.dumps({"sweep": "C5 column-parallel FP8 linear", "proj": name, "M": M, "N": N, "K": K,
                                  "gpus": world, "fused_us": round(times["fused"], 2),
                                  "nccl_us": round(times["nccl"], 2),
                                  "fused_tflops": round(flops / times["fused"] / 1e6, 1),
                                  "nccl_tflops": round(flops / times["nccl"] / 1e6, 1),
                                  "bound_us": round(bound_us, 2),
                                  "fused_of_bound": round(bound_us / times["fused"], 3),
                                  "timing": how}), flush=True)
        del m, full
    if rank == 0:
        print(json.dumps({"faults": b2._lib.device_faults(local_rank)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--case", choices=sorted(CASES), help="run one small profiling case instead of the benchmark")
    ap.add_argument("--no-decisions", action="store_true", help="skip the C5 decisions/s measurement")
    ap.add_argument("--decisions-only", action="store_true", help="only the C5 decisions/s measurement (one line)")
    ap.add_argument("--sweep", metavar="FMTS", help="run the C3/C4 sweeps for these parts (fp8,int8,nvfp4,readout, "
                    "glu,res; c5: one C5 micro-batch and its kernels) instead of the benchmark; 'tp' (under "
                    "torchrun): C5's column-parallel linears")
    args = ap.parse_args()
    if args.sweep == "tp":  # under torchrun, 2 or more GPUs
        import datetime

        import torch
        import torch.distributed as dist
        rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
        local_rank = int(os.environ.get("LOCAL_RANK", 0))
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
        try:
            run_sweep_tp(rank, world, local_rank)
        finally:
            dist.destroy_process_group()
        return
    if args.sweep and args.sweep.startswith("ref"):  # ref,fp8,int8,nvfp4,c2: the reference's GPU paths
        run_ref_sweep(args.sweep.split(",")[1:])
        return
    if args.sweep:
        run_sweep(args.sweep.split(","))
        return
    if args.case:
        run_case(args.case)
        return
    if args.warmup < 3:
        args.warmup = 3
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.decisions_only:
            import torch
            torch.cuda.set_device(local_rank)
            d = run_decisions(rank, world, local_rank)
            if rank == 0:
                print(json.dumps({"metric": "decisions/s (BASELINE config 5)", **d}), flush=True)
            return
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
