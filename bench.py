#!/usr/bin/env python3
"""Benchmark of the B200 routed-MoE layer (Gyro trellis experts) through its C ABI.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload decode]

Workload "decode" (default): a 40-layer stack of the config-0 routed
layer (hidden 2048, 256 experts of gate/up [512x2048] and down [2048x512] TQ2_T, top-8,
router f32 ~N(0, 0.02)), independent seeded weights per layer (8.56 GB of packed experts
resident in HBM), batch-1 greedy decode: each step pushes one fresh bf16 token ~N(0,1) through
all 40 layers with x_{l+1} = x_l + MoE_l(RMSNorm(x_l)) (pre-norm residual stand-in for the
hyper-connection mixer; the plain x + MoE(x) diverges within a few dozen random layers).
A step touches 40 x 8 distinct experts = 267 MB of packed weights, more than the 126 MB L2, and
consecutive steps route differently, so no step is served from L2.

One JSON line on rank 0. value = tokens/s over the whole job (device-timed with CUDA events on
the library's stream, max over ranks); e2e = the same through gx_stack_forward_host with host
buffers; roofline = the gate/up decode GEMV (the dominant kernel), algorithmic bytes per launch
over its event-timed duration in the final timed step; cpu_baseline = the CPU oracle (restated
reference engine) on the host cores, on a bounded sample. With N > 1 GPUs each rank runs an
independent replica on its own tokens ("replicas": decode does not exchange data).

Workload "prefill": one 1,024-token bf16 sequence through the config-0
layer with Zipf(1.1) routing; roofline = the tcgen05 gate/up grouped GEMM in useful TFLOP/s.

Workload "ep-prefill": 32 packed sequences (log-uniform lengths in
[1, 512]) through the 40-layer stack with Zipf(1.1) routing. With N ranks the experts are
sharded 256/N per GPU and tokens travel by NCCL dispatch / combine inside the library; the batch
is fixed, so scaling is strong.

--impl reference times the reference's CPU engine (restated in oracle/, the reference's Zig code
cannot be built here) on the same workload with all host threads; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "gyro-dx_b200"))

import numpy as np  # noqa: E402

METRIC = "routed-MoE layer tok/s (decode & prefill) at 1/2/4/8 B200; HBM GB/s % peak"
N_LAYERS = 40
E, F, NE, U = 2048, 512, 256, 8
TYPE_ID = 144
EXPERT_BYTES = 835_584                        # gate + up + down of one TQ2_T expert
GATE_UP_BYTES = 2 * 278_528
ROUTER_BYTES = NE * E * 4
LAYER_SEED = 1000


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=128)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=["decode", "prefill", "ep-prefill"], default="decode")
    p.add_argument("--tokens", type=int, default=1024, help="prefill: tokens per step")
    p.add_argument("--layers", type=int, default=N_LAYERS)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=15.0)
    p.add_argument("--no-replicas", action="store_true", help="ep-prefill: plain expert sharding, no replicas")
    return p.parse_args()


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def traffic_bytes(key: str):
    """DRAM bytes per launch of a kernel from the committed ncu summary (profiles/traffic.json)."""
    f = ROOT / "profiles" / "traffic.json"
    return json.loads(f.read_text()).get(key) if f.exists() else None


def make_layers(n_layers: int):
    from gyro_moe import synth
    for l in range(n_layers):
        yield synth.make_layer(LAYER_SEED + l)


def step_tokens(n_steps: int, n_tok: int, rank: int) -> np.ndarray:
    from gyro_moe import synth
    x = np.random.default_rng(7 + 1000 * rank).standard_normal((n_steps, n_tok, E)).astype(np.float32)
    return synth.bf16_bits(x.reshape(-1, E)).reshape(n_steps, n_tok, E)


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.file.flush()
        rows = [l.split(",") for l in Path(self.file.name).read_text().splitlines() if l.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for name, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_baseline(layers, seconds: float) -> dict:
    """The restated reference CPU engine (oracle/, fast build, all host threads) on a bounded
    sample: whole tokens through the 40-layer stack until `seconds` have passed."""
    from oracle import oracle
    from gyro_moe import synth
    threads = oracle.max_threads()
    rng = np.random.default_rng(99)
    done, t0 = 0, time.perf_counter()
    while True:
        x = synth.bf16_round(rng.standard_normal((1, E)).astype(np.float32))
        oracle.stack(layers, x, threads=threads, fast=True)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= 64:
            break
    return {"value": done / el, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{done} tokens x {len(layers)} layers, batch 1, {el:.1f} s on {threads} threads"}


def run_reference(args):
    """Reference arm: the CPU engine restated in oracle/ (the reference's own CPU engine is Zig,
    which is absent), all host threads, rank 0 only. Each step is a bounded sample of the
    workload: decode, one token through the 40-layer stack; prefill, 64 of the 1,024 tokens
    through the layer; ep-prefill, 64 tokens of the packed batch through the 40-layer stack."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle
    from gyro_moe import synth
    threads = oracle.max_threads()
    steps = args.warmup + args.steps
    if args.workload == "decode":
        layers = list(make_layers(args.layers))
        xs = [(t.astype(np.uint32) << 16).view(np.float32) for t in step_tokens(steps, 1, 0)]
        run = lambda x: oracle.stack(layers, x, threads=threads, fast=True)
        per_step, scaling = 1, "weak"
        config = {"workload": "decode: 40-layer stack of the config-0 routed layer (BASELINE.json configs[1]), "
                              "batch 1, fresh token per step",
                  "layers": args.layers, "n_tok": 1}
        sample = f"{args.steps} steps x 1 token x {args.layers} layers"
    elif args.workload == "prefill":
        layer = synth.make_layer(LAYER_SEED, zipf=1.1)
        xb = step_tokens(1, args.tokens, 0)[0]
        xf = (xb.astype(np.uint32) << 16).view(np.float32)
        xs = [xf[(64 * i) % args.tokens:(64 * i) % args.tokens + 64] for i in range(steps)]
        run = lambda x: oracle.moe_ffn(layer, x, threads=threads, fast=True)
        per_step, scaling = 64, "weak"
        config = {"workload": f"prefill: one {args.tokens}-token sequence through the config-0 routed layer, "
                              "Zipf(1.1) routing", "tokens": args.tokens}
        sample = f"{args.steps} steps x 64 of the {args.tokens} tokens through the layer"
    else:
        layers = [synth.make_layer(LAYER_SEED + l, zipf=1.1) for l in range(args.layers)]
        lengths, offsets, xall = ep_batch()
        T = int(offsets[-1])
        xf = (xall.astype(np.uint32) << 16).view(np.float32)
        xs = [xf[(64 * i) % T:(64 * i) % T + 64] for i in range(steps)]
        run = lambda x: oracle.stack(layers, x, threads=threads, fast=True)
        per_step, scaling = 64, "strong"
        config = {"workload": f"expert-parallel prefill: {EP_SEQS} packed sequences (log-uniform lengths in "
                              f"[1, 512], {T} tokens) through the {args.layers}-layer stack of the config-0 layer, "
                              "Zipf(1.1)", "tokens": T, "layers": args.layers}
        sample = f"{args.steps} steps x up to 64 tokens of the packed batch through {args.layers} layers"
    times, done = [], 0
    for i in range(steps):
        t0 = time.perf_counter()
        run(xs[i])
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
            done += xs[i].shape[0]
    total = sum(times)
    value = done / total
    config.update({"hidden": E, "experts": NE, "top_k": U, "ffn": F, "type": "TQ2_T", "parallelism": "host threads"})
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; shapes and distributions of the BASELINE.json config)",
        "config": config,
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample + " (oracle/ restatement of src/engine.zig:520-642; the reference's "
                                            "Zig engine cannot be built here)"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    from gyro_moe import abi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n_tok = 1
    K, W = args.steps, args.warmup

    ctx = abi.Context(device=local, max_tokens=max(n_tok, 1), max_layers=args.layers)
    keep_host = (rank == 0 and world == 1 and not args.no_cpu_baseline)
    host_layers = []
    for l, layer in enumerate(make_layers(args.layers)):
        ctx.upload_layer(l, layer)
        if keep_host:
            host_layers.append(layer)
    xs_host = step_tokens(W + K, n_tok, rank)
    xs = torch.from_numpy(xs_host.view(np.int16)).to(dev).view(torch.bfloat16)
    y = torch.empty((n_tok, E), dtype=torch.float32, device=dev)
    stream = torch.cuda.ExternalStream(ctx.stream(), device=dev)

    for i in range(W):
        ticket = ctx.stack_forward(0, args.layers, xs[i], y)
    ctx.wait(ticket)
    torch.cuda.synchronize(dev)

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
        for i in range(K):
            ticket = ctx.stack_forward(0, args.layers, xs[W + i], y)
        with torch.cuda.stream(stream):
            end.record(stream)
        end.synchronize()
    ctx.wait(ticket)  # raises if a kernel reported an error during the timed steps
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    ms = start.elapsed_time(end)
    # Kernel durations: the same steps replayed once more with phase events between the kernels
    # (events separate the kernels, so the headline loop above runs without them).
    ctx.set_flags(abi.GX_FLAG_PROFILE)
    prof = []
    for i in range(min(K, 8) + 1):
        ctx.wait(ctx.stack_forward(0, args.layers, xs[W + i % K], y))
        if i:
            prof.append(ctx.timings())
    ctx.set_flags(0)
    t = abi.Timings()
    for p in prof:
        for f in ("router_ns", "gate_up_ns", "down_ns", "experts_ns", "total_ns", "layers"):
            setattr(t, f, getattr(t, f) + getattr(p, f))
    timing_source = (f"CUDA events on the library stream between the kernels of {len(prof)} replayed steps "
                     f"({t.layers} layer launches) right after the timed region")
    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())

    # End to end: host bf16 token in (pinned staging inside the library), host f32 out.
    e2e_steps = min(K, 64)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        ctx.stack_forward_host(0, args.layers, xs_host[W + i], out_dtype=np.float32)
    e2e_s = time.perf_counter() - t0
    e2e_t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_s = float(e2e_t.item())

    pk = peaks()
    layers = max(t.layers, 1)
    layer_bytes = EXPERT_BYTES * U + ROUTER_BYTES          # algorithmic bytes per token per layer
    traffic = None
    tfile = ROOT / "profiles" / "traffic.json"
    if t.gate_up_ns == 0 and t.total_ns > 0:
        # one persistent kernel per step (the whole stack): its bytes over its event-timed duration
        launch_s = t.total_ns / len(prof) * 1e-9
        roofline = {
            "kernel": "decode_stack_kernel (persistent: router, selection, fused Gyro decode gate/up + SwiGLU, "
                      "down + combine, for all layers)",
            "bound": "hbm", "achieved": layer_bytes * args.layers * n_tok / launch_s / 1e9, "peak": pk["hbm_gbs"],
            "unit": "GB/s", "traffic": None,
            "algorithmic_bytes_per_launch": layer_bytes * args.layers * n_tok,
            "bytes_per_layer": "8 selected experts x 835,584 B + router 2,097,152 B per token",
            "launch_us": launch_s * 1e6, "per_layer_us": launch_s * 1e6 / args.layers,
            "peak_source": f"{pk['source']} (MEASURED_PEAKS.json hbm_gbs, burst copy)",
            "timing": f"CUDA events around the stack kernel on the library stream, {len(prof)} replayed steps "
                      "right after the timed region",
        }
        if tfile.exists():
            roofline["traffic"] = json.loads(tfile.read_text()).get("decode_stack_kernel_per_launch")
    else:
        gate_up_s = t.gate_up_ns / layers * 1e-9
        down_s = t.down_ns / layers * 1e-9
        router_s = t.router_ns / layers * 1e-9
        achieved = GATE_UP_BYTES * 8 / gate_up_s / 1e9 if gate_up_s > 0 else None
        experts_gbs = EXPERT_BYTES * 8 / (gate_up_s + down_s) / 1e9 if gate_up_s > 0 else None
        roofline = {
            "kernel": "gate_up_kernel (fused Gyro decode + gate/up GEMV + SwiGLU)",
            "bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "traffic": None,
            "algorithmic_bytes_per_launch": GATE_UP_BYTES * 8,
            "launch_us": gate_up_s * 1e6, "peak_source": f"{pk['source']} (MEASURED_PEAKS.json hbm_gbs, burst copy)",
            "timing": timing_source,
            "experts_phase_gbs": experts_gbs,
            "experts_phase_frac": experts_gbs / pk["hbm_gbs"] if experts_gbs else None,
            "per_layer_us": {"router": router_s * 1e6, "gate_up": gate_up_s * 1e6, "down": down_s * 1e6},
            "layer_bytes": layer_bytes,
            "layer_gbs": layer_bytes / (router_s + gate_up_s + down_s) / 1e9 if gate_up_s else None,
        }
        if tfile.exists():
            roofline["traffic"] = json.loads(tfile.read_text()).get("gate_up_kernel_decode_per_launch")
    roofline["frac"] = roofline["achieved"] / pk["hbm_gbs"] if roofline["achieved"] else None
    value = K * n_tok * world / (ms_max / 1e3)
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded; shapes and distributions of BASELINE.json config 1)",
        "config": {"workload": "decode: 40-layer stack of the config-0 routed layer (BASELINE.json configs[1]), "
                               "batch 1, fresh token per step",
                   "layers": args.layers, "n_tok": n_tok, "hidden": E, "experts": NE, "top_k": U, "ffn": F,
                   "type": "TQ2_T", "expert_bytes_resident": args.layers * NE * EXPERT_BYTES,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2: each step reads 40 x 8 distinct experts (267 MB)"},
        "roofline": roofline,
        "e2e": {"value": e2e_steps * n_tok * world / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": n_tok * E * 2,
                "d2h_bytes_per_step": n_tok * E * 4, "steps": e2e_steps,
                "api": "gx_stack_forward_host (host bf16 in, host f32 out)"},
        "gpu_launches": K if t.gate_up_ns == 0 and t.total_ns > 0 else K * args.layers * 3,
        "clocks": clocks.summary(),
    }
    if keep_host:
        line["cpu_baseline"] = cpu_baseline(host_layers, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_prefill(args):
    """one sequence of --tokens bf16 tokens ~N(0,1) through the config-0
    layer with Zipf(1.1) expert popularity (ragged segments, some experts empty), bf16 output.
    Each step is one forward of the whole sequence; 4 distinct input batches rotate."""
    import torch
    from gyro_moe import abi, synth
    from oracle import oracle

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    T, K, W = args.tokens, args.steps, args.warmup
    layer = synth.make_layer(LAYER_SEED, zipf=1.1)
    ctx = abi.Context(device=0, max_tokens=T, max_layers=1)
    ctx.upload_layer(0, layer)
    xs_host = step_tokens(4, T, 0)
    xs = torch.from_numpy(xs_host.view(np.int16)).to(dev).view(torch.bfloat16)
    y = torch.empty((T, E), dtype=torch.bfloat16, device=dev)
    ids = torch.empty((T, U), dtype=torch.int32, device=dev)
    for i in range(W):
        ctx.forward(0, xs[i % 4], y, ids)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.ExternalStream(ctx.stream(), device=dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
        for i in range(K):
            ticket = ctx.forward(0, xs[i % 4], y)
        with torch.cuda.stream(stream):
            end.record(stream)
        end.synchronize()
    ctx.wait(ticket)
    ms = start.elapsed_time(end)
    ctx.set_flags(abi.GX_FLAG_PROFILE)
    prof = []
    for i in range(5):
        ctx.wait(ctx.forward(0, xs[i % 4], y, ids))
        prof.append(ctx.timings())
    ctx.set_flags(0)
    ids_np = ids.cpu().numpy().astype(np.int64)
    counts = np.bincount(ids_np.reshape(-1), minlength=NE)
    slots = T * U
    gu_flops = slots * 2 * F * E * 2
    dn_flops = slots * F * E * 2
    gu_s = statistics.median(p.gate_up_ns for p in prof) * 1e-9
    dn_s = statistics.median(p.down_ns for p in prof) * 1e-9
    rt_s = statistics.median(p.router_ns for p in prof) * 1e-9
    pk = peaks()
    achieved = gu_flops / gu_s / 1e12
    tiles = int(np.sum((counts + 127) // 128))
    touched = int((counts > 0).sum()) * EXPERT_BYTES
    # end to end: host bf16 in, host bf16 out
    e2e_steps = min(K, 16)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        ctx.forward_host(0, xs_host[i % 4], out_dtype=np.uint16)
    e2e_s = time.perf_counter() - t0
    line = {
        "metric": METRIC, "value": K * T / (ms / 1e3), "unit": "tok/s", "n_gpus": 1, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded; shapes and distributions of BASELINE.json config 2)",
        "config": {"workload": f"prefill: one {T}-token sequence through the config-0 routed layer, Zipf(1.1) routing",
                   "tokens": T, "hidden": E, "experts": NE, "top_k": U, "ffn": F, "type": "TQ2_T",
                   "experts_hit": int((counts > 0).sum()), "max_segment": int(counts.max()), "row_tiles": tiles,
                   "l2": "inputs larger than L2: a step reads every touched expert (up to 214 MB)"},
        "roofline": {
            "kernel": "moe_gemm_kernel<gate/up> (tcgen05 grouped GEMM, in-smem trellis decode, SwiGLU epilogue)",
            "bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
            "frac": achieved / pk["bf16_tflops"], "traffic": traffic_bytes("moe_gemm_gateup_prefill_per_launch"),
            "traffic_unit": "DRAM bytes per launch (ncu capture of this workload)",
            "algorithmic_flops_per_launch": gu_flops, "launch_us": gu_s * 1e6,
            "padded_flops_per_launch": tiles * 128 * 2 * F * E * 2,
            "peak_source": f"{pk['source']} (MEASURED_PEAKS.json bf16_tflops, burst; f16 has the same dense rate)",
            "phase_us": {"select_group_pack": rt_s * 1e6, "gate_up_gemm": gu_s * 1e6, "down_gemm_combine": dn_s * 1e6},
            "down_tflops": dn_flops / dn_s / 1e12,
            "hbm_gbs_experts": touched / (ms / K / 1e3) / 1e9,
        },
        "e2e": {"value": e2e_steps * T / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": T * E * 2,
                "d2h_bytes_per_step": T * E * 2, "steps": e2e_steps,
                "api": "gx_moe_forward_host (host bf16 in, host bf16 out)"},
        "gpu_launches": K * 8,
        "clocks": clocks.summary(),
    }
    if not args.no_cpu_baseline:
        threads = oracle.max_threads()
        xs32 = (xs_host[0].astype(np.uint32) << 16).view(np.float32)
        done, el = 0, 0.0
        t0 = time.perf_counter()
        while el < args.cpu_seconds and done < T:       # 64-token chunks of the sequence, bounded time
            oracle.moe_ffn(layer, xs32[done:done + 64], threads=threads, fast=True)
            done += 64
            el = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": done / el, "unit": "tok/s", "cores": threads, "kind": "port",
                                "sample": f"{done} of the {T} tokens through the layer in 64-token chunks, "
                                          f"{el:.1f} s on {threads} threads"}
    print(json.dumps(line), flush=True)
    ctx.close()


EP_SEQS, EP_SEED = 32, 4


def ep_batch():
    """32 sequences with log-uniform lengths in [1, 512] packed into one
    ragged buffer (offsets), bf16 tokens ~N(0, 1)."""
    from gyro_moe import synth
    lengths = synth.loguniform_lengths(EP_SEED, EP_SEQS)
    offsets = np.concatenate([[0], np.cumsum(lengths)])
    x = synth.bf16_bits(np.random.default_rng(EP_SEED + 1).standard_normal((int(offsets[-1]), E)).astype(np.float32))
    return lengths, offsets, x


def rank_sequences(lengths, world: int) -> list:
    """Sequences of every rank: longest first, each to the rank with the fewest tokens so far
    (ties to the lower rank), so the busiest rank holds close to 1/world of the batch; a rank
    keeps its sequences in batch order."""
    load = [0] * world
    seqs = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i)):
        r = min(range(world), key=lambda r: (load[r], r))
        load[r] += int(lengths[i])
        seqs[r].append(i)
    return [sorted(q) for q in seqs]


def rank_tokens(offsets, x, rank: int, world: int) -> np.ndarray:
    """A rank's slice of the ragged batch (its sequences from rank_sequences, concatenated)."""
    lengths = np.diff(offsets)
    parts = [x[offsets[i]:offsets[i + 1]] for i in rank_sequences(lengths, world)[rank]]
    return np.concatenate(parts) if parts else np.zeros((0, E), np.uint16)


def run_ep(args):
    """the packed batch through the 40-layer stack (Zipf(1.1) routing per
    layer). With N ranks each rank holds 256/N experts of every layer (plus replicas of the hot
    ones) and routes its own sequences (rank_sequences balances their tokens); dispatch and
    combine run inside the library, over NVLink peer memory or NCCL. The total batch is
    fixed, so scaling is strong: value = all tokens / max-over-ranks time per step."""
    import datetime
    import torch
    from gyro_moe import abi, synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    nccl_id = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        idt = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            idt.copy_(torch.frombuffer(bytearray(abi.unique_id()), dtype=torch.uint8))
        dist.broadcast(idt, 0)
        nccl_id = bytes(idt.cpu().numpy())
    lengths, offsets, xall = ep_batch()
    T = int(offsets[-1])
    mine = rank_tokens(offsets, xall, rank, world)
    n_tok = mine.shape[0]
    max_tok = max(rank_tokens(offsets, xall, r, world).shape[0] for r in range(world))
    K, W = args.steps, args.warmup
    ctx = abi.Context(device=local, max_tokens=max(max_tok, 1), max_layers=args.layers, rank=rank, world=world,
                      nccl_id=nccl_id)
    keep_host = rank == 0 and world == 1 and not args.no_cpu_baseline
    host_layers = []
    for l in range(args.layers):
        layer = synth.make_layer(LAYER_SEED + l, zipf=1.1)
        ctx.upload_layer(l, layer)
        if keep_host:
            host_layers.append(layer)
    # two input batches alternate: the same tokens scaled by 1 and by -1 route differently
    x0 = torch.from_numpy(mine.view(np.int16)).to(dev).view(torch.bfloat16)
    xs = [x0, -x0]
    y = torch.empty((n_tok, E), dtype=torch.bfloat16, device=dev)
    for i in range(W):
        ticket = ctx.stack_forward(0, args.layers, xs[i % 2], y)
    ctx.wait(ticket)
    replicas, rep0 = [], []
    if dist and not args.no_replicas:
        # expert-parallel load balance: the warm-up's routed-slot counts, summed over ranks,
        # choose per layer the popular experts every rank serves for its own tokens
        from gyro_moe import balance
        for l in range(args.layers):
            cnt = torch.from_numpy(ctx.expert_counts(l, reset=True).astype(np.int64)).to(dev)
            dist.all_reduce(cnt)
            rep = balance.choose_replicas(cnt.cpu().numpy(), world)
            ctx.replicate_experts(l, rep)
            replicas.append(len(rep))
            if l == 0:
                rep0 = list(rep)
        for i in range(W):
            ticket = ctx.stack_forward(0, args.layers, xs[i % 2], y)
        ctx.wait(ticket)
    torch.cuda.synchronize(dev)
    exchange = ctx.caps().ep_exchange
    stream = torch.cuda.ExternalStream(ctx.stream(), device=dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
        for i in range(K):
            ticket = ctx.stack_forward(0, args.layers, xs[i % 2], y)
        with torch.cuda.stream(stream):
            end.record(stream)
        end.synchronize()
    ctx.wait(ticket)
    ms_t = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    # phase times of one profiled layer-0 call and this rank's received slots, for the roofline
    ids = torch.empty((n_tok, U), dtype=torch.int32, device=dev)
    ctx.set_flags(abi.GX_FLAG_PROFILE)
    ctx.wait(ctx.forward(0, xs[0], y, ids))
    ph = ctx.timings()
    ctx.set_flags(0)
    per = NE // world
    # slots each rank serves: a shard expert's slots on its owner, a replicated expert's slots on
    # the token's own rank (layer 0's replica list)
    flat = ids.cpu().numpy().reshape(-1).astype(np.int64)
    replicated = np.isin(flat, np.array(rep0, np.int64))
    own = np.bincount(flat[~replicated] // per, minlength=world).astype(np.float64)
    sent = torch.from_numpy(own).to(dev)
    if dist:
        dist.all_reduce(sent)                     # shard slots every rank serves, summed over sources
    slots_here = float(sent[rank].item()) + float(replicated.sum())
    gu_flops = slots_here * 2 * F * E * 2
    agg = torch.tensor([gu_flops, ph.gate_up_ns * 1e-9, ph.router_ns * 1e-9, ph.down_ns * 1e-9, ph.total_ns * 1e-9],
                       dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(agg)
    flops_sum, gu_sum, rt_sum, dn_sum, tot_sum = (float(v) for v in agg.cpu())
    pk = peaks()
    achieved = flops_sum / gu_sum / 1e12 if gu_sum > 0 else None
    # end to end: host bf16 in, host bf16 out
    e2e_steps = min(K, 8)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        src = mine if i % 2 == 0 else (mine ^ np.uint16(0x8000))
        ctx.stack_forward_host(0, args.layers, src, out_dtype=np.uint16)
    e2e_t = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_s = float(e2e_t.item())
    # router, top-k, rotation (push with peer memory), three grouping kernels, two packs, two
    # GEMMs, combine (return with peer memory); expert parallel adds the two plan kernels and the
    # sum of partial rows, and with peer memory the two bounded waits
    launches_per_layer = 11 if world == 1 else 16 if exchange == abi.GX_EP_PEER else 14
    line = {
        "metric": METRIC, "value": K * T / (ms / 1e3), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded; shapes and distributions of BASELINE.json config 4)",
        "config": {"workload": f"expert-parallel prefill: {EP_SEQS} packed sequences (log-uniform lengths in [1, 512], "
                               f"{T} tokens) through the {args.layers}-layer stack of the config-0 layer, Zipf(1.1)",
                   "tokens": T, "sequences": EP_SEQS, "layers": args.layers, "hidden": E, "experts": NE,
                   "experts_per_gpu": per, "top_k": U, "ffn": F, "type": "TQ2_T",
                   "parallelism": (f"expert parallel x{world} (dispatch/combine over "
                                   f"{'NVLink peer memory' if exchange == abi.GX_EP_PEER else 'NCCL'})")
                                  if world > 1 else "single GPU",
                   "replicated_experts_per_layer": (sum(replicas) / len(replicas)) if replicas else 0,
                   "tokens_per_rank_max": max_tok,
                   "l2": "inputs larger than L2: a step reads every touched expert of 40 layers"},
        "roofline": {
            "kernel": "moe_gemm_kernel<gate/up> on each rank's received slots (tcgen05 grouped GEMM)",
            "bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
            "frac": achieved / pk["bf16_tflops"] if achieved else None, "traffic": None,
            "how": "sum over ranks of (received slots x 2 x F x E x 2) / sum over ranks of the gate/up GEMM "
                   "event time, one profiled layer-0 call",
            "phase_ms_mean_per_rank": {"select_dispatch": rt_sum / world * 1e3, "gate_up": gu_sum / world * 1e3,
                                       "down_combine": dn_sum / world * 1e3, "layer": tot_sum / world * 1e3},
            "peak_source": f"{pk['source']} (MEASURED_PEAKS.json bf16_tflops, burst)",
        },
        "e2e": {"value": e2e_steps * T / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": n_tok * E * 2,
                "d2h_bytes_per_step": n_tok * E * 2, "steps": e2e_steps,
                "api": "gx_stack_forward_host (host bf16 in, host bf16 out), per rank"},
        "gpu_launches": K * args.layers * launches_per_layer,
        "clocks": clocks.summary(),
    }
    if keep_host:
        from oracle import oracle
        threads = oracle.max_threads()
        xf = (mine.astype(np.uint32) << 16).view(np.float32)
        done, el, t0 = 0, 0.0, time.perf_counter()
        while el < args.cpu_seconds and done < T:
            oracle.stack(host_layers, xf[done:done + 64], threads=threads, fast=True)
            done += min(64, T - done)
            el = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": done / el, "unit": "tok/s", "cores": threads, "kind": "port",
                                "sample": f"{done} of the {T} tokens in 64-token chunks through the "
                                          f"{args.layers}-layer stack, {el:.1f} s on {threads} threads"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "ep-prefill":
        run_ep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
