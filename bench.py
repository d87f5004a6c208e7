#!/usr/bin/env python3
"""Benchmark of the B200 routed-MoE layer (Gyro trellis experts) through its C ABI.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload ep-prefill|decode|prefill|sweep]

Default workload "ep-prefill", the same at every N: 32 packed sequences
(log-uniform lengths in [1, 512], 4,067 tokens with this seed) through a 40-layer stack of the
config-0 routed layer (hidden 2048, 256 experts of gate/up [512x2048] and down [2048x512] TQ2_T,
top-8, router f32 ~N(0, 0.02)) with Zipf(1.1) expert popularity and the pre-norm residual
x_{l+1} = x_l + MoE_l(RMSNorm(x_l)) between layers. With N ranks (one process per GPU under
torchrun) the experts are sharded 256/N per GPU, each rank routes its own sequences, and rows
travel inside the library (NVLink peer memory, or NCCL); the batch is fixed, so scaling is
strong. value = all tokens / max-over-ranks device time per step. After the timed region every
rank checks a sample of its tokens against the CPU oracle ("parity").

At N = 1 the same line also carries the other benchmark configurations ("secondary"):
  decode  (config 1) the 40-layer stack at batch 1, 128 fresh tokens, per-token p50/p95;
  prefill (config 2) one 1,024-token sequence through the config-0 layer, Zipf(1.1);
  sweep   (config 3) the decode GEMV of every Gyro type at [512x2048] and [2048x512], batch 1/4/16,
          over more than 4x the L2 of distinct matrices, with a bit-exact decode check.
Each is also a standalone line with --workload decode|prefill|sweep.

roofline: the dominant kernel's algorithmic work per launch over its CUDA-event duration
(grouped GEMM: useful FLOPs vs the measured bf16 peak; decode GEMVs: packed bytes vs the measured
HBM copy bandwidth). cpu_baseline: the CPU oracle (restated reference engine) on all host threads
on a bounded sample of the same workload. --impl reference times that CPU engine alone (rank 0).
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
EP_SEQS, EP_SEED = 32, 4
DECODE_STEPS, DECODE_WARMUP = 128, 8          # config 1: 128 consecutive single-token steps
PREFILL_TOKENS = 1024
SWEEP_SHAPES = [(512, 2048), (2048, 512)]
SWEEP_BATCHES = (1, 4, 16)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=["ep-prefill", "decode", "prefill", "sweep"], default="ep-prefill")
    p.add_argument("--tokens", type=int, default=PREFILL_TOKENS, help="prefill: tokens per step")
    p.add_argument("--layers", type=int, default=N_LAYERS)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-secondary", action="store_true", help="ep-prefill at N=1: skip configs 1-3")
    p.add_argument("--cpu-seconds", type=float, default=15.0)
    p.add_argument("--parity-tokens", type=int, default=4, help="ep-prefill: tokens per rank checked")
    p.add_argument("--no-replicas", action="store_true", help="ep-prefill: plain expert sharding, no replicas")
    p.add_argument("--sweep-only", default="", help="sweep: one case, e.g. TQ2_T:512x2048 (profiling)")
    p.add_argument("--sweep-l2x", type=float, default=4.5, help="sweep: matrix bytes per launch in units of L2")
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


def make_layers(n_layers: int, zipf: float | None = None):
    from gyro_moe import synth
    for l in range(n_layers):
        yield synth.make_layer(LAYER_SEED + l, zipf=zipf)


def step_tokens(n_steps: int, n_tok: int, rank: int) -> np.ndarray:
    from gyro_moe import synth
    x = np.random.default_rng(7 + 1000 * rank).standard_normal((n_steps, n_tok, E)).astype(np.float32)
    return synth.bf16_bits(x.reshape(-1, E)).reshape(n_steps, n_tok, E)


def bf16_values(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


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


def parity_rows(n_tok: int, k: int) -> np.ndarray:
    """Evenly spaced sample of a rank's token rows (first and last included)."""
    if n_tok == 0 or k <= 0:
        return np.zeros(0, np.int64)
    return np.unique(np.linspace(0, n_tok - 1, min(k, n_tok)).round().astype(np.int64))


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


class Dist:
    """torchrun environment (one process per GPU); a world of 1 runs without a process group."""

    def __init__(self):
        import datetime
        import torch
        self.torch = torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.pg = None
        if self.world > 1:
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=self.dev)
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def reduce(self, values, op: str = "sum") -> list:
        t = self.torch.tensor([float(v) for v in values], dtype=self.torch.float64, device=self.dev)
        if self.pg:
            self.pg.all_reduce(t, op={"sum": self.pg.ReduceOp.SUM, "max": self.pg.ReduceOp.MAX,
                                      "min": self.pg.ReduceOp.MIN}[op])
        return [float(v) for v in t.cpu()]

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


def timed_steps(torch, stream, dev, K: int, step, per_step: bool = False):
    """K calls of step(i) bracketed by CUDA events on the library stream (and one event per step
    when per_step). Returns (total ms, [per-step ms], clock summary)."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(K + 1)] if per_step else []
    torch.cuda.synchronize(dev)
    with ClockSampler(dev.index) as clocks:
        start.record(stream)
        for i in range(K):
            if per_step:
                marks[i].record(stream)
            step(i)
        if per_step:
            marks[K].record(stream)
        end.record(stream)
        end.synchronize()
    steps = [marks[i].elapsed_time(marks[i + 1]) for i in range(K)] if per_step else []
    return start.elapsed_time(end), steps, clocks.summary()


# ------------------------------------------------------------------------------------------
# Config 1: 40-layer decode stack at batch 1
# ------------------------------------------------------------------------------------------
def measure_decode(torch, dev, host_layers, n_layers: int, K: int = DECODE_STEPS, W: int = DECODE_WARMUP) -> dict:
    """host_layers: the config-0 layers (no popularity bias). A fresh bf16 token per step."""
    from gyro_moe import abi
    ctx = abi.Context(device=dev.index, max_tokens=1, max_layers=n_layers)
    try:
        for l, layer in enumerate(host_layers):
            ctx.upload_layer(l, layer)
        xs_host = step_tokens(W + K, 1, 0)
        xs = torch.from_numpy(xs_host.view(np.int16)).to(dev).view(torch.bfloat16)
        y = torch.empty((1, E), dtype=torch.float32, device=dev)
        stream = torch.cuda.ExternalStream(ctx.stream(), device=dev)
        for i in range(W):
            ticket = ctx.stack_forward(0, n_layers, xs[i], y)
        ctx.wait(ticket)
        tickets = []
        ms, per, clocks = timed_steps(torch, stream, dev, K,
                                      lambda i: tickets.append(ctx.stack_forward(0, n_layers, xs[W + i], y)),
                                      per_step=True)
        ctx.wait(tickets[-1])             # raises if a kernel reported an error during the timed steps
        # per-kernel durations: the same steps replayed with phase events between the kernels
        ctx.set_flags(abi.GX_FLAG_PROFILE)
        prof = []
        for i in range(min(K, 8) + 1):
            ctx.wait(ctx.stack_forward(0, n_layers, xs[W + i % K], y))
            if i:
                prof.append(ctx.timings())
        ctx.set_flags(0)
        layers = max(sum(p.layers for p in prof), 1)
        gate_up_s = sum(p.gate_up_ns for p in prof) / layers * 1e-9
        down_s = sum(p.down_ns for p in prof) / layers * 1e-9
        router_s = sum(p.router_ns for p in prof) / layers * 1e-9
        # end to end: host bf16 token in (pinned staging inside the library), host f32 out
        e2e_steps = min(K, 64)
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            ctx.stack_forward_host(0, n_layers, xs_host[W + i], out_dtype=np.float32)
        e2e_s = time.perf_counter() - t0
    finally:
        ctx.close()
    pk = peaks()
    layer_bytes = EXPERT_BYTES * U + ROUTER_BYTES
    step_s = ms / K * 1e-3
    achieved = GATE_UP_BYTES * U / gate_up_s / 1e9 if gate_up_s > 0 else None
    per_sorted = sorted(per)
    return {
        "workload": "decode: 40-layer stack of the config-0 routed layer (BASELINE.json configs[1]), batch 1, "
                    f"{K} fresh bf16 tokens",
        "value": K / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms / K, "steps": K, "warmup": W,
        "p50_us": 1e3 * per_sorted[len(per) // 2], "p95_us": 1e3 * per_sorted[min(len(per) - 1, int(0.95 * len(per)))],
        "max_us": 1e3 * per_sorted[-1],
        "latency_timing": "one CUDA event pair per step on the library stream, back-to-back steps",
        "hbm_gbs_whole_step": layer_bytes * n_layers / step_s / 1e9,
        "hbm_frac_whole_step": layer_bytes * n_layers / step_s / 1e9 / pk["hbm_gbs"],
        "roofline": {
            "kernel": "gate_up_kernel (fused Gyro decode + gate/up GEMV + SwiGLU)", "bound": "hbm",
            "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"] if achieved else None,
            "traffic": traffic_bytes("gate_up_kernel_decode_per_launch"),
            "algorithmic_bytes_per_launch": GATE_UP_BYTES * U, "launch_us": gate_up_s * 1e6,
            "per_layer_us": {"router": router_s * 1e6, "gate_up": gate_up_s * 1e6, "down": down_s * 1e6},
            "timing": "CUDA events between the kernels of 8 replayed steps (the events separate the kernels, so "
                      "these durations exclude the programmatic overlap of the timed steps)",
            "peak_source": f"{pk['source']} (MEASURED_PEAKS.json hbm_gbs, burst copy)",
        },
        "e2e": {"value": e2e_steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": E * 2, "d2h_bytes_per_step": E * 4,
                "steps": e2e_steps, "api": "gx_stack_forward_host (host bf16 in, host f32 out)"},
        "gpu_launches": K * n_layers * 3,
        "clocks": clocks,
        "l2": "inputs larger than L2: each step reads 40 x 8 distinct experts (267 MB)",
    }


# ------------------------------------------------------------------------------------------
# Config 2: one 1,024-token sequence through the config-0 layer
# ------------------------------------------------------------------------------------------
def measure_prefill(torch, dev, T: int, K: int, W: int) -> dict:
    from gyro_moe import abi, synth
    layer = synth.make_layer(LAYER_SEED, zipf=1.1)
    ctx = abi.Context(device=dev.index, max_tokens=T, max_layers=1)
    try:
        ctx.upload_layer(0, layer)
        xs_host = step_tokens(4, T, 0)
        xs = torch.from_numpy(xs_host.view(np.int16)).to(dev).view(torch.bfloat16)
        y = torch.empty((T, E), dtype=torch.bfloat16, device=dev)
        ids = torch.empty((T, U), dtype=torch.int32, device=dev)
        for i in range(W):
            ticket = ctx.forward(0, xs[i % 4], y, ids)
        ctx.wait(ticket)
        stream = torch.cuda.ExternalStream(ctx.stream(), device=dev)
        tickets = []
        ms, _, clocks = timed_steps(torch, stream, dev, K, lambda i: tickets.append(ctx.forward(0, xs[i % 4], y)))
        ctx.wait(tickets[-1])
        ctx.set_flags(abi.GX_FLAG_PROFILE)
        prof = []
        for i in range(5):
            ctx.wait(ctx.forward(0, xs[i % 4], y, ids))
            prof.append(ctx.timings())
        ctx.set_flags(0)
        ids_np = ids.cpu().numpy().astype(np.int64)
        e2e_steps = min(K, 16)
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            ctx.forward_host(0, xs_host[i % 4], out_dtype=np.uint16)
        e2e_s = time.perf_counter() - t0
    finally:
        ctx.close()
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
    return {
        "workload": f"prefill: one {T}-token bf16 sequence through the config-0 routed layer, Zipf(1.1) routing "
                    "(BASELINE.json configs[2])",
        "value": K * T / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms / K, "steps": K, "warmup": W,
        "experts_hit": int((counts > 0).sum()), "max_segment": int(counts.max()), "row_tiles": tiles,
        "roofline": {
            "kernel": "moe_gemm_ts_kernel<gate/up> (tcgen05 grouped GEMM, decoded weights in TMEM, SwiGLU epilogue)",
            "bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
            "frac": achieved / pk["bf16_tflops"], "traffic": traffic_bytes("moe_gemm_gateup_prefill_per_launch"),
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
        "gpu_launches": K * 9,
        "clocks": clocks,
        "l2": "inputs larger than L2: a step reads every touched expert (up to 214 MB)",
    }


# ------------------------------------------------------------------------------------------
# Config 3: decode-GEMV type sweep
# ------------------------------------------------------------------------------------------
def reference_decode(type_id: int, packed: np.ndarray, n: int) -> np.ndarray:
    """The CPU decoder the decoded weights must match bit for bit: the reference's own tq_ref.c
    (oracle/_ref) when it was built, else its restatement in oracle/."""
    import ctypes
    from oracle import oracle
    ref = oracle.ref_lib()
    out = np.empty(n, np.float32)
    if ref is not None:
        src = np.ascontiguousarray(packed, dtype=np.uint8)
        if ref.tq_dequantize_row(type_id, src.ctypes.data, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n) != 0:
            raise RuntimeError("reference decoder rejected the blocks")
        return out
    return oracle.decode_row(type_id, packed.tobytes(), n)


def measure_sweep(torch, dev, l2_bytes: int, reps: int = 5, warm: int = 3, only: str = "",
                  l2x: float = 4.5) -> dict:
    """Every Gyro type at [512x2048] and [2048x512]: n distinct matrices of the projection shape,
    together more than 4.5x the L2, stored as one tall matrix (rows are independent, so row block
    i is matrix i) and multiplied in one launch per batch size. only = "TYPE:ROWSxCOLS" runs one
    case (profiling)."""
    from gyro_moe import abi, synth
    pk = peaks()
    rows_out = []
    for type_id in sorted(synth.BLOCK_BYTES):
        for rows, cols in SWEEP_SHAPES:
            if only and only != f"{synth.TYPE_NAMES[type_id]}:{rows}x{cols}":
                continue
            proj = rows * (cols // 128) * synth.BLOCK_BYTES[type_id]
            n_mats = int(np.ceil(l2x * l2_bytes / proj))
            W = synth.packed_matrix(np.random.default_rng(type_id * 100 + rows), type_id, rows * n_mats, cols)
            # bit-exact decoded weights: a sample of 64 rows against the reference CPU decoder
            sample = np.ascontiguousarray(W[:64]).reshape(-1)
            count = 64 * cols
            entry = {"type": synth.TYPE_NAMES[type_id], "shape": f"{rows}x{cols}", "matrices": n_mats,
                     "packed_bytes": int(W.nbytes)}
            with abi.Context(device=dev.index, max_tokens=16, max_layers=1) as ctx:
                rc, _, err = ctx.decode_blocks(type_id, sample, count, expected=reference_decode(type_id, sample, count))
                entry["decode_bit_exact"] = rc == 0
                h = ctx.upload_matrix(type_id, rows * n_mats, cols, W)
                del W
                stream = torch.cuda.ExternalStream(ctx.stream(), device=dev)
                for b in SWEEP_BATCHES:
                    x = torch.randn((b, cols), dtype=torch.float32, device=dev)
                    y = torch.empty((b, rows * n_mats), dtype=torch.float32, device=dev)
                    torch.cuda.synchronize(dev)
                    for _ in range(warm):
                        t = ctx.matvec(h, x, y)
                    ctx.wait(t)
                    tickets = []
                    ms, _, _ = timed_steps(torch, stream, dev, reps, lambda i: tickets.append(ctx.matvec(h, x, y)))
                    ctx.wait(tickets[-1])
                    s = ms / reps * 1e-3
                    act = b * (rows + cols) * 4 * n_mats
                    gbs = (entry["packed_bytes"] + act) / s / 1e9
                    entry[f"batch{b}"] = {"gbs": gbs, "frac": gbs / pk["hbm_gbs"], "launch_us": s * 1e6,
                                          "weights_per_s": rows * cols * n_mats / s}
            rows_out.append(entry)
    return {
        "workload": "decode-GEMV type sweep (BASELINE.json configs[3]): 8 Gyro types x [512x2048], [2048x512] x "
                    "batch 1/4/16, f32 activations",
        "unit": "GB/s", "peak": pk["hbm_gbs"], "peak_source": f"{pk['source']} (MEASURED_PEAKS.json hbm_gbs)",
        "bytes": "packed codes + scales of all matrices + batch x (rows + cols) x 4 B of activations per matrix",
        "timing": f"CUDA events around {reps} launches after {warm} warm-up launches; one launch covers {l2x}x L2 "
                  "of distinct matrices (no L2 reuse between launches)",
        "kernel": "matvec_kernel (bulk-copied tiles, 16 bank-interleaved shared-memory codebooks, mma.sync)",
        "results": rows_out,
        "decode_bit_exact_all": all(r["decode_bit_exact"] for r in rows_out),
    }


# ------------------------------------------------------------------------------------------
# Config 4 (default): expert-parallel prefill of the packed batch through the 40-layer stack
# ------------------------------------------------------------------------------------------
def run_ep(args):
    """BASELINE.json config 4 on N ranks (N = 1 included): each rank holds 256/N experts of every
    layer (plus replicas of the hot ones) and routes its own sequences (rank_sequences balances
    their tokens); dispatch and combine run inside the library."""
    from gyro_moe import abi, metrics, synth
    from oracle import oracle      # the checker (parity sample) and the timed CPU baseline only

    d = Dist()
    torch, dev, world, rank = d.torch, d.dev, d.world, d.rank
    nccl_id = None
    if world > 1:
        idt = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            idt.copy_(torch.frombuffer(bytearray(abi.unique_id()), dtype=torch.uint8))
        d.pg.broadcast(idt, 0)
        nccl_id = bytes(idt.cpu().numpy())
    lengths, offsets, xall = ep_batch()
    T = int(offsets[-1])
    mine = rank_tokens(offsets, xall, rank, world)
    n_tok = mine.shape[0]
    max_tok = max(rank_tokens(offsets, xall, r, world).shape[0] for r in range(world))
    K, W = args.steps, args.warmup
    ctx = abi.Context(device=d.local, max_tokens=max(max_tok, 1), max_layers=args.layers, rank=rank, world=world,
                      nccl_id=nccl_id)
    secondary = world == 1 and not args.no_secondary
    keep_host = world == 1 and (secondary or not args.no_cpu_baseline)
    host_layers = []
    # parity sample: the oracle runs the sampled tokens through its own chain as the layers are
    # uploaded (the whole-chain comparison; the per-layer check follows the timed region)
    prow = parity_rows(n_tok, args.parity_tokens)
    cur = bf16_values(mine[prow])
    for l in range(args.layers):
        layer = synth.make_layer(LAYER_SEED + l, zipf=1.1)
        ctx.upload_layer(l, layer)
        if prow.size:
            out, _, _ = oracle.moe_ffn(layer, oracle.rms_norm(cur))
            cur = cur + out
        if keep_host:
            host_layers.append(layer)
    ref_out = cur
    # two input batches alternate: the same tokens scaled by 1 and by -1 route differently
    x0 = torch.from_numpy(mine.view(np.int16)).to(dev).view(torch.bfloat16)
    xs = [x0, -x0]
    y = torch.empty((n_tok, E), dtype=torch.bfloat16, device=dev)
    for i in range(W):
        ticket = ctx.stack_forward(0, args.layers, xs[i % 2], y)
    ctx.wait(ticket)
    replicas = []
    rep0 = []
    if world > 1 and not args.no_replicas:
        # load balance: the warm-up's routed-slot counts, summed over ranks, choose per layer the
        # popular experts every rank serves for its own tokens
        from gyro_moe import balance
        for l in range(args.layers):
            cnt = torch.from_numpy(ctx.expert_counts(l, reset=True).astype(np.int64)).to(dev)
            d.pg.all_reduce(cnt)
            rep = balance.choose_replicas(cnt.cpu().numpy(), world)
            ctx.replicate_experts(l, rep)
            replicas.append(len(rep))
            if l == 0:
                rep0 = list(rep)
        for i in range(W):
            ticket = ctx.stack_forward(0, args.layers, xs[i % 2], y)
        ctx.wait(ticket)
    exchange = ctx.caps().ep_exchange
    stream = torch.cuda.ExternalStream(ctx.stream(), device=dev)
    d.barrier()
    tickets = []
    ms, _, clocks = timed_steps(torch, stream, dev, K,
                                lambda i: tickets.append(ctx.stack_forward(0, args.layers, xs[i % 2], y)))
    ctx.wait(tickets[-1])
    (ms,) = d.reduce([ms], "max")

    # parity (after the timed region), per layer: the batch goes through the stack one layer at a
    # time in f32 (the same pre-norm residual step, x_{l+1} = x_l + MoE_l(RMSNorm(x_l))), and for
    # the sampled tokens the oracle computes MoE_l on the GPU's own input x_l of that layer. The
    # whole-stack comparison (both sides run their own 40-layer chain) is reported as well: there
    # a near tie in a deep layer's top-k can route a token differently on the two sides, which is
    # not a per-layer error, so it is not the pass/fail criterion.
    ctx.wait(ctx.stack_forward(0, args.layers, xs[0], y))
    got_chain = y[torch.from_numpy(prow).to(dev)].float().cpu().numpy() if prow.size else np.zeros((0, E), np.float32)
    ids = torch.empty((n_tok, U), dtype=torch.int32, device=dev)
    ctx.set_flags(abi.GX_FLAG_PROFILE)
    ctx.wait(ctx.forward(0, xs[0], y, ids))
    ph = ctx.timings()
    ctx.set_flags(0)
    ids_np = ids.cpu().numpy()
    prow_t = torch.from_numpy(prow).to(dev)
    xl = xs[0].float().contiguous()
    yl = torch.empty_like(xl)
    sample_in, sample_out = [], []
    for l in range(args.layers):
        ctx.wait(ctx.stack_forward(l, 1, xl, yl))
        if prow.size:
            sample_in.append(xl[prow_t].cpu().numpy())
            sample_out.append(yl[prow_t].cpu().numpy())
        xl, yl = yl, xl
    worst_rel, worst_cos, sq_err, sq_ref = 0.0, 1.0, 0.0, 0.0
    ids0_raw = None
    for l in range(args.layers if prow.size else 0):
        layer = host_layers[l] if keep_host else synth.make_layer(LAYER_SEED + l, zipf=1.1)
        if l == 0:
            # the routing of the plain layer-0 call above (raw bf16 tokens, no pre-norm)
            ids0_raw = oracle.moe_ffn(layer, bf16_values(mine[prow]))[1]
        want, _, _ = oracle.moe_ffn(layer, oracle.rms_norm(sample_in[l]))
        have = sample_out[l].astype(np.float64) - sample_in[l].astype(np.float64)
        m = metrics.compare(want, have)
        worst_rel, worst_cos = max(worst_rel, m["rel_rms"]), min(worst_cos, m["cosine"])
        sq_err += float(((want.astype(np.float64) - have) ** 2).sum())
        sq_ref += float((want.astype(np.float64) ** 2).sum())
    if prow.size:
        flips = metrics.topk_sets(ids0_raw, ids_np[prow])["flips"]
        mc = metrics.compare(ref_out, got_chain)
        c_err = float(((ref_out.astype(np.float64) - got_chain) ** 2).sum())
        c_ref = float((ref_out.astype(np.float64) ** 2).sum())
    else:
        flips, c_err, c_ref, mc = 0, 0.0, 0.0, {"cosine": 1.0, "rel_rms": 0.0}
    sq_err, sq_ref, c_err, c_ref, flips_all, checked = d.reduce([sq_err, sq_ref, c_err, c_ref, flips, prow.size], "sum")
    worst_cos, chain_cos = d.reduce([worst_cos, mc["cosine"]], "min")
    worst_rel, chain_worst = d.reduce([worst_rel, mc["rel_rms"]], "max")
    parity = {"tokens_checked": int(checked), "layers_checked": args.layers,
              "rel_rms": float(np.sqrt(sq_err / sq_ref)) if sq_ref else 0.0,
              "worst_layer_rel_rms": worst_rel, "worst_layer_cosine": worst_cos, "layer0_topk_flips": int(flips_all),
              "oracle": "oracle/ CPU restatement of src/engine.zig:520-642 (strict build): MoE_l of every layer on "
                        "the GPU's own f32 input of that layer, for the sampled tokens of every rank, after the "
                        "timed region; the top-k sets of a plain layer-0 call against the oracle's on the same tokens",
              "tolerance": {"rel_rms": 1e-2, "cosine": 0.9999},
              "chain": {"rel_rms": float(np.sqrt(c_err / c_ref)) if c_ref else 0.0, "worst_rank_rel_rms": chain_worst,
                        "worst_rank_cosine": chain_cos,
                        "what": f"bf16 tokens through both sides' own {args.layers}-layer chains (informational: a "
                                "routing near-tie in a deep layer moves a token's whole remaining chain)"}}
    parity["ok"] = worst_rel <= 1e-2 and worst_cos >= 0.9999 and parity["layer0_topk_flips"] == 0

    # roofline: the gate/up grouped GEMM on every rank's received slots, one profiled layer-0 call
    per = NE // world
    flat = ids_np.reshape(-1).astype(np.int64)
    replicated = np.isin(flat, np.array(rep0, np.int64))
    own = np.bincount(flat[~replicated] // per, minlength=world).astype(np.float64)
    served = d.reduce(own.tolist(), "sum")
    slots_here = served[rank] + float(replicated.sum())
    gu_flops = slots_here * 2 * F * E * 2
    flops_sum, gu_sum, rt_sum, dn_sum, tot_sum = d.reduce(
        [gu_flops, ph.gate_up_ns * 1e-9, ph.router_ns * 1e-9, ph.down_ns * 1e-9, ph.total_ns * 1e-9], "sum")
    pk = peaks()
    achieved = flops_sum / gu_sum / 1e12 if gu_sum > 0 else None

    # end to end: host bf16 in, host bf16 out, through gx_stack_forward_host
    e2e_steps = min(K, 8)
    d.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        src = mine if i % 2 == 0 else (mine ^ np.uint16(0x8000))
        ctx.stack_forward_host(0, args.layers, src, out_dtype=np.uint16)
    (e2e_s,) = d.reduce([time.perf_counter() - t0], "max")
    (h2d_max,) = d.reduce([n_tok * E * 2], "max")
    ctx.close()

    # one GPU: router, top-k, three grouping kernels, rotation + pack (one kernel), two GEMMs (the
    # gate/up epilogue writes the down operand), combine = 9. Expert parallel: router, top-k, plan,
    # three grouping kernels, pack, two GEMMs, sum of the partial rows, plus push, bounded wait,
    # return, bounded wait with peer memory (14) or rotation and combine with NCCL (12; NCCL's
    # own kernels not counted)
    launches_per_layer = 9 if world == 1 else 14 if exchange == abi.GX_EP_PEER else 12
    line = {
        "metric": METRIC, "value": K * T / (ms / 1e3), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded; shapes and distributions of BASELINE.json config 4)",
        "config": {"workload": f"expert-parallel prefill (BASELINE.json configs[4]): {EP_SEQS} packed sequences "
                               f"(log-uniform lengths in [1, 512], {T} tokens) through the {args.layers}-layer stack "
                               "of the config-0 routed layer, Zipf(1.1)",
                   "tokens": T, "sequences": EP_SEQS, "layers": args.layers, "hidden": E, "experts": NE,
                   "experts_per_gpu": per, "top_k": U, "ffn": F, "type": "TQ2_T",
                   "parallelism": (f"expert parallel x{world} (dispatch/combine over "
                                   f"{'NVLink peer memory' if exchange == abi.GX_EP_PEER else 'NCCL'})")
                                  if world > 1 else "single GPU",
                   "tokens_per_rank_max": max_tok,
                   "l2": "inputs larger than L2: a step reads every touched expert of 40 layers"},
        "roofline": {
            "kernel": "moe_gemm_ts_kernel<gate/up> on each rank's received slots (tcgen05 grouped GEMM)",
            "bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
            "frac": achieved / pk["bf16_tflops"] if achieved else None,
            "traffic": traffic_bytes("moe_gemm_gateup_ep_per_launch"),
            "how": "sum over ranks of (received slots x 2 x F x E x 2 useful FLOPs) / sum over ranks of the gate/up "
                   "GEMM's CUDA-event time, one profiled layer-0 call after the timed region",
            "phase_ms_mean_per_rank": {"select_dispatch": rt_sum / world * 1e3, "gate_up": gu_sum / world * 1e3,
                                       "down_combine": dn_sum / world * 1e3, "layer": tot_sum / world * 1e3},
            "peak_source": f"{pk['source']} (MEASURED_PEAKS.json bf16_tflops, burst; f16 has the same dense rate)",
        },
        "parity": parity,
        "ep": {"exchange": {abi.GX_EP_PEER: "NVLink peer memory", abi.GX_EP_NCCL: "NCCL"}.get(exchange, "none"),
               "replicated_experts_per_layer": (sum(replicas) / len(replicas)) if replicas else 0,
               "tokens_per_rank": d.reduce([n_tok if r == rank else 0 for r in range(world)], "sum")},
        "e2e": {"value": e2e_steps * T / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": int(h2d_max),
                "d2h_bytes_per_step": int(h2d_max), "steps": e2e_steps,
                "api": "gx_stack_forward_host (host bf16 in, host bf16 out), every rank its own tokens; the "
                       "byte counts are the busiest rank's"},
        "gpu_launches": K * args.layers * launches_per_layer,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = oracle.max_threads()
        xf = bf16_values(mine)
        done, el, t0 = 0, 0.0, time.perf_counter()
        while el < args.cpu_seconds and done < T:
            oracle.stack(host_layers, xf[done:done + 64], threads=threads, fast=True)
            done += min(64, T - done)
            el = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": done / el, "unit": "tok/s", "cores": threads, "kind": "port",
                                "sample": f"{done} of the {T} tokens in 64-token chunks through the "
                                          f"{args.layers}-layer stack, {el:.1f} s on {threads} threads (persistent "
                                          "worker pool)"}
    if secondary:
        for layer in host_layers:                 # config 1 routes without the popularity bias
            layer["router_bias"] = None
        sec = {"decode": measure_decode(torch, dev, host_layers, args.layers)}
        del host_layers
        sec["prefill"] = measure_prefill(torch, dev, PREFILL_TOKENS, 20, 5)
        l2 = int(torch.cuda.get_device_properties(dev).L2_cache_size)
        sec["sweep"] = measure_sweep(torch, dev, l2)
        line["secondary"] = sec
        line["gpu_launches"] += sec["decode"]["gpu_launches"] + sec["prefill"]["gpu_launches"]
    if rank == 0:
        print(json.dumps(line), flush=True)
    d.close()


# ------------------------------------------------------------------------------------------
# Standalone lines for configs 1-3 (one GPU)
# ------------------------------------------------------------------------------------------
def run_single(args):
    from oracle import oracle      # the timed CPU baseline only
    d = Dist()
    torch, dev = d.torch, d.dev
    if d.world > 1:
        raise SystemExit(f"--workload {args.workload} runs on one GPU; the multi-GPU workload is ep-prefill")
    if args.workload == "decode":
        layers = list(make_layers(args.layers))
        r = measure_decode(torch, dev, layers, args.layers, args.steps, args.warmup)
        dtype = "bf16"
        scaling = "weak"
    elif args.workload == "prefill":
        r = measure_prefill(torch, dev, args.tokens, args.steps, args.warmup)
        dtype, scaling = "f16", "weak"
    else:
        r = measure_sweep(torch, dev, int(torch.cuda.get_device_properties(dev).L2_cache_size),
                          only=args.sweep_only, l2x=args.sweep_l2x)
        tq2 = next((e for e in r["results"] if e["type"] == "TQ2_T" and e["shape"] == "512x2048"), r["results"][0])
        line = {"metric": METRIC, "value": tq2["batch1"]["gbs"], "unit": "GB/s", "n_gpus": 1, "steps": 5, "warmup": 3,
                "ms_per_step": tq2["batch1"]["launch_us"] / 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; BASELINE.json config 3)",
                "config": {"workload": r["workload"], "headline": f"{tq2['type']} {tq2['shape']} batch 1"},
                "roofline": {"kernel": r["kernel"], "bound": "hbm", "achieved": tq2["batch1"]["gbs"], "peak": r["peak"],
                             "unit": "GB/s", "frac": tq2["batch1"]["frac"], "traffic": None},
                "sweep": r, "gpu_launches": 8 * 2 * 3 * 8}
        print(json.dumps(line), flush=True)
        d.close()
        return
    line = {"metric": METRIC, "value": r.pop("value"), "unit": r.pop("unit"), "n_gpus": 1, "steps": r.pop("steps"),
            "warmup": r.pop("warmup"), "ms_per_step": r.pop("ms_per_step"), "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": dtype,
            "data": "synthetic (seeded; shapes and distributions of the BASELINE.json config)",
            "config": {"workload": r.pop("workload"), "hidden": E, "experts": NE, "top_k": U, "ffn": F,
                       "type": "TQ2_T", "l2": r.pop("l2")},
            "roofline": r.pop("roofline"), "e2e": r.pop("e2e"), "gpu_launches": r.pop("gpu_launches"),
            "clocks": r.pop("clocks")}
    line.update(r)
    if not args.no_cpu_baseline and args.workload == "decode":
        threads = oracle.max_threads()
        rng = np.random.default_rng(99)
        done, t0 = 0, time.perf_counter()
        while True:
            from gyro_moe import synth
            oracle.stack(layers, synth.bf16_round(rng.standard_normal((1, E)).astype(np.float32)), threads=threads,
                         fast=True)
            done += 1
            el = time.perf_counter() - t0
            if el >= args.cpu_seconds or done >= 64:
                break
        line["cpu_baseline"] = {"value": done / el, "unit": "tok/s", "cores": threads, "kind": "port",
                                "sample": f"{done} tokens x {len(layers)} layers, batch 1, {el:.1f} s on {threads} threads"}
    print(json.dumps(line), flush=True)
    d.close()


# ------------------------------------------------------------------------------------------
# Reference arm: the reference's CPU engine (restated in oracle/) on the host cores
# ------------------------------------------------------------------------------------------
def run_reference(args):
    """The CPU engine restated in oracle/ (the reference's own CPU engine is Zig, which is absent),
    all host threads, rank 0 only. Each step is a bounded sample of the workload: ep-prefill, 64
    tokens of the packed batch through the 40-layer stack; decode, one token through the stack;
    prefill, 64 of the 1,024 tokens through the layer."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle
    from gyro_moe import synth
    threads = oracle.max_threads()
    steps = args.warmup + args.steps
    world = args.gpus
    if args.workload == "decode":
        layers = list(make_layers(args.layers))
        xs = [bf16_values(t) for t in step_tokens(steps, 1, 0)]
        run = lambda x: oracle.stack(layers, x, threads=threads, fast=True)
        scaling = "weak"
        config = {"workload": "decode: 40-layer stack of the config-0 routed layer (BASELINE.json configs[1]), "
                              f"batch 1, {DECODE_STEPS} fresh bf16 tokens", "hidden": E, "experts": NE, "top_k": U,
                  "ffn": F, "type": "TQ2_T", "l2": "inputs larger than L2: each step reads 40 x 8 distinct experts (267 MB)"}
        sample = f"{args.steps} steps x 1 token x {args.layers} layers"
    elif args.workload == "prefill":
        layer = synth.make_layer(LAYER_SEED, zipf=1.1)
        xf = bf16_values(step_tokens(1, args.tokens, 0)[0])
        xs = [xf[(64 * i) % args.tokens:(64 * i) % args.tokens + 64] for i in range(steps)]
        run = lambda x: oracle.moe_ffn(layer, x, threads=threads, fast=True)
        scaling = "weak"
        config = {"workload": f"prefill: one {args.tokens}-token bf16 sequence through the config-0 routed layer, "
                              "Zipf(1.1) routing (BASELINE.json configs[2])", "hidden": E, "experts": NE, "top_k": U,
                  "ffn": F, "type": "TQ2_T", "l2": "inputs larger than L2: a step reads every touched expert (up to 214 MB)"}
        sample = f"{args.steps} steps x 64 of the {args.tokens} tokens through the layer"
    elif args.workload == "sweep":
        print(json.dumps({"impl": "reference", "unavailable": "the decode-GEMV sweep has no CPU counterpart line; the "
                          "CPU engine is timed on the layer workloads"}), flush=True)
        return
    else:
        layers = [synth.make_layer(LAYER_SEED + l, zipf=1.1) for l in range(args.layers)]
        lengths, offsets, xall = ep_batch()
        T = int(offsets[-1])
        xf = bf16_values(xall)
        xs = [xf[(64 * i) % T:(64 * i) % T + 64] for i in range(steps)]
        run = lambda x: oracle.stack(layers, x, threads=threads, fast=True)
        scaling = "strong"
        max_tok = max(rank_tokens(offsets, xall, r, world).shape[0] for r in range(world))
        config = {"workload": f"expert-parallel prefill (BASELINE.json configs[4]): {EP_SEQS} packed sequences "
                              f"(log-uniform lengths in [1, 512], {T} tokens) through the {args.layers}-layer stack "
                              "of the config-0 routed layer, Zipf(1.1)",
                  "tokens": T, "sequences": EP_SEQS, "layers": args.layers, "hidden": E, "experts": NE,
                  "experts_per_gpu": NE // world, "top_k": U, "ffn": F, "type": "TQ2_T",
                  "tokens_per_rank_max": max_tok,
                  "l2": "inputs larger than L2: a step reads every touched expert of 40 layers"}
        sample = f"{args.steps} steps x 64 tokens of the packed batch through {args.layers} layers"
    times, done = [], 0
    for i in range(steps):
        t0 = time.perf_counter()
        run(xs[i])
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
            done += xs[i].shape[0]
    total = sum(times)
    value = done / total
    config["parallelism"] = (f"expert parallel x{world}" if world > 1 else "single GPU") + \
        f" (this arm: the CPU engine on {threads} host threads)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; shapes and distributions of the BASELINE.json config)",
        "config": config,
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample + " (oracle/ restatement of src/engine.zig:520-642 with a persistent "
                                            "worker pool as src/pool.zig:63-114; the reference's Zig engine cannot "
                                            "be built here)"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "ep-prefill":
        run_ep(args)
    else:
        run_single(args)


if __name__ == "__main__":
    main()
