#!/usr/bin/env python
"""Benchmark of the Krea2 W4A4 DiT block hot path on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (config 4 of the benchmark): 8 independent latents x 4224 tokens
(128 text + 64x64 image), 28 Krea2-shaped W4A4 blocks (hidden 6144, 48/12
heads, MLP 16384), random-init weights (N(0,0.02), H128-rotated, INT4),
synthetic N(0,1) hidden states.  One step = the 28-block forward of all 8
latents; with N ranks each rank runs 8/N latents (batch sharding, no
collective: "scaling": "strong" over the fixed 8-latent job).  ``--tp T``
runs T-way KV-head tensor parallelism inside groups of T ranks (NCCL
reduce-scatter after the out- and down-projections, INT4 all-gather before
the QKV and gate/up projections, k2b.parallel) and batch sharding across the
N/T groups.  The metric's
other half, the 28-block forward at 4050 tokens batch 1 (config 3), is
measured on rank 0 at N=1 and reported as "forward_ms_4050".

value: latents/s with inputs resident in HBM.  e2e: the same through the
public forward with every step's hidden states copied host->device from pinned
memory and its result copied back inside the timed region (the copies of
neighbouring steps overlap the forward on two copy streams, double-buffered).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "comfyui-k2-precompile_b200"))

METRIC = "W4A4 DiT forward ms @4050 tok x28 blocks; latents/s at 1/2/4/8 B200"
LATENTS = 8
TEXT, GRID = 128, 64
LENGTH = TEXT + GRID * GRID  # 4224
OP_NAMES = ["norm_quant_pre", "qkv_qknorm_rope", "attention_quant", "out_proj_residual", "norm_quant_post",
            "gate_up_swiglu_quant", "down_proj_residual"]


def _env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


# ------------------------------------------------------------ CPU baseline

CPU_SAMPLE_ROWS = 512  # token rows per CPU sample, shared by the reference arm and the cpu_baseline leg


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


_CPU_W = {}


def _cpu_weights():
    """One block's weights for the CPU arm, unpacked to fp32 codes + fp32 scales
    once per process (the GPU arm's weights are likewise prepared once, outside
    the timed region).  Values are random (irrelevant to timing)."""
    if not _CPU_W:
        import numpy as np

        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        rng = np.random.default_rng(99)
        H, F, heads, kvh = 6144, 16384, 48, 12
        for name, (n, k) in {"q": (heads * 128, H), "k": (kvh * 128, H), "v": (kvh * 128, H), "o": (H, H),
                             "g": (F, H), "u": (F, H), "d": (H, F)}.items():
            wq = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
            ws = rng.uniform(0.001, 0.01, (n, k // 128)).astype(np.float16).view(np.uint16)
            wu, swf = O.unpack_weight(wq, ws)
            _CPU_W[name] = (wu.astype(np.float32), swf)
    return _CPU_W


def cpu_sample_latent_seconds(rows_sample: int = CPU_SAMPLE_ROWS, seed: int = 0):
    """Times the CPU oracle (oracle/, a C + numpy restatement of the reference
    path) on `rows_sample` token rows of one config-4 latent through every
    stage of one block, and extrapolates to seconds per latent forward
    (x 4224/rows_sample rows x 28 blocks).  Returns (seconds, threads, note)."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    rng = np.random.default_rng(seed)
    H, F, heads, kvh = 6144, 16384, 48, 12
    W = _cpu_weights()
    x = O.bf16_bits(rng.standard_normal((rows_sample, H)).astype(np.float32))
    w = np.zeros(H, np.float32)
    mod = O.bf16_bits(rng.normal(0, 0.1, (6, 1, H)).astype(np.float32))
    normw = np.zeros(128, np.float32)
    pos = np.stack([np.arange(LENGTH), np.arange(LENGTH)], 1).astype(np.float32)
    freqs = O.rope_table(pos, (64, 64), 10000.0)
    kv = O.bf16_bits(rng.standard_normal((1, kvh, LENGTH, 128)).astype(np.float32))
    O.lib()
    t0 = time.perf_counter()
    xq, xs = O.norm_quant(x, w, mod[0], mod[1])
    pq = O.gemm_w4a4(xq, xs, None, None, unpacked=W["q"])
    pk = O.gemm_w4a4(xq, xs, None, None, unpacked=W["k"])
    pv = O.gemm_w4a4(xq, xs, None, None, unpacked=W["v"])
    q = O.qk_norm_rope(pq, heads, normw, 1e-6, freqs, LENGTH)
    O.qk_norm_rope(pk, kvh, normw, 1e-6, freqs, LENGTH)
    O.bf16_bits(pv)
    q4 = q.reshape(1, rows_sample, heads, 128).transpose(0, 2, 1, 3)
    o = O.attention(q4, kv, kv).reshape(rows_sample, H)
    oq, os_ = O.rotate_quant(o)
    x1 = O.gated_residual(O.gemm_w4a4(oq, os_, None, None, unpacked=W["o"]), mod[2], x, rows_sample)
    hq_in, hs_in = O.norm_quant(x1, w, mod[3], mod[4])
    hq, hs = O.swiglu_quant(O.gemm_w4a4(hq_in, hs_in, None, None, unpacked=W["g"]),
                            O.gemm_w4a4(hq_in, hs_in, None, None, unpacked=W["u"]))
    O.gated_residual(O.gemm_w4a4(hq, hs, None, None, unpacked=W["d"]), mod[5], x1, rows_sample)
    dt = time.perf_counter() - t0
    per_latent = dt * (LENGTH / rows_sample) * 28
    note = (f"oracle/ C+numpy port (group GEMMs as exact fp32 BLAS matmuls of the INT4 codes), one block on "
            f"{rows_sample} of {LENGTH} token rows of one latent (all 7 stages, attention over all {LENGTH} keys), "
            f"{dt:.2f} s, scaled x{LENGTH / rows_sample:.2f} rows x28 blocks; CPU: {cpu_model()}")
    return per_latent, O._workers(), note


def workload_config():
    """The config-4 workload keys shared by both bench arms."""
    return {"workload": "config 4: 8 latents x 4224 tokens (128 text + 64x64 image), 28 Krea2 blocks",
            "latents": LATENTS, "tokens_per_latent": LENGTH, "blocks": 28, "hidden": 6144, "heads": 48,
            "kvheads": 12, "mlp": 16384}


def run_reference(args, rank):
    """--impl reference: the reference path's CPU restatement (the reference's
    own kernels are SM89 CUDA + un-vendored comfy-kitchen and cannot build
    here), timed on the host cores.  Each step is one bounded sample."""
    if rank != 0:
        return
    samples = []
    threads, note = 1, ""
    for i in range(args.warmup + args.steps):
        sec, threads, note = cpu_sample_latent_seconds(rows_sample=CPU_SAMPLE_ROWS, seed=i)
        if i >= args.warmup:
            samples.append(sec)
    per_latent = statistics.median(samples)
    value = 1.0 / per_latent
    line = {
        "metric": METRIC, "value": value, "unit": "latents/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_latent * LATENTS * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "w4a4: int4 x int4 codes -> exact fp32 group sums / bf16 attention",
        "data": "synthetic",
        "config": dict(workload_config(), parallelism=f"host CPU, {threads} threads",
                       sampling="bounded row sample per step, extrapolated (see cpu_baseline.sample)"),
        "cpu_baseline": {"value": value, "unit": "latents/s", "cores": threads, "kind": "port", "sample": note},
        "e2e": {"value": value, "unit": "latents/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU helpers

class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, indices):
        self.indices = set(indices)
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._t.join(timeout=2)
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if self.indices and idx not in self.indices:
                continue
            try:
                sm.append(float(parts[1].split()[0]))
                mx = float(parts[2].split()[0])
                power.append(float(parts[3].split()[0]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def int8_peak_tops(torch):
    """Dense int8 tensor throughput measured here: torch._int_mm (cuBLASLt)
    8192^3, best of 10 with CUDA events."""
    n = 8192
    a = torch.randint(-8, 8, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-8, 8, (n, n), dtype=torch.int8, device="cuda").t()
    for _ in range(3):
        torch._int_mm(a, b)
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


def recorded_int8_peak():
    """The int8 tensor peak the roofline fraction is reported against: a fixed,
    recorded measurement (profiles/int8_peak.json), so that the fraction does not
    move with the per-run probe."""
    with open(os.path.join(ROOT, "profiles", "int8_peak.json")) as f:
        return json.load(f)


def load_traffic():
    """dram bytes per launch of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


# ------------------------------------------------- single-kernel profiling

def run_kernel_case(args):
    """--kernel NAME: launches one kernel of the block on a small synthetic
    case (one latent by default) `--reps` times; used for ncu captures."""
    import torch

    from k2b import ops
    from k2b.model import ModelConfig, quantize_weight, rope_positions, rope_table

    cfg = ModelConfig()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rows = args.rows
    g = torch.Generator(device=dev).manual_seed(5)
    H, F = cfg.hidden, cfg.mlp

    def weight(n, k):
        q, s = quantize_weight((torch.randn((n, k), generator=g, device=dev) * 0.02).to(torch.bfloat16))
        return ops.prepare_weight(q, s)

    x = torch.randn((rows, H), generator=g, device=dev).to(torch.bfloat16)
    w = torch.zeros(H, device=dev)
    mod = (torch.randn((6, 1, H), generator=g, device=dev) * 0.1).to(torch.bfloat16)
    # the block loop's forms: INT4 codes in e4m3 byte containers between kernels
    xq, xs = ops.norm_quant_e4m3(x, w, mod[0], mod[1])
    name = args.kernel
    if name == "norm_quant":
        fn = lambda: ops.norm_quant_e4m3(x, w, mod[0], mod[1])
    elif name == "qkv":
        wq, wk, wv = weight(cfg.heads * 128, H), weight(cfg.kvheads * 128, H), weight(cfg.kvheads * 128, H)
        L = rows
        freqs = rope_table(rope_positions(L % 64, L // 64, 64), (64, 64)).to(dev)
        nw = torch.zeros(128, device=dev)
        fn = lambda: ops.qkv_e4m3(xq, xs, wq, wk, wv, nw, nw, freqs, length=L)
    elif name == "out_proj":
        wo = weight(H, H)
        fn = lambda: ops.gated_residual_e4m3(xq, xs, wo, mod[2], x, length=rows)
    elif name == "gate_up":
        wg, wu = weight(F, H), weight(F, H)
        fn = lambda: ops.swiglu_quant_e4m3(xq, xs, wg, wu)
    elif name == "down":
        wd = weight(H, F)
        codes = torch.randint(-8, 8, (rows, F), device=dev).to(torch.float32)
        hq = codes.to(torch.float8_e4m3fn).view(torch.uint8)
        hs = torch.full((rows, F // 128), 0.01, dtype=torch.float16, device=dev)
        fn = lambda: ops.gated_residual_e4m3(hq, hs, wd, mod[5], x, length=rows)
    elif name == "attention":
        q = torch.randn((1, cfg.heads, rows, 128), device=dev).to(torch.bfloat16)
        k = torch.randn((1, cfg.kvheads, rows, 128), device=dev).to(torch.bfloat16)
        fn = lambda: ops.attention_quant_e4m3(q, k, k)
    else:
        raise SystemExit(f"unknown kernel {name}")
    fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    print(json.dumps({"kernel": name, "rows": rows, "reps": args.reps,
                      "avg_us": s.elapsed_time(e) * 1e3 / args.reps}), flush=True)


def run_profile_pass(args):
    """--profile: the step's kernels and nothing else (no peak probe, no
    end-to-end pass, no CPU baseline): `warmup` forward passes, then one more
    inside the NVTX range k2b_step.  Each pass launches 7 kernels per block after
    one input copy.  The default is a small case (one latent, two blocks, about
    0.5 GB on the device) for multi-pass ncu captures; the launch list of the
    full config-4 step (time only, one ncu pass) uses --profile-latents 8
    --profile-blocks 28."""
    import torch

    from k2b.model import Krea2Blocks, ModelConfig, rope_positions, rope_table, synthetic_blocks

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = ModelConfig(blocks=args.profile_blocks)
    lat = args.profile_latents
    blocks = synthetic_blocks(cfg, lat, seed=1234, device=dev)
    freqs = rope_table(rope_positions(TEXT, GRID, GRID), (64, 64), cfg.theta).to(dev)
    model = Krea2Blocks(cfg, blocks, lat, LENGTH, device=dev)
    gen = torch.Generator(device="cpu").manual_seed(77)
    x0 = torch.randn((lat * LENGTH, cfg.hidden), generator=gen).to(torch.bfloat16).to(dev)
    x = torch.empty_like(x0)
    for _ in range(args.warmup):
        x.copy_(x0)
        model.forward_(x, freqs)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("k2b_step")  # ncu --nvtx --nvtx-include k2b_step/
    x.copy_(x0)
    model.forward_(x, freqs)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    print(json.dumps({"profile_passes": args.warmup + 1, "launches_per_pass": 1 + 7 * cfg.blocks}), flush=True)


# --------------------------------------------------------------------- main

class Workload:
    """One rank's share of the config-4 job and how one step runs it.

    tp == 1: the native block loop (k2b_forward_blocks) over this rank's
    latents, 8 events per block (7 kernels).  tp > 1: k2b.parallel.TPBlocks
    over this rank's rows of its group's latents, 13 events per block
    (12 phases: 9 kernels and 4 NCCL collectives)."""

    def __init__(self, torch, cfg, topo, dev, latents, fused=True):
        from k2b.model import Krea2Blocks, rope_positions, rope_table, synthetic_blocks
        from k2b.parallel import PHASES, TPBlocks, TPPlan, shard_fn

        self.torch, self.cfg, self.topo, self.latents = torch, cfg, topo, latents
        self.freqs = rope_table(rope_positions(TEXT, GRID, GRID), (64, 64), cfg.theta).to(dev)
        rows = latents * LENGTH
        if topo.tp == 1:
            self.blocks = synthetic_blocks(cfg, latents, seed=1234, device=dev)
            self.model = Krea2Blocks(cfg, self.blocks, latents, LENGTH, device=dev)
            self.rows_here = rows
            self.phases = OP_NAMES
            self.ev_per_block = 8
        else:
            plan = TPPlan.of(cfg, topo.tp, topo.tp_rank)
            self.blocks = synthetic_blocks(cfg, latents, seed=1234, device=dev, shard=shard_fn(plan))
            self.model = TPBlocks(cfg, self.blocks, plan, topo.tp_group, latents, LENGTH, device=dev, fused=fused)
            self.rows_here = self.model.shard.chunk
            self.phases = PHASES
            self.ev_per_block = len(PHASES)
        self.plan_rows = rows

    def events(self):
        n = self.ev_per_block * self.cfg.blocks + (0 if self.topo.tp == 1 else 1)
        return [self.torch.cuda.Event(enable_timing=True) for _ in range(n)]

    def step(self, x, events=None):
        self.model.forward_(x, self.freqs, events=events)

    def phase_times(self, ev):
        """[(phase, ms)] for every block from one step's events."""
        out = []
        nb, e = self.cfg.blocks, self.ev_per_block
        for b in range(nb):
            for i, n in enumerate(self.phases):
                out.append((n, ev[e * b + i].elapsed_time(ev[e * b + i + 1])))
        return out

    def phase_work(self):
        """Algorithmic work per launch of each phase: (amount, unit kind)."""
        cfg, t = self.cfg, self.topo.tp
        H, F, L = cfg.hidden, cfg.mlp, LENGTH
        rows = self.plan_rows
        hq, kv, f = cfg.heads // t, cfg.kvheads // t, F // t
        own = rows if t == 1 else self.model.shard.count
        nq = own * (H * 2 + H // 2 + (H // 128) * 2) + H * 4 + 2 * self.latents * H * 2
        w = {"qkv": (2 * rows * (hq + 2 * kv) * 128 * H, "int"), "attn": (4 * self.latents * hq * L * L * 128, "bf16"),
             "out": (2 * rows * H * hq * 128, "int"), "gu": (2 * rows * 2 * f * H, "int"),
             "down": (2 * rows * H * f, "int"), "nq": (nq, "bytes")}
        if t == 1:
            return {"norm_quant_pre": w["nq"], "qkv_qknorm_rope": w["qkv"], "attention_quant": w["attn"],
                    "out_proj_residual": w["out"], "norm_quant_post": w["nq"], "gate_up_swiglu_quant": w["gu"],
                    "down_proj_residual": w["down"]}
        c = self.model.shard.chunk
        gather = (t - 1) * c * (H // 2 + (H // 128) * 2)  # bytes each rank receives
        rs = (t - 1) * c * H * 4                            # bytes each rank receives (fp32)
        add = own * (H * 4 + 2 * H * 2)
        return {"norm_quant_pre": w["nq"], "gather_act": (gather, "link"), "qkv_qknorm_rope": w["qkv"],
                "attention_quant": w["attn"], "out_proj_partial": w["out"], "reduce_scatter_out": (rs, "link"),
                "gated_add_norm_quant_post": (w["nq"][0] + add, "bytes"), "gather_mlp_in": (gather, "link"),
                "gate_up_swiglu_quant": w["gu"], "down_proj_partial": w["down"],
                "reduce_scatter_down": (rs, "link"), "gated_add": (add, "bytes")}

    def launches_per_step(self):
        return self.cfg.blocks * (7 if self.topo.tp == 1 else 9)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tp", type=int, default=1,
                    help="KV-head tensor-parallel degree (1, 2, 4); the remaining factor of the world is batch "
                         "sharding (8 GPUs: --tp 4 gives 4-way head TP x 2-way batch)")
    ap.add_argument("--tp-nccl", action="store_true",
                    help="with --tp: an NCCL reduce-scatter of the fp32 partials after the out/down projections "
                         "instead of the default fused projection that stores them straight into the owner rank's "
                         "buffer over NVLink peer memory (k2b_gemm_f32_scatter)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel", default=None,
                    help="profile mode: norm_quant|qkv|out_proj|gate_up|down|attention on one small case")
    ap.add_argument("--rows", type=int, default=LENGTH)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--profile", action="store_true",
                    help="profile mode: only `warmup` + one forward pass (ncu launch lists); a small case by default")
    ap.add_argument("--profile-latents", type=int, default=1)
    ap.add_argument("--profile-blocks", type=int, default=2)
    args = ap.parse_args()
    if args.kernel:
        run_kernel_case(args)
        return
    if args.profile:
        run_profile_pass(args)
        return
    args.warmup = max(args.warmup, 3)

    world = _env_int("WORLD_SIZE", 1)
    rank = _env_int("RANK", 0)
    local_rank = _env_int("LOCAL_RANK", 0)

    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from k2b import ops
    from k2b.model import Krea2Blocks, ModelConfig
    from k2b.parallel import topology

    tp = args.tp if world > 1 else 1
    topo = topology(world, rank, tp)
    lat0, lat1 = topo.latent_range(LATENTS)
    local = lat1 - lat0
    cfg = ModelConfig()
    peaks, peak_kind = measured_peaks()
    int8_tops = int8_peak_tops(torch) if rank == 0 else None
    int8_rec = recorded_int8_peak()["int8_tops"]

    wl = Workload(torch, cfg, topo, dev, local, fused=not args.tp_nccl)
    freqs = wl.freqs
    rows = wl.rows_here
    # this rank's hidden-state rows of its group's latents (whole latents when tp == 1)
    gen = torch.Generator(device="cpu").manual_seed(77 + topo.dp_index)
    x_group = torch.randn((local * LENGTH, cfg.hidden), generator=gen).to(torch.bfloat16)
    if tp == 1:
        x_host = x_group.pin_memory()
    else:
        sh = wl.model.shard
        x_host = torch.zeros((sh.chunk, cfg.hidden), dtype=torch.bfloat16)
        x_host[:sh.count] = x_group[sh.base:sh.base + sh.count]
        x_host = x_host.pin_memory()
    del x_group
    x0 = x_host.to(dev)
    x = torch.empty_like(x0)
    out_host = torch.empty_like(x_host).pin_memory()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------------------------------------------- device-resident timing
    events = [wl.events() for _ in range(args.steps)]
    for ev in events:  # create the CUDA events before their handles are passed down
        for e in ev:
            e.record()
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        x.copy_(x0)
        wl.step(x)
    torch.cuda.synchronize()
    # the sampler starts before the barrier: a rank that enters the timed
    # region while rank 0 still waits for nvidia-smi would time that wait at
    # its first collective
    sampler = ClockSampler([local_rank] if world == 1 else range(world)) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        x.copy_(x0)
        wl.step(x, events=events[i])
    end.record()
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    barrier()
    elapsed_ms = max_over_ranks(start.elapsed_time(end))
    err = ops.device_error(reset=True)
    if err:
        raise SystemExit(f"device-side wait gave up (error word {err})")
    ms_per_step = elapsed_ms / args.steps
    value = LATENTS / (ms_per_step / 1e3)

    # per-phase durations inside the timed region
    per_op = {n: [] for n in wl.phases}
    for ev in events:
        for n, ms in wl.phase_times(ev):
            per_op[n].append(ms)
    total_ms = sum(sum(v) for v in per_op.values())
    work = wl.phase_work()
    kernels = {}
    for n, ts in per_op.items():
        if not ts:
            continue
        avg = statistics.mean(ts)
        amount, kind = work[n]
        d = {"launches": len(ts), "avg_us": avg * 1e3, "share": sum(ts) / total_ms}
        if kind == "bytes":
            d["achieved"] = amount / (avg * 1e-3) / 1e9
            d["unit"] = "GB/s"
            d["frac"] = d["achieved"] / peaks["hbm_gbs"]
        elif kind == "link":
            d["achieved"] = amount / (avg * 1e-3) / 1e9
            d["unit"] = "GB/s received per rank (NCCL)"
            d["frac_of_peer_copy_770"] = d["achieved"] / 770.0
        elif kind == "bf16":
            d["achieved"] = amount / (avg * 1e-3) / 1e12
            d["unit"] = "TFLOP/s"
            d["frac"] = d["achieved"] / peaks["bf16_tflops_sustained"]
        else:
            d["achieved"] = amount / (avg * 1e-3) / 1e12
            d["unit"] = "TOP/s int"
            d["frac_of_int8_recorded"] = d["achieved"] / int8_rec
            if int8_tops:
                d["frac_of_int8_measured"] = d["achieved"] / int8_tops
            d["frac_of_int8_datasheet"] = d["achieved"] / 4500.0
        kernels[n] = d
    dom = max((k for k in kernels if work[k][1] == "int"), key=lambda k: kernels[k]["share"])
    traffic = load_traffic().get(dom) if tp == 1 else None

    # ------------------------------------------------------------ end to end
    # Every step copies its hidden states host -> device from pinned memory and
    # its result device -> host.  Two device buffers alternate: the input copy
    # of step i+1 (one copy stream) and the result copy of step i (another,
    # the other direction of the link) run while step i computes, so inside the
    # timed region only the first input copy and the last result copy are not
    # overlapped.
    cur = torch.cuda.current_stream()
    h2d_s, d2h_s = torch.cuda.Stream(), torch.cuda.Stream()
    xs = [x, torch.empty_like(x)]

    def run_e2e(n):
        mk = torch.cuda.Event
        h2d_ev, comp_ev, d2h_ev = [mk(), mk()], [mk(), mk()], [mk(), mk()]
        start = mk()
        start.record(cur)
        h2d_s.wait_event(start)
        with torch.cuda.stream(h2d_s):
            xs[0].copy_(x_host, non_blocking=True)
        h2d_ev[0].record(h2d_s)
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                nb = (i + 1) % 2
                if i >= 1:
                    h2d_s.wait_event(d2h_ev[nb])  # that buffer's previous result is out
                with torch.cuda.stream(h2d_s):
                    xs[nb].copy_(x_host, non_blocking=True)
                h2d_ev[nb].record(h2d_s)
            cur.wait_event(h2d_ev[b])
            wl.step(xs[b])
            comp_ev[b].record(cur)
            d2h_s.wait_event(comp_ev[b])
            with torch.cuda.stream(d2h_s):
                out_host.copy_(xs[b], non_blocking=True)
            d2h_ev[b].record(d2h_s)
        cur.wait_event(d2h_ev[(n - 1) % 2])

    run_e2e(args.warmup)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    run_e2e(args.steps)
    e2.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2)) / args.steps
    e2e_value = LATENTS / (e2e_ms / 1e3)
    finite = bool(torch.isfinite(out_host.float()).all())

    # ------------------------------------------- config 3 (4050 tok, batch 1)
    fwd4050 = dit_ms = dit_finite = ref_contract_ms = ref_contract_finite = None
    if world == 1:
        from k2b.model import rope_positions, rope_table

        L3 = 4050
        import copy

        b3 = []
        for b in wl.blocks:
            c = copy.copy(b)
            c.mod = b.mod[:, :1].contiguous()
            b3.append(c)
        m3 = Krea2Blocks(cfg, b3, 1, L3, device=dev)
        f3 = rope_table(rope_positions(98, 76, 52), (64, 64), cfg.theta).to(dev)
        x3 = x0[:L3].clone()
        x3w = torch.empty_like(x3)
        for _ in range(args.warmup):
            x3w.copy_(x3)
            m3.forward_(x3w, f3)
        torch.cuda.synchronize()
        s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s3.record()
        for _ in range(args.steps):
            x3w.copy_(x3)
            m3.forward_(x3w, f3)
        e3.record()
        torch.cuda.synchronize()
        fwd4050 = s3.elapsed_time(e3) / args.steps
        del m3, x3, x3w
        # the whole DiT forward around the same 28 blocks (k2b.dit): patch
        # embedding, timestep MLP, 4 W4A4 text-fusion blocks (H20/KV20) over
        # the 98 text tokens, the blocks, the final norm + projection;
        # latent 16 x 152 x 104 -> 76 x 52 image tokens
        from k2b.dit import DiTConfig, Krea2DiT, synthetic_dit

        dcfg = DiTConfig(core=cfg)
        dit = Krea2DiT(dcfg, synthetic_dit(dcfg, batch=1, seed=3, device=dev, blocks=b3))
        g3 = torch.Generator(device=dev).manual_seed(11)
        xl = torch.randn((1, dcfg.channels, 152, 104), generator=g3, device=dev).to(torch.bfloat16)
        ctx = torch.randn((1, 98, dcfg.txtdim), generator=g3, device=dev).to(torch.bfloat16)
        tsv = torch.full((1,), 0.5, device=dev)
        for _ in range(args.warmup):
            dit.forward(xl, tsv, ctx)
        torch.cuda.synchronize()
        s3.record()
        for _ in range(args.steps):
            yl = dit.forward(xl, tsv, ctx)
        e3.record()
        torch.cuda.synchronize()
        dit_ms = s3.elapsed_time(e3) / args.steps
        dit_finite = bool(torch.isfinite(yl.float()).all())
        del dit, xl, ctx, yl
        # the same 28-block forward in the reference's own contract (a ConvRot
        # W4A4 checkpoint's arithmetic: ConvRot 256, one fp32 scale per row and
        # per channel, the attention gate, joint kernels; k2b.ref_blocks)
        from k2b.ref_blocks import ref_forward, synthetic_ref_blocks

        rb = synthetic_ref_blocks(cfg, 1, seed=5, device=dev)
        for _ in range(args.warmup):
            ref_forward(cfg, rb, x0[:L3], f3, 1, L3)
        torch.cuda.synchronize()
        s3.record()
        for _ in range(args.steps):
            yr = ref_forward(cfg, rb, x0[:L3], f3, 1, L3)
        e3.record()
        torch.cuda.synchronize()
        ref_contract_ms = s3.elapsed_time(e3) / args.steps
        ref_contract_finite = bool(torch.isfinite(yr.float()).all())
        del rb, yr

    # ------------------------------------------------------------ CPU baseline
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sec, threads, note = cpu_sample_latent_seconds(rows_sample=CPU_SAMPLE_ROWS)
        cpu = {"value": 1.0 / sec, "unit": "latents/s", "cores": threads, "kind": "port", "sample": note}

    if rank == 0:
        kd = kernels[dom]
        rec = recorded_int8_peak()
        roof = {"kernel": dom, "bound": "tensor", "achieved": kd["achieved"],
                "peak": rec["int8_tops"], "unit": "TOP/s int8",
                "peak_source": "recorded measurement, profiles/int8_peak.json: " + rec["method"],
                "frac": kd["achieved"] / rec["int8_tops"],
                "peak_this_run": int8_tops, "frac_of_peak_this_run": kd.get("frac_of_int8_measured"),
                "frac_of_datasheet_4500": kd.get("frac_of_int8_datasheet"),
                "traffic": traffic,
                "work_per_launch": work[dom][0], "avg_launch_us": kd["avg_us"]}
        par = f"batch-shard x{world}" if tp == 1 else (
            f"kv-head TP x{tp} (row-sharded residual; "
            f"{'NCCL reduce-scatter' if args.tp_nccl else 'GEMM epilogue scatter over NVLink peer memory'} + "
            f"INT4 NCCL all-gather) x batch-shard x{topo.dp}")
        line = {
            "metric": METRIC, "value": value, "unit": "latents/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "w4a4: int4 x int4 codes -> exact fp32 group sums / bf16 attention", "data": "synthetic",
            "config": dict(workload_config(),
                       parallelism=par, tp=tp, dp=topo.dp, latents_per_group=local,
                       l2="inputs larger than L2 (11 GB resident weights + 415 MB hidden states per step)"),
            "forward_ms_4050": fwd4050,
            "dit_forward_ms_4050": dit_ms,
            "forward_ms_4050_reference_contract": ref_contract_ms,
            "reference_contract_note": "the 28 blocks at config 3 in the reference's own contract (ConvRot 256, "
                                       "per-row / per-channel fp32 scales, attention gate, joint kernels on e4m3 "
                                       "code bytes; k2b.ref_blocks); output finite: " + str(ref_contract_finite),
            "dit_forward_note": "whole DiT forward at config 3 (98 text + 76x52 image tokens, 1 latent): "
                                "patch embed, timestep MLP, 4 W4A4 text-fusion blocks (H20/KV20), 28 blocks, "
                                "final norm + projection (k2b.dit); output finite: " + str(dit_finite),
            "e2e": {"value": e2e_value, "unit": "latents/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": x_host.numel() * 2 * world,
                    "d2h_bytes_per_step": out_host.numel() * 2 * world},
            "roofline": roof,
            "kernels": kernels,
            "peaks": {"hbm_gbs": peaks.get("hbm_gbs"), "bf16_tflops": peaks.get("bf16_tflops"),
                      "bf16_tflops_sustained": peaks.get("bf16_tflops_sustained"), "source": peak_kind,
                      "int8_tops": int8_tops},
            "gpu_launches": wl.launches_per_step() * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "output_finite": finite,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        if tp > 1:
            wl.model.close()
        del wl
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
