#!/usr/bin/env python3
"""bench.py -- decode tokens/s of the one-token FP4 MoE FFN.

One step = one token through the MoE FFN layer of DeepSeek-V4-Flash shape:
router (256 x 4096 bf16 gate, top-6 by raw logit, softmax over the selected),
6 routed + 1 shared FP4 E2M1 expert (4096 -> 2048 -> 4096, UE8M0 per 32),
SwiGLU with the reference clamps, act quant before every matvec, combine with
w_i/sum(w) in route order.  Weights are seeded synthetic (random init, no
checkpoint), HBM-resident; every step uses a fresh token, and L2 is flushed
(256 MiB memset) between steps outside the timed events, so each step reads
its experts from HBM.

N > 1 (torchrun): the path has no exchange at batch 1, so every rank runs a
full replica on its own token stream (weak scaling, no collective on the data
path); the timed region is the max over ranks.

--impl reference: the reference's CPU implementation of the same step (the
C++ restatement of its Rust AVX2 kernels, oracle/), on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

E, HID, INTER, TOPK = 256, 4096, 2048, 6
PACKED_W13 = INTER * HID // 2            # bytes of w1 (= w3) packed
SCALES_W13 = INTER * HID // 32
PACKED_W2 = HID * INTER // 2
SCALES_W2 = HID * INTER // 32
EXPERT_BYTES = 2 * (PACKED_W13 + SCALES_W13) + PACKED_W2 + SCALES_W2   # 13,369,344
ROUTER_BYTES = E * HID * 2
SLOTS = TOPK + 1
STEP_BYTES = SLOTS * EXPERT_BYTES + ROUTER_BYTES + 2 * HID * 4
UP_BYTES = SLOTS * 2 * (PACKED_W13 + SCALES_W13)       # moe_up algorithmic bytes / launch
DOWN_BYTES = SLOTS * (PACKED_W2 + SCALES_W2)
# DRAM bytes (read + write) of one moe_up launch from an ncu capture of the
# --ncu-case moe16 workload, which processes the same units per launch
UP_TRAFFIC = 63_314_688
# DRAM bytes of one moe_decode_kernel launch (the whole config-2 step); None until
# captured with ncu
STEP_TRAFFIC = None
STEP_TRAFFIC_SOURCE = "not captured yet"
# grouped up GEMM: DRAM bytes read per algorithmic byte read in the ncu capture of the
# grouped16 case (161,668,608 / 159,088,640 bytes, bench.py --ncu-case grouped16); the
# config-3 launch is too large to capture, its traffic is scaled by the units processed
GROUPED_UP_TRAFFIC_RATIO = 161_668_608 / 159_088_640
METRIC = "decode tokens/s (one-token FP4 MoE FFN, config 2)"
WORKLOAD = ("config 2: one-token FP4 MoE FFN, 256 experts 4096->2048->4096 E2M1/UE8M0-32, "
            "bf16 router top-6 softmax-renormalised, 6 routed + 1 shared expert")


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks + throttle reasons during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [v.strip() for v in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for name, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(gpus: int):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def all_max(world, value: float) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU side (oracle = the reference's CPU kernels restated): cpu_baseline and
# the --impl reference arm.  Experts are generated per id on first use.
# ---------------------------------------------------------------------------
class HostModel:
    def __init__(self, seed: int):
        from tests import helpers as H

        self.H = H
        self.seed = seed
        self.gate = H.router_gate(seed + 7, E, HID)
        self.cache: dict = {}

    def expert(self, e: int):
        import oracle as O

        if e not in self.cache:
            keep: list = []
            w1, s1 = self.H.fp4_matrix(self.seed * 1000 + 3 * e, INTER, HID)
            w3, s3 = self.H.fp4_matrix(self.seed * 1000 + 3 * e + 1, INTER, HID)
            w2, s2 = self.H.fp4_matrix(self.seed * 1000 + 3 * e + 2, HID, INTER)
            spec = O.Fp4Expert(O.fp4_spec(w1, s1, INTER, HID, HID // 32, keep),
                               O.fp4_spec(w3, s3, INTER, HID, HID // 32, keep),
                               O.fp4_spec(w2, s2, HID, INTER, INTER // 32, keep))
            self.cache[e] = (spec, keep)
        return self.cache[e][0]

    def step(self, x):
        import oracle as O

        n, ids, w, _ = O.router(self.gate, x, TOPK, mode=0)
        arr = (O.Fp4Expert * (E + 1))()
        for e in list(ids) + [E]:
            arr[e] = self.expert(int(e))
        st, y = O.moe_combine_token(arr, ids, w, arr[E], x)
        assert st == O.OK
        return y


def cpu_run(steps: int, warmup: int, seed: int = 900, budget_s: float | None = None):
    import oracle as O

    model = HostModel(seed)
    xs = model.H.activations(seed + 1, steps + warmup, HID)
    # generate (untimed) every expert the sampled tokens route to
    for i in range(steps + warmup):
        _, ids, _, _ = O.router(model.gate, xs[i], TOPK, mode=0)
        for e in list(ids) + [E]:
            model.expert(int(e))
    for i in range(warmup):
        model.step(xs[i])
    t0 = time.perf_counter()
    done = 0
    for i in range(steps):
        model.step(xs[warmup + i])
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return done / dt, done, O.threads()


def config2_dict(world: int, fp8_shared: bool, step_bytes: int) -> dict:
    """The config-2 workload description, the same on both arms."""
    return {
        "workload": WORKLOAD, "experts": E, "topk": TOPK, "hidden": HID, "inter": INTER,
        "batch": 1,
        "shared_expert": ("fp8 e4m3 x ue8m0-128x128 (DeepSeek-V4's layout), on the FP8 "
                          "GEMV after the routed experts" if fp8_shared else "fp4"),
        "l2": "flushed between steps (256 MiB memset outside the timed events)",
        "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
        "bytes_per_step": step_bytes,
    }


# ---------------------------------------------------------------------------
def run_ours(args):
    import torch

    world, rank, local = dist_setup(args.gpus)
    import wohper_b200 as W
    from tests import helpers as H

    dev = torch.device("cuda", local)
    ctx = W.Context(local)
    stack = H.torch_fp4_experts(1000 + rank, E + 1, HID, INTER, device=dev)
    gate = torch.from_numpy(H.router_gate(1007, E, HID).view(np.int16)).to(dev)

    def wexp(e):
        w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
        return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, INTER, HID, HID // 32),
                                     W.Fp4Matvec(w3, s3, INTER, HID, HID // 32),
                                     W.Fp4Matvec(w2, s2, HID, INTER, INTER // 32))

    # --shared fp8: DeepSeek-V4's layout, an FP8 E4M3 shared expert (UE8M0 per
    # 128x128) run on the FP8 GEMV after the routed experts
    fp8_shared = args.shared == "fp8"
    if fp8_shared:
        def f8(seed, r, c):
            w, sc = H.fp8_weight(seed, r, c)
            return W.Fp8Matrix(torch.from_numpy(w).to(dev), torch.from_numpy(sc).to(dev))

        shared = W.DeepSeekV4Fp8Expert(f8(4001, INTER, HID), f8(4002, INTER, HID),
                                       f8(4003, HID, INTER))
        slots = TOPK
        shared_bytes = 3 * INTER * HID + 3 * (INTER // 128) * (HID // 128)
    else:
        shared = wexp(E)
        slots = SLOTS
        shared_bytes = EXPERT_BYTES
    up_bytes = slots * 2 * (PACKED_W13 + SCALES_W13)
    down_bytes = slots * (PACKED_W2 + SCALES_W2)
    step_bytes = TOPK * EXPERT_BYTES + shared_bytes + ROUTER_BYTES + 2 * HID * 4
    up_traffic = UP_TRAFFIC if not fp8_shared else int(UP_TRAFFIC * slots / SLOTS)
    layer = W.MoeLayer(ctx, [wexp(e) for e in range(E)], shared, gate, topk=TOPK,
                       router_mode=W.ROUTER_RAW_LOGITS, max_tokens=1)
    n_tok = args.warmup + args.steps
    xs = torch.from_numpy(H.activations(2000 + rank, n_tok, HID)).to(dev)
    y = torch.empty(1, HID, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]

    # ---- device-resident timing -------------------------------------------
    # One step = one wh_moe_ffn call, replayed from a captured CUDA graph so
    # host launch overhead never shows up as device time.  The token is
    # copied into the graph's static input and L2 is flushed before the
    # start event of every step.
    x_static = torch.empty(1, HID, device=dev)
    for i in range(args.warmup):
        flush.zero_()
        layer.forward(xs[i:i + 1], y)
    ctx.sync()
    timing = "cuda graph replay"
    graph = None
    try:
        x_static.copy_(xs[0:1])
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            layer.forward(x_static, y)  # attribute set-up outside the capture
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=cap):
                layer.forward(x_static, y)
        stream.wait_stream(cap)
        torch.cuda.synchronize()
        for i in range(args.warmup):
            x_static.copy_(xs[i:i + 1])
            flush.zero_()
            graph.replay()
        torch.cuda.synchronize()
        ctx.sync()
    except Exception as exc:  # capture unsupported: time direct calls
        graph = None
        timing = f"direct calls (graph capture failed: {type(exc).__name__})"
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for k in range(args.steps):
            x_static.copy_(xs[args.warmup + k:args.warmup + k + 1])
            flush.zero_()
            ev[k][0].record(stream)
            if graph is not None:
                graph.replay()
            else:
                layer.forward(x_static, y)
            ev[k][1].record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ctx.sync()
    ms_local = sum(a.elapsed_time(b) for a, b in ev)
    ms_total = all_max(world, ms_local)
    ms_step = ms_total / args.steps
    clocks = clk.summary()
    # parity spot check of the timed path: graph output of the last token vs a
    # direct call on the same token (bit-identical)
    y_direct = layer.forward(x_static)
    torch.cuda.synchronize()
    graph_matches_direct = bool(torch.equal(y_direct, y))
    del graph

    # ---- roofline of the timed kernel (profiling: CUDA events around it) -----
    def profile_phases():
        ctx.set_profiling(True)
        phases = []
        for k in range(min(args.steps, 10)):
            flush.zero_()
            layer.forward(xs[args.warmup + k:args.warmup + k + 1], y)
            phases.append(ctx.phase_times())
        ctx.set_profiling(False)
        ctx.sync()
        return np.array(phases)

    ph3 = profile_phases()
    fused = ph3.shape[1] == 1  # the timed step ran as the persistent decode kernel
    step_kernel_ms = float(ph3[:, 0].mean()) if fused else None
    # the other schedule of the same step, for comparison (A/B)
    layer.set_fused_decode(not fused)
    ph_ab = profile_phases()
    layer.set_fused_decode(fused)
    if fused:
        ph3, ph_ab = ph_ab, ph3
    fused_ab_ms = float(ph_ab[:, 0].mean()) if ph_ab.shape[1] == 1 else None
    up_ms = float(ph3[:, 1].mean())
    down_ms = float(ph3[:, 2].mean())
    router_ms = float(ph3[:, 0].mean())
    peak, peak_kind = peaks()
    up_gbs = up_bytes / (up_ms * 1e-3) / 1e9

    # ---- end to end through the C ABI with host buffers ---------------------
    # wh_moe_ffn takes the token and the output as pinned host memory (the
    # reference's interface is host slices): a kernel pulls x over the bus into
    # device scratch and moe_down writes y straight into host memory, so each
    # step moves hidden*4 bytes in each direction with no copy-engine transfer
    xh = torch.from_numpy(H.activations(3000 + rank, n_tok, HID)).pin_memory()
    yh = torch.empty(args.steps, HID).pin_memory()
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for i in range(args.warmup):
        flush.zero_()
        layer.forward(xh[i:i + 1], yh[0:1])
    torch.cuda.synchronize()
    barrier(world)
    for k in range(args.steps):
        flush.zero_()
        ev2[k][0].record(stream)
        layer.forward(xh[args.warmup + k:args.warmup + k + 1], yh[k:k + 1])
        ev2[k][1].record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = all_max(world, sum(a.elapsed_time(b) for a, b in ev2)) / args.steps
    # the host copy holds the device results of the same tokens, bit for bit
    e2e_check = layer.forward(xh[args.warmup:args.warmup + 1].to(dev))
    torch.cuda.synchronize()
    e2e_matches_device = bool(torch.equal(e2e_check.cpu(), yh[0:1]))
    ctx.sync()

    result = None
    if rank == 0:
        value = world / (ms_step * 1e-3)
        result = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 6),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp4-e2m1 x fp8-e4m3 (act-quant) products, f32 accumulate",
            "data": "synthetic (seeded random-init weights and N(0,1) tokens)",
            "config": config2_dict(world, fp8_shared, step_bytes),
            "step_hbm_gbs": round(step_bytes / (ms_step * 1e-3) / 1e9, 1),
            "phases_ms": {"router": round(router_ms, 5), "moe_up": round(up_ms, 5),
                          "moe_down": round(down_ms, 5)},
            "persistent_decode_kernel_ms": (round(fused_ab_ms, 5) if fused_ab_ms is not None
                                            else None),
            "roofline": ({
                "kernel": "moe_decode_kernel (router + w1/w3 + SwiGLU + act quant + w2 + combine, "
                          "one persistent kernel)",
                "bound": "hbm", "achieved": round(step_bytes / (step_kernel_ms * 1e-3) / 1e9, 1),
                "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                "frac": round(step_bytes / (step_kernel_ms * 1e-3) / 1e9 / peak, 4),
                "algorithmic_bytes": step_bytes, "kernel_ms": round(step_kernel_ms, 5),
                "traffic": STEP_TRAFFIC,
                "traffic_source": STEP_TRAFFIC_SOURCE,
            } if fused else {
                "kernel": f"moe_up_kernel (w1+w3 FP4 matvecs of {slots} experts + SwiGLU + "
                          "act quant)",
                "bound": "hbm", "achieved": round(up_gbs, 1), "peak": peak,
                "peak_kind": peak_kind, "unit": "GB/s", "frac": round(up_gbs / peak, 4),
                "algorithmic_bytes": up_bytes, "traffic": up_traffic,
                "traffic_source": "ncu dram__bytes_read+write of one moe_up launch "
                                  "(bench.py --ncu-case moe16: same 7 experts' w1/w3 per launch)"
                                  + (", scaled by 6/7 slots" if fp8_shared else ""),
                "down_kernel_gbs": round(down_bytes / (down_ms * 1e-3) / 1e9, 1),
            }),
            "e2e": {"value": round(world / (e2e_ms * 1e-3), 3), "unit": "tokens/s",
                    "ms_per_step": round(e2e_ms, 6), "h2d_bytes_per_step": HID * 4,
                    "d2h_bytes_per_step": HID * 4,
                    "path": "pinned host x -> wh_moe_ffn (C ABI; the device reads x and "
                            "writes y through the mapped host buffers)",
                    "matches_device_pointer_call": e2e_matches_device},
            "gpu_launches": ((1 if fused else 3) + (4 if fp8_shared else 0)) * args.steps,
            "timing": timing,
            "graph_output_matches_direct_call": graph_matches_direct,
            "clocks": clocks,
        }
    layer.close()
    ctx.close()
    del stack
    torch.cuda.empty_cache()
    if not args.no_ep:
        # the path that shards: config 4's expert-parallel layer on the same
        # ranks, so that a 1 -> N scaling run records its curve
        ep = ep_measure(args, world, rank, local, "p2p")
        if rank == 0:
            result["ep"] = ep
            result["gpu_launches"] += 11 * args.steps
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, n, cores = cpu_run(steps=24, warmup=1, budget_s=20.0)
        result["cpu_baseline"] = {
            "value": round(v, 4), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{n} tokens of the same workload (router + 6 routed + shared expert"
                      + (", the shared expert in FP4" if fp8_shared else "") + "), "
                      "C++ restatement of the reference's AVX2 kernels, reference threading "
                      "(nproc-2 threads)"}
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return result


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    import oracle as O

    O.set_threads(os.cpu_count() or 1)
    v, n, cores = cpu_run(steps=args.steps, warmup=args.warmup)
    return {
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tokens/s",
        "n_gpus": world, "steps": n, "warmup": args.warmup,
        "ms_per_step": round(1e3 / v, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp4-e2m1 x fp8-e4m3 (act-quant) products, f32 accumulate",
        "data": "synthetic (seeded random-init weights and N(0,1) tokens)",
        "config": config2_dict(world, False, STEP_BYTES),
        "cpu_baseline": {"value": round(v, 4), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{n} tokens, one per step"},
        "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# config 1: one FP8 block-scaled GEMV, W [4096 x 4096] E4M3 + UE8M0 per 128x128
# ---------------------------------------------------------------------------
R1 = C1 = 4096
FP8_BYTES = R1 * C1 + (R1 // 128) * (C1 // 128) + 4 * C1 + 4 * R1   # 16,811,008 per call
FP8_COPIES = 16          # distinct weight matrices: 269 MB, over twice the 126 MB L2
# DRAM bytes (read + write) of one fp8_gemv_rowgroup_kernel launch at 4096 x 4096 from
# an ncu capture (bench.py --ncu-case fp8)
FP8_TRAFFIC = 16_831_232
METRIC1 = "FP8 GEMV HBM GB/s (config 1: 4096x4096 E4M3, UE8M0 per 128x128, f32 x)"
WORKLOAD1 = ("config 1: gemv_fp8_e4m3_ue8m0_tensorwise, W [4096 x 4096] E4M3 of N(0,0.05), "
             "UE8M0 block scales 2^[-8,-2] per 128x128, x f32 N(0,1), f32 accumulate in the "
             "reference's 16-chain order; one GEMV per step over 16 distinct weight copies "
             "in rotation, back to back as a decode step's projections run")


def config1_dict(world: int) -> dict:
    return {"workload": WORKLOAD1, "rows": R1, "cols": C1, "batch": 1,
            "weight_copies": FP8_COPIES,
            "l2": f"inputs larger than L2: {FP8_COPIES} distinct weight copies "
                  f"({FP8_COPIES * R1 * C1 >> 20} MiB) in rotation",
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            "bytes_per_step": FP8_BYTES}


def config1_cpu(budget_s: float, threads_all: bool):
    """The reference's tensorwise FP8 GEMV (oracle restatement) on host cores:
    (GB/s of the same algorithmic bytes, calls, threads)."""
    import oracle as O
    from tests import helpers as H

    if threads_all:
        O.set_threads(os.cpu_count() or 1)
    w, sc = H.fp8_weight(11, R1, C1)
    x = H.activations(12, 1, C1).reshape(-1)
    O.fp8_gemv(w, sc, x, R1, C1, R1 // 128, C1 // 128)  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        st, _ = O.fp8_gemv(w, sc, x, R1, C1, R1 // 128, C1 // 128)
        assert st == O.OK
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return FP8_BYTES * n / dt / 1e9, n, O.threads()


def run_config1(args):
    import torch

    world, rank, local = dist_setup(args.gpus)
    import oracle as O
    import wohper_b200 as W
    from tests import helpers as H

    dev = torch.device("cuda", local)
    ctx = W.Context(local)
    w0, s0 = H.fp8_weight(11 + rank, R1, C1)
    x0 = H.activations(12 + rank, 1, C1).reshape(-1)
    # distinct copies (the same bytes at distinct addresses: every call reads
    # its weights from HBM, never from L2)
    wd = [torch.from_numpy(w0).to(dev) for _ in range(FP8_COPIES)]
    sd = torch.from_numpy(s0).to(dev)
    x = torch.from_numpy(x0).to(dev)
    ys = torch.empty(FP8_COPIES, R1, device=dev)
    stream = torch.cuda.current_stream()

    def call(i, xin=x, yout=None):
        W.gemv_fp8_e4m3_ue8m0_tensorwise(ctx, wd[i % FP8_COPIES], sd, xin,
                                         ys[i % FP8_COPIES] if yout is None else yout)

    for i in range(max(args.warmup, FP8_COPIES)):
        call(i)
    ctx.sync()
    # parity spot check of the timed path: bit-exact with the reference order
    st, want = O.fp8_gemv(w0, s0, x0, R1, C1, R1 // 128, C1 // 128)
    parity = bool(st == O.OK and np.array_equal(ys[0].cpu().numpy().view(np.uint32),
                                                 want.view(np.uint32)))
    # ---- K calls back to back, captured once as a CUDA graph ---------------
    K = args.steps
    timing = "cuda graph of the K calls (PDL between them)"
    graph = None
    try:
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=cap):
                for i in range(K):
                    call(i)
        stream.wait_stream(cap)
        torch.cuda.synchronize()
        for _ in range(max(1, args.warmup // K)):
            graph.replay()
        torch.cuda.synchronize()
    except Exception as exc:
        graph = None
        timing = f"direct calls (graph capture failed: {type(exc).__name__})"
        torch.cuda.synchronize()
    ctx.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for i in range(K):
                call(i)
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ctx.sync()
    ms_step = all_max(world, e0.elapsed_time(e1)) / K
    del graph
    # ---- one isolated call (L2 flushed before it), for comparison ----------
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    iso = []
    for i in range(8):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        call(i)
        b.record(stream)
        torch.cuda.synchronize()
        iso.append(a.elapsed_time(b))
    iso_ms = statistics.median(iso)
    # ---- end to end: pinned host x in, host y out, every call -------------
    xh = torch.from_numpy(H.activations(13 + rank, K, C1)).pin_memory()
    yh = torch.empty(K, R1).pin_memory()
    xd = torch.empty(C1, device=dev)
    yd = torch.empty(R1, device=dev)
    for i in range(args.warmup):
        xd.copy_(xh[i], non_blocking=True)
        call(i, xd, yd)
        yh[i].copy_(yd, non_blocking=True)
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(K):
        xd.copy_(xh[i], non_blocking=True)
        call(i, xd, yd)
        yh[i].copy_(yd, non_blocking=True)
    b.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = all_max(world, a.elapsed_time(b)) / K
    ctx.sync()
    peak, peak_kind = peaks()
    res = None
    if rank == 0:
        gbs = FP8_BYTES / (ms_step * 1e-3) / 1e9
        res = {
            "metric": METRIC1, "value": round(gbs * world, 1), "unit": "GB/s", "n_gpus": world,
            "steps": K, "warmup": args.warmup, "ms_per_step": round(ms_step, 6),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp8-e4m3 weights x f32 x, f32 accumulate",
            "data": "synthetic (seeded E4M3 weights, N(0,1) x)",
            "config": config1_dict(world),
            "calls_per_s": round(world / (ms_step * 1e-3), 1),
            "isolated_call_ms": round(iso_ms, 5),
            "isolated_call_gbs": round(FP8_BYTES / (iso_ms * 1e-3) / 1e9, 1),
            "roofline": {"kernel": "fp8_gemv_rowgroup_kernel (one GEMV per launch)",
                         "bound": "hbm", "achieved": round(gbs, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(gbs / peak, 4),
                         "algorithmic_bytes": FP8_BYTES, "traffic": FP8_TRAFFIC,
                         "traffic_source": "ncu dram__bytes_read+write of one launch "
                                           "(bench.py --ncu-case fp8, the same shape)"},
            "e2e": {"value": round(FP8_BYTES / (e2e_ms * 1e-3) / 1e9 * world, 1), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 6), "h2d_bytes_per_step": 4 * C1,
                    "d2h_bytes_per_step": 4 * R1,
                    "path": "pinned host x -> H2D -> wh_fp8_gemv (C ABI) -> D2H pinned host y"},
            "parity_bit_exact_vs_oracle": parity,
            "gpu_launches": K, "timing": timing, "clocks": clk.summary(),
        }
    ctx.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, n, cores = config1_cpu(10.0, False)
        res["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": cores,
                               "kind": "port",
                               "sample": f"{n} calls of the same GEMV (one weight matrix), C++ "
                                         "restatement of the reference's AVX2 kernel, "
                                         "reference threading (nproc-2 threads)"}
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return res


def run_reference_config1(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    v, n, cores = config1_cpu(max(5.0, 0.2 * args.steps), True)
    return {"impl": "reference", "metric": METRIC1, "value": round(v, 3), "unit": "GB/s",
            "n_gpus": world, "steps": n, "warmup": args.warmup,
            "ms_per_step": round(FP8_BYTES / (v * 1e9) * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "fp8-e4m3 weights x f32 x, f32 accumulate",
            "data": "synthetic (seeded E4M3 weights, N(0,1) x)", "config": config1_dict(world),
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": f"{n} calls"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# config 5: the full synthetic-weight DeepSeek-V4 decode step (43 layers)
# ---------------------------------------------------------------------------
V4_LAYERS = 43
V4_VOCAB = 129280
V4_POS = 4095
V4_ATTN_BYTES = sum(r * c + (-(-r // 128)) * (-(-c // 128)) for r, c in
                    ((1024, 4096), (32768, 1024), (512, 4096), (8192, 4096), (4096, 8192)))
METRIC5 = "decode tokens/s (config 5: full synthetic 43-layer DeepSeek-V4 decode step)"


def config5_dict(world: int, batch: int, layers: int) -> dict:
    return {"workload": f"config 5: {layers} DeepSeek-V4-Flash-shape layers (mHC hc=4, MLA 64 "
                        "heads x 512 with q/kv low-rank FP8 projections, 256 routed FP4 "
                        "experts top-6 sqrt-softplus + shared), pooled head, bf16 lm_head "
                        f"129280 x 4096 top-1; KV cache filled to {V4_POS + 1} positions "
                        "(window 128 + compressed rows 512 / 32 by layer ratio)",
            "layers": layers, "batch": batch, "token_pos": V4_POS, "experts": E, "topk": TOPK,
            "hidden": HID, "inter": INTER,
            "l2": "inputs larger than L2 (about 8.6 GB of weights read per step)",
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU"}


def config5_cpu(batch: int, seed: int = 880, vocab_sample: int = 16384, layer_index: int = 2,
                reps: int = 1):
    """The reference's decode step on this host's cores, sampled (oracle = the
    reference's CPU kernels restated, composed as run_model_for_one_token does).

    One V4-Flash-shape layer -- hc_pre, attention norm, the MLA attention with
    its FP8 projections, hc_post, hc_pre, FFN norm, the sqrt-softplus router
    and the 6 routed + shared FP4 experts, hc_post -- runs for `batch`
    sequences at position 4095, then the pooled head, the final norm and the
    lm_head top-1 over `vocab_sample` vocabulary rows.  Host-generated weights
    of the config-5 shapes (generation untimed), `reps` timed passes.  Returns
    ([estimated step seconds = 43 x the layer + the head scaled to the full
    vocabulary, one per pass], threads)."""
    import oracle as O
    import wohper_b200 as Wp  # host-side rope constants only
    from tests import helpers as H

    O.set_threads(os.cpu_count() or 1)
    keep: list = []
    m = {}
    for i, (name, (r, c)) in enumerate(H.V4_SHAPES.items()):
        w, sc = H.fp8_weight(seed * 100 + i, r, c)
        keep += [w, sc]
        m[name] = O.fp8_matrix(w, sc, r, c, sc.shape[0], sc.shape[1], keep)
    g = H.rng(seed)
    qn = H.bf16_bits(1.0 + 0.1 * g.standard_normal(1024).astype(np.float32))
    kn = H.bf16_bits(1.0 + 0.1 * g.standard_normal(512).astype(np.float32))
    sink = g.standard_normal(64).astype(np.float32)
    keep += [qn, kn, sink]
    spec = O.V4Attn(HID, 64, 512, 448, 1024, 8, 1024, 128, m["wq_a"], m["wq_b"], m["wkv"],
                    m["wo_a"], m["wo_b"], qn.ctypes.data, kn.ctypes.data, sink.ctypes.data)
    attn_norm = H.bf16_bits(1.0 + 0.1 * g.standard_normal(HID).astype(np.float32))
    ffn_norm = H.bf16_bits(1.0 + 0.1 * g.standard_normal(HID).astype(np.float32))
    hc = 4

    def hc_params(mix):
        return ((0.02 * g.standard_normal((mix, hc * HID))).astype(np.float32),
                np.array([0.5, 0.5, 0.5], np.float32),
                (0.1 * g.standard_normal(mix)).astype(np.float32))

    hc_attn, hc_ffn = hc_params((2 + hc) * hc), hc_params((2 + hc) * hc)
    head_fn = (0.02 * g.standard_normal((hc, hc * HID))).astype(np.float32)
    head_base = (0.1 * g.standard_normal(hc)).astype(np.float32)
    final_norm = H.bf16_bits(1.0 + 0.1 * g.standard_normal(HID).astype(np.float32))
    gate = H.router_gate(seed * 100 + 18, E, HID)
    bias = (0.01 * g.standard_normal(E)).astype(np.float32)
    model = HostModel(seed)
    fr = Wp.rope_inv_freqs(64, *Wp.deepseek_rope_for_layer(layer_index))
    n_comp = H.v4_compressed_count(layer_index, V4_POS)
    kv = [(g.standard_normal((V4_POS + 1, 512))).astype(np.float32) for _ in range(batch)]
    comp = [(g.standard_normal((n_comp, 512))).astype(np.float32) if n_comp else None
            for _ in range(batch)]
    xs0 = [(g.standard_normal(hc * HID)).astype(np.float32) for _ in range(batch)]
    lm = H.bf16_bits((0.02 * g.standard_normal((vocab_sample, HID))).astype(np.float32))
    # the experts the sampled tokens route to, generated before the timed region
    arr = (O.Fp4Expert * (E + 1))()
    arr[E] = model.expert(E)

    def check(st):
        if st != O.OK:
            raise RuntimeError(f"oracle status {st} in the config-5 CPU sample")

    steps = []
    for _ in range(reps):
        t_layer = 0.0
        pooled_all = []
        for b in range(batch):
            xs = xs0[b]
            t0 = time.perf_counter()
            st, y, post, cm = O.hc_pre(*hc_attn, xs, hc, HID)
            check(st)
            y = O.rms_norm(y, attn_norm)
            st, y = O.v4_attention(spec, V4_POS, y, kv[b], comp[b], fr)
            check(st)
            xs = O.hc_post(y, xs, post, cm, hc, HID)
            st, y, post, cm = O.hc_pre(*hc_ffn, xs, hc, HID)
            check(st)
            y = O.rms_norm(y, ffn_norm)
            _, ids, w, _ = O.router(gate, y, TOPK, mode=1, bias=bias, route_scale=1.5)
            t_route = time.perf_counter() - t0
            for e in ids:
                arr[int(e)] = model.expert(int(e))  # generated untimed
            t1 = time.perf_counter()
            st, y = O.moe_combine_token(arr, ids, w, arr[E], y)
            check(st)
            xs = O.hc_post(y, xs, post, cm, hc, HID)
            t_layer += t_route + time.perf_counter() - t1
            pooled_all.append(xs)
        t0 = time.perf_counter()
        for xs in pooled_all:
            pooled = O.hc_head(head_fn, 0.5, head_base, xs, hc, HID)
            pooled = O.rms_norm(pooled, final_norm)
            O.lm_head_topk(lm, pooled, 1)
        t_head = (time.perf_counter() - t0) * V4_VOCAB / vocab_sample
        steps.append(V4_LAYERS * t_layer + t_head)
    return steps, O.threads()


def run_reference_config5(args):
    """--config 5 --impl reference: the sampled CPU decode step (config5_cpu),
    one sample per step, on config 5's metric and unit."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    B = args.batch
    times, threads = config5_cpu(B, reps=args.warmup + args.steps)
    times = times[args.warmup:]
    step_s = sum(times) / len(times)
    v = B / step_s
    sample = (f"one layer (index 2, compressed rows at position 4095) and the head for {B} "
              f"sequence(s) through the oracle's composition, the lm_head over 16384 of "
              f"{V4_VOCAB} rows; the step estimated as {V4_LAYERS} x the layer + the head "
              f"scaled to the full vocabulary")
    return {
        "impl": "reference", "metric": METRIC5, "value": round(v, 4), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_s * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8/fp4 weights x act-quantised fp8 activations, f32 accumulate",
        "data": "synthetic (seeded random-init weights, N(0,1) KV cache and residual stream)",
        "config": config5_dict(world, B, args.layers),
        "cpu_baseline": {"value": round(v, 4), "unit": "tokens/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_reference_moe_batch(args, config: int):
    """--config 3/4 --impl reference: the oracle's batched MoE (exact router +
    expert-major path for config 3, the given uniform routes for config 4) on a
    16-token sample per step, all host threads, on the config's metric."""
    import oracle as O

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    O.set_threads(os.cpu_count() or 1)
    vals = []
    for i in range(args.warmup + args.steps):
        if config == 3:
            v, th = config3_cpu(16, 1000, threads_all=True)
        else:
            v, th = config4_cpu(16)
        if i >= args.warmup:
            vals.append(v)
    v = sum(vals) / len(vals)
    metric, workload, tokens = (METRIC3, workload3(), T3) if config == 3 else (METRIC4, WORKLOAD4, T4)
    return {
        "impl": "reference", "metric": metric, "value": round(v, 3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(16 / v * 1e3, 3), "higher_is_better": True,
        "scaling": "weak" if config == 3 else "strong", "vs_baseline": None,
        "dtype": "fp4-e2m1 x fp8-e4m3 (act-quant) products, f32 accumulate",
        "data": "synthetic (seeded random-init weights, N(0,1) tokens)",
        "config": {"workload": workload, "experts": E, "topk": TOPK, "hidden": HID,
                   "inter": INTER, "tokens": tokens},
        "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": th, "kind": "port",
                         "sample": "16 tokens of the workload per step through the C++ "
                                   "restatement's batched MoE path"},
        "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_config5(args):
    import torch

    world, rank, local = dist_setup(args.gpus)
    import wohper_b200 as W
    from tests import helpers as H
    from wohper_b200.v4model import V4Decoder

    dev = torch.device("cuda", local)
    ctx = W.Context(local)
    B, NL = args.batch, args.layers
    t0 = time.time()
    layers, raws = [], []
    for li in range(NL):
        L, raw = H.v4_layer(W, ctx, li, E, seed=600 + li, max_tokens=B, router_mode=1,
                            device=dev)
        layers.append(L)
        raws.append(raw)
    g = torch.Generator(device=dev)
    g.manual_seed(700 + rank)
    kv = [[torch.randn(V4_POS + 1, 512, generator=g, device=dev) for _ in range(NL)]
          for _ in range(B)]
    comp = [[(torch.randn(n, 512, generator=g, device=dev) if n else None)
             for n in (H.v4_compressed_count(li, V4_POS) for li in range(NL))] for _ in range(B)]
    head = H.torch_hc_params(701, 4, HID, head=True, device=dev)
    final_norm = H.torch_bf16_norm(702, HID, device=dev)
    lm = (torch.randn(V4_VOCAB, HID, generator=g, device=dev) * 0.02).to(torch.bfloat16).view(
        torch.int16)
    build_s = time.time() - t0
    dec = V4Decoder(ctx, layers, head, final_norm, lm, kv, comp, batch=B, top_k=1)
    positions = [V4_POS] * B
    n_tok = args.warmup + args.steps
    xs = torch.randn(n_tok, B, 4 * HID, generator=g, device=dev)
    x = torch.empty(B, 4 * HID, device=dev)
    stream = torch.cuda.current_stream()
    x.copy_(xs[0])
    dec.step(x, positions)  # sizes the workspaces outside the capture
    torch.cuda.synchronize()
    ctx.sync()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            dec.step(x, positions)
    stream.wait_stream(cap)
    torch.cuda.synchronize()
    for i in range(args.warmup):
        x.copy_(xs[i])
        graph.replay()
    torch.cuda.synchronize()
    ctx.sync()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for k in range(args.steps):
            x.copy_(xs[args.warmup + k])
            ev[k][0].record(stream)
            graph.replay()
            ev[k][1].record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ctx.sync()
    ms_step = all_max(world, sum(a.elapsed_time(b) for a, b in ev)) / args.steps
    # graph output equals a direct step on the same input (bit for bit)
    x.copy_(xs[0])
    graph.replay()
    tg = dec.tokens.clone()
    xg = x.clone()
    x.copy_(xs[0])
    dec.step(x, positions)
    torch.cuda.synchronize()
    graph_ok = bool(torch.equal(tg, dec.tokens) and torch.equal(xg, x))
    # ---- end to end: the residual stream from pinned host memory, the token ids back
    xh = torch.randn(n_tok, B, 4 * HID, generator=torch.Generator().manual_seed(703)).pin_memory()
    th = torch.empty(args.steps, B, dtype=torch.int32).pin_memory()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for k in range(args.steps):
        x.copy_(xh[k], non_blocking=True)
        graph.replay()
        th[k].copy_(dec.tokens[:, 0], non_blocking=True)
    a1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = all_max(world, a0.elapsed_time(a1)) / args.steps
    # ---- the two halves of a layer, timed alone over all layers (graphs) ----
    def part_ms(fn):
        gp = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            fn()
            torch.cuda.synchronize()
            with torch.cuda.graph(gp, stream=cap):
                fn()
        torch.cuda.synchronize()
        gp.replay()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record(stream)
        for _ in range(3):
            gp.replay()
        b1.record(stream)
        torch.cuda.synchronize()
        return b0.elapsed_time(b1) / 3

    yb = torch.randn(B, HID, generator=g, device=dev)

    def attn_only():
        for li, L in enumerate(layers):
            W.v4_attention(ctx, L.attn, positions, yb, [kv[b][li] for b in range(B)],
                           dec.freqs[li], [comp[b][li] for b in range(B)], dec.attn_scratch)

    def moe_only():
        for L in layers:
            L.moe.forward(yb, dec.y2)

    def mhc_only():
        for L in layers:
            W.hc_pre(ctx, *L.hc_attn, x, 4, HID, out=(dec.y, dec.post, dec.comb))
            W.hc_post(ctx, dec.y, dec.resid, dec.post, dec.comb, 4, HID, out=dec.x2)
            W.hc_pre(ctx, *L.hc_ffn, x, 4, HID, out=(dec.y, dec.post, dec.comb))
            W.hc_post(ctx, dec.y, dec.resid, dec.post, dec.comb, 4, HID, out=dec.x2)

    # this library's kernels in one replay of the step graph (CUPTI through the
    # torch profiler, after the timed region)
    launches_per_step = None
    try:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            graph.replay()
            torch.cuda.synchronize()
        launches_per_step = sum(1 for ev in prof.events()
                                if ev.device_type.name == "CUDA" and ev.name.startswith(("wh::", "void wh::")))
    except Exception:  # the profiler is unavailable: the line says null
        launches_per_step = None
    parts = {"attention_all_layers": round(part_ms(attn_only), 4),
             "moe_all_layers": round(part_ms(moe_only), 4),
             "mhc_all_layers": round(part_ms(mhc_only), 4)}
    ctx.sync()
    res = None
    if rank == 0:
        # HBM bytes one step reads: attention weights, the experts each token
        # selects (a union at batch > 1: counted as min(batch * 6, 256) + shared),
        # the router, the mHC parameters, the KV rows the attention reads, the lm_head
        experts_read = min(B * TOPK, E) + 1
        kv_rows = sum(min(V4_POS + 1, 128) + H.v4_compressed_count(li, V4_POS)
                      for li in range(NL)) * B
        step_bytes = (NL * (V4_ATTN_BYTES + experts_read * EXPERT_BYTES + ROUTER_BYTES
                            + 2 * 24 * 4 * HID * 4)
                      + kv_rows * 512 * 4 + V4_VOCAB * HID * 2)
        peak, peak_kind = peaks()
        gbs = step_bytes / (ms_step * 1e-3) / 1e9
        res = {
            "metric": METRIC5, "value": round(B * world / (ms_step * 1e-3), 3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp8/fp4 weights x act-quantised fp8 activations, f32 accumulate, "
                     "bit-exact reference order",
            "data": "synthetic (seeded random-init weights, N(0,1) KV cache and residual stream)",
            "config": config5_dict(world, B, NL),
            "hbm_bytes_per_step": int(step_bytes),
            "roofline": {"kernel": "the whole decode step", "bound": "hbm",
                         "achieved": round(gbs, 1), "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": round(gbs / peak, 4),
                         "algorithmic_bytes": int(step_bytes), "traffic": None},
            "parts_ms": parts,
            "e2e": {"value": round(B * world / (e2e_ms * 1e-3), 3), "unit": "tokens/s",
                    "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": B * 4 * HID * 4,
                    "d2h_bytes_per_step": B * 4,
                    "path": "pinned host residual stream -> the captured step (C ABI kernels) "
                            "-> top-1 token ids to pinned host"},
            "graph_output_matches_direct_step": graph_ok,
            "build_s": round(build_s, 1),
            "gpu_launches": (launches_per_step * args.steps if launches_per_step else None),
            "gpu_launches_per_step": launches_per_step,
            "timing": "cuda graph of one step, replayed",
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            # the sampled CPU step of the reference arm (config5_cpu), once
            try:
                times, threads = config5_cpu(B)
                v = B / times[0]
                res["cpu_baseline"] = {
                    "value": round(v, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
                    "sample": f"one layer and the head for {B} sequence(s) through the oracle's "
                              f"composition, the lm_head over 16384 rows; the step estimated as "
                              f"{V4_LAYERS} x the layer + the head scaled to {V4_VOCAB} rows"}
            except Exception as e:  # the line stands without it
                res["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    del graph
    for L in layers:
        L.moe.close()
    ctx.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return res


# ---------------------------------------------------------------------------
# config 3: batched (prefill) MoE FFN on the tensor cores
# ---------------------------------------------------------------------------
T3 = 2048
METRIC3 = "prefill tokens/s (batched FP4 MoE FFN, config 3)"
WORKLOAD3 = ("config 3: 2048 tokens through the FP4 MoE FFN, 256 experts + shared, "
             "4096->2048->4096, Zipf(1.1)-skewed top-6 routing, grouped block-scaled GEMMs")


def workload3() -> str:
    """WORKLOAD3, or with --tokens the same workload at another token count (the
    compute-bound point of the grouped GEMMs is 16384 tokens)."""
    return WORKLOAD3 if T3 == 2048 else WORKLOAD3.replace("2048 tokens", f"{T3} tokens", 1)
W13_BYTES = 2 * (PACKED_W13 + SCALES_W13)   # w1 + w3 of one expert
W2_BYTES = PACKED_W2 + SCALES_W2


def config3_inputs(H, seed):
    gate, x = H.zipf_routing(seed + 9, H.router_gate(seed + 6, E, HID),
                             H.activations(seed + 7, T3, HID))
    return gate, x


def config3_cpu(T_sample: int, seed: int, threads_all: bool):
    """Oracle (the reference's CPU kernels restated) on T_sample tokens of the
    config-3 workload: exact router per token, then the expert-major batched
    path.  Returns (tokens/s, threads)."""
    import oracle as O
    from tests import helpers as H

    if threads_all:
        O.set_threads(os.cpu_count() or 1)
    gate, x = config3_inputs(H, seed)
    x = x[:T_sample]
    model = HostModel(seed)
    model.gate = gate
    t0 = time.perf_counter()
    ids = np.zeros((T_sample, TOPK), np.int32)
    ws = np.zeros((T_sample, TOPK), np.float32)
    for t in range(T_sample):
        _, ids[t], ws[t], _ = O.router(gate, x[t], TOPK, mode=0)
    t_route = time.perf_counter() - t0
    arr = (O.Fp4Expert * (E + 1))()
    for e in set(ids.reshape(-1).tolist()) | {E}:
        arr[e] = model.expert(int(e))  # generated untimed
    t1 = time.perf_counter()
    st, _ = O.moe_batched(arr, E, ids, ws, arr[E], x)
    dt = t_route + time.perf_counter() - t1
    assert st == O.OK
    return T_sample / dt, O.threads()


def run_config3(args):
    import torch

    world, rank, local = dist_setup(args.gpus)
    import wohper_b200 as W
    from tests import helpers as H

    dev = torch.device("cuda", local)
    ctx = W.Context(local)
    stack = H.torch_fp4_experts(1000 + rank, E + 1, HID, INTER, device=dev)
    gate_np, x_np = config3_inputs(H, 1000 + rank)

    def wexp(e):
        w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
        return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, INTER, HID, HID // 32),
                                     W.Fp4Matvec(w3, s3, INTER, HID, HID // 32),
                                     W.Fp4Matvec(w2, s2, HID, INTER, INTER // 32))

    layer = W.MoeLayer(ctx, [wexp(e) for e in range(E)], wexp(E),
                       torch.from_numpy(gate_np.view(np.int16)).to(dev), topk=TOPK,
                       max_tokens=T3)
    x = torch.from_numpy(x_np).to(dev)
    y = torch.empty_like(x)
    ids = torch.zeros(T3, TOPK, dtype=torch.int32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        flush.zero_()
        layer.forward(x, y, ids=ids)
    ctx.sync()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for k in range(args.steps):
            flush.zero_()
            ev[k][0].record(stream)
            layer.forward(x, y, ids=ids)
            ev[k][1].record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ctx.sync()
    ms_step = all_max(world, sum(a.elapsed_time(b) for a, b in ev)) / args.steps
    counts = np.bincount(ids.cpu().numpy().reshape(-1), minlength=E)
    used = int((counts > 0).sum()) + 1  # + shared
    R = T3 * TOPK + T3
    # per-kernel times (events between kernels)
    ctx.set_profiling(True)
    phases = []
    for _ in range(3):
        flush.zero_()
        layer.forward(x, y, ids=ids)
        phases.append(ctx.phase_times())
    ctx.set_profiling(False)
    ctx.sync()
    ph = np.array(phases).mean(0)  # router, route+dispatch, up, down, combine
    up_ms, down_ms = float(ph[2]), float(ph[3])
    up_bytes = used * W13_BYTES + R * HID + R * INTER + R * (HID + INTER) // 32
    up_flops = 2.0 * R * 2 * INTER * HID
    peak, peak_kind = peaks()
    up_gbs = up_bytes / (up_ms * 1e-3) / 1e9
    step_flops = 2.0 * R * 3 * INTER * HID
    # end to end: pinned host tokens -> H2D -> wh_moe_ffn -> D2H
    xh = torch.from_numpy(x_np).pin_memory()
    yh = torch.empty(T3, HID).pin_memory()
    xd = torch.empty_like(x)
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for k in range(args.steps):
        flush.zero_()
        ev2[k][0].record(stream)
        xd.copy_(xh, non_blocking=True)
        layer.forward(xd, y)
        yh.copy_(y, non_blocking=True)
        ev2[k][1].record(stream)
    torch.cuda.synchronize()
    e2e_ms = all_max(world, sum(a.elapsed_time(b) for a, b in ev2)) / args.steps
    res = None
    if rank == 0:
        res = {
            "metric": METRIC3, "value": round(world * T3 / (ms_step * 1e-3), 1),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp4-e2m1 (as e4m3) x fp8-e4m3, ue8m0 block scales, f32 accumulate",
            "data": "synthetic (seeded random-init weights, N(0,1) tokens, Zipf prior on routing)",
            "config": {"workload": workload3(), "experts": E, "topk": TOPK, "hidden": HID,
                       "inter": INTER, "tokens": T3, "experts_used": used,
                       "max_expert_rows": int(counts.max()), "rows": R,
                       "l2": "flushed between steps (256 MiB memset outside the timed events)",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "phases_ms": {"router": round(float(ph[0]), 4), "route_dispatch": round(float(ph[1]), 4),
                          "up": round(up_ms, 4), "down": round(down_ms, 4),
                          "combine": round(float(ph[4]), 4)},
            "roofline": {"kernel": "grouped_gemm_kernel<up> (w1+w3 of the used experts, SwiGLU, act quant)",
                         "bound": "hbm", "achieved": round(up_gbs, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(up_gbs / peak, 4),
                         "algorithmic_bytes": int(up_bytes),
                         "traffic": int(up_bytes * GROUPED_UP_TRAFFIC_RATIO),
                         "traffic_note": "scaled from the ncu capture of the grouped16 case",
                         "tensor_tflops": round(up_flops / (up_ms * 1e-3) / 1e12, 1),
                         # the MMA is kind::mxf8f6f4 on E4M3 operands (the reference's FP4
                         # code 1 has no E2M1 encoding), so its dense peak is the FP8 rate,
                         # twice the measured bf16 GEMM; the nominal FP4 rate is twice that
                         "tensor_peak_tflops": round(2 * bf16_peak(), 1),
                         "tensor_peak_kind": "2 x measured bf16 dense (the fp8 kind::f8f6f4 rate)",
                         "tensor_frac": round(up_flops / (up_ms * 1e-3) / 1e12 / (2 * bf16_peak()), 4),
                         "tensor_frac_of_nominal_fp4": round(
                             up_flops / (up_ms * 1e-3) / 1e12 / 9000.0, 4)},
            "step_tflops": round(step_flops / (ms_step * 1e-3) / 1e12, 1),
            "e2e": {"value": round(world * T3 / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": T3 * HID * 4,
                    "d2h_bytes_per_step": T3 * HID * 4,
                    "path": "pinned host x -> H2D -> wh_moe_ffn (C ABI) -> D2H y"},
            "gpu_launches": 8 * args.steps,
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline:
            v, th = config3_cpu(16, 1000, threads_all=False)
            res["cpu_baseline"] = {"value": round(v, 3), "unit": "tokens/s", "cores": th,
                                   "kind": "port",
                                   "sample": "16 tokens of the same workload: exact router + "
                                             "expert-major batched path of the C++ restatement"}
    layer.close()
    ctx.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return res


# ---------------------------------------------------------------------------
# config 4: expert-parallel MoE layer over the ranks (NCCL all-to-all)
# ---------------------------------------------------------------------------
T4 = 8192
METRIC4 = "expert-parallel MoE layer tokens/s (config 4)"
WORKLOAD4 = ("config 4: 8192 tokens per step through the FP4 MoE FFN, 256 experts sharded "
             "contiguously over the ranks + replicated shared expert, seeded uniform-random "
             "top-6 routes; rows and results cross NVLink as peer-memory stores from the "
             "dispatch kernel and the down GEMM's epilogue (--ep-transport nccl: NCCL "
             "all-to-all)")


def config4_routes(seed: int):
    g = np.random.default_rng(seed)
    ids = np.array([g.choice(E, TOPK, replace=False) for _ in range(T4)], np.int32)
    w = g.uniform(0.1, 1.0, (T4, TOPK)).astype(np.float32)
    return ids, w


def config4_cpu(T_sample: int):
    """The reference's batched MoE (oracle restatement) on T_sample tokens of
    the config-4 workload (uniform routes): tokens/s on this host."""
    import oracle as O
    from tests import helpers as H

    ids, w = config4_routes(4000)
    ids, w = ids[:T_sample], w[:T_sample]
    x = H.activations(4001, T_sample, HID)
    model = HostModel(4002)
    arr = (O.Fp4Expert * (E + 1))()
    for e in set(ids.reshape(-1).tolist()) | {E}:
        arr[e] = model.expert(int(e))
    t0 = time.perf_counter()
    st, _ = O.moe_batched(arr, E, ids, w, arr[E], x)
    dt = time.perf_counter() - t0
    assert st == O.OK
    return T_sample / dt, O.threads()


def ep_measure(args, world: int, rank: int, local: int, transport: str = "p2p"):
    """Config 4 on this process group: T4 tokens per step split over the ranks,
    the 256 experts sharded contiguously.  Returns (rank 0) a dict with the
    step time (max over ranks), the per-phase medians over the timed steps
    and the per-rank roofline; None on the other ranks."""
    import torch
    import torch.distributed as dist

    import wohper_b200 as W
    from tests import helpers as H
    from wohper_b200.ep import DeviceOps, EpMoeLayer

    dev = torch.device("cuda", local)
    ctx = W.Context(local)
    El = E // world
    stack = H.torch_fp4_experts(4100 + rank, El + 1, HID, INTER, device=dev)

    def wexp(e):
        w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
        return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, INTER, HID, HID // 32),
                                     W.Fp4Matvec(w3, s3, INTER, HID, HID // 32),
                                     W.Fp4Matvec(w2, s2, HID, INTER, INTER // 32))

    Tl = T4 // world
    layer = EpMoeLayer(ctx, [wexp(e) for e in range(El)], wexp(El), world,
                       transport=transport, max_tokens=Tl)
    ids_all, w_all = config4_routes(4000)
    lo = rank * Tl
    x = torch.from_numpy(H.activations(4200 + rank, Tl, HID)).to(dev)
    ids = torch.from_numpy(ids_all[lo:lo + Tl]).to(dev)
    wts = torch.from_numpy(w_all[lo:lo + Tl]).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        flush.zero_()
        layer.forward(x, ids, wts)
    torch.cuda.synchronize()
    ctx.sync()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for k in range(args.steps):
            flush.zero_()
            ev[k][0].record(stream)
            layer.forward(x, ids, wts)
            ev[k][1].record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ctx.sync()
    ms_step = all_max(world, sum(a.elapsed_time(b) for a, b in ev)) / args.steps
    # phase split: events between the calls on every timed-length pass, the
    # median of each phase over the steps, then the max over ranks
    flat = ids.reshape(-1).to(torch.int64) // El
    per_dest = torch.bincount(flat, minlength=world).tolist()
    if transport == "p2p":
        names = ["dispatch_and_row_stores", "expert_ffn_and_result_stores", "wait_and_combine"]
        samples = []
        for k in range(args.steps):
            pe = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            flush.zero_()
            layer.forward_p2p(x, ids, wts, marks=lambda i: pe[i].record(stream))
            torch.cuda.synchronize()
            samples.append([pe[i].elapsed_time(pe[i + 1]) for i in range(3)])
        ctx.sync()
        med = np.median(np.array(samples), axis=0)
        ph = [all_max(world, float(v)) for v in med]
    else:
        names = ["dispatch", "all_to_all_rows", "expert_ffn", "all_to_all_results", "combine"]
        ops = DeviceOps(layer)
        samples = []
        for k in range(args.steps):
            pe = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            flush.zero_()
            pe[0].record(stream)
            send, cnt, pos = ops.dispatch(x, ids)
            rc = torch.empty_like(cnt)
            dist.all_to_all_single(rc, cnt)
            both = ops.to_list(ops.cat([cnt.view(world, El).sum(1), rc.view(world, El).sum(1)]))
            pdst, psrc = both[:world], both[world:]
            R = sum(psrc)
            recv = ops.empty_rows(R)
            pe[1].record(stream)
            dist.all_to_all_single(recv, send, output_split_sizes=psrc, input_split_sizes=pdst)
            pe[2].record(stream)
            y_rows = ops.expert_ffn(recv, rc, R, x)
            pe[3].record(stream)
            y_back = ops.empty_results(send.shape[0])
            dist.all_to_all_single(y_back, y_rows[:R], output_split_sizes=pdst,
                                   input_split_sizes=psrc)
            pe[4].record(stream)
            ops.combine(ids, wts, pos, y_back, y_rows[R:])
            pe[5].record(stream)
            torch.cuda.synchronize()
            samples.append([pe[i].elapsed_time(pe[i + 1]) for i in range(5)])
        ctx.sync()
        med = np.median(np.array(samples), axis=0)
        ph = [all_max(world, float(v)) for v in med]
    phases = {n: round(v, 4) for n, v in zip(names, ph)}
    rb = layer.row_bytes
    sent_remote = sum(n for d, n in enumerate(per_dest) if d != rank)
    # per-rank roofline: the rank's local experts' weights once, its rows in
    # and results out; FLOPs of the routed rows it receives (T4*topk/world on
    # average) and of the shared expert over its own tokens
    flops_rank = (T4 * TOPK / world + Tl) * 2 * 3 * HID * INTER
    bytes_rank = (El + 1) * EXPERT_BYTES
    link_bytes = (T4 * TOPK / world) * (world - 1) / world * (rb + 4 * HID)
    hbm, _ = peaks()
    tflops_peak = 2 * bf16_peak()
    t_tensor = flops_rank / (tflops_peak * 1e12)
    t_hbm = bytes_rank / (hbm * 1e9)
    t_link = link_bytes / (770e9) if world > 1 else 0.0
    bound = max(("tensor", t_tensor), ("hbm", t_hbm), ("nvlink", t_link), key=lambda p: p[1])
    res = None
    if rank == 0:
        res = {
            "tokens_per_s": round(T4 / (ms_step * 1e-3), 1), "ms_per_step": round(ms_step, 5),
            "n_gpus": world, "tokens": T4, "tokens_per_rank": Tl, "experts_per_rank": El,
            "transport": transport, "dispatch_row_bytes": int(rb),
            "phases_ms_median_over_steps_max_over_ranks": phases,
            "rank0_remote_rows_sent": sent_remote,
            "roofline_per_rank": {
                "bound": bound[0], "target_ms": round(bound[1] * 1e3, 4),
                "frac": round(bound[1] * 1e3 / ms_step, 4),
                "tensor_tflops_achieved": round(flops_rank / (ms_step * 1e-3) / 1e12, 1),
                "tensor_peak_tflops": tflops_peak,
                "tensor_peak_kind": "2 x measured bf16 dense (B200's fp8 kind::f8f6f4 rate is "
                                    "twice its bf16 rate)",
                "flops_per_rank": flops_rank, "hbm_bytes_per_rank": bytes_rank,
                "nvlink_bytes_per_rank": int(link_bytes), "nvlink_gbs_per_direction": 770.0},
            "gpu_launches_per_step": 11,
            "clocks": clk.summary(),
        }
    layer.close()
    ctx.close()
    return res


def bf16_peak() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"])
    return 1590.0


def run_config4(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_setup(args.gpus)
    if world == 1 and not dist.is_initialized() and args.ep_transport == "nccl":
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29631")
        dist.init_process_group("nccl", rank=0, world_size=1,
                                device_id=torch.device("cuda", local))
    m = ep_measure(args, world, rank, local, args.ep_transport)
    res = None
    if rank == 0:
        res = {
            "metric": METRIC4, "value": m["tokens_per_s"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": m["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": "fp4-e2m1 (as e4m3) x fp8-e4m3, ue8m0 block scales, f32 accumulate",
            "data": "synthetic (seeded random-init weights, N(0,1) tokens, uniform routes)",
            "config": {"workload": WORKLOAD4, "experts": E, "topk": TOPK, "hidden": HID,
                       "inter": INTER, "tokens": T4, "tokens_per_rank": m["tokens_per_rank"],
                       "experts_per_rank": m["experts_per_rank"],
                       "dispatch_row_bytes": m["dispatch_row_bytes"],
                       "l2": "flushed between steps (256 MiB memset outside the timed events)",
                       "parallelism": f"expert parallel x{world}"},
            "transport": args.ep_transport,
            "phases_ms_median_over_steps_max_over_ranks":
                m["phases_ms_median_over_steps_max_over_ranks"],
            "rank0_remote_rows_sent": m["rank0_remote_rows_sent"],
            "roofline_per_rank": m["roofline_per_rank"],
            # count, scan, pack | totals, units, permute, pack_local, map_tail, up,
            # down | combine (the NCCL transport adds the collectives' kernels)
            "gpu_launches": 11 * args.steps,
            "clocks": m["clocks"],
        }
        if not args.no_cpu_baseline:
            v, th = config4_cpu(16)
            res["cpu_baseline"] = {"value": round(v, 3), "unit": "tokens/s", "cores": th,
                                   "kind": "port",
                                   "sample": "16 tokens of the workload through the C++ "
                                             "restatement's batched path, one host"}
    if dist.is_initialized():
        dist.destroy_process_group()
    return res


# ---------------------------------------------------------------------------
# expert loading: a layer's FP4 expert blocks from the experts pack into HBM
# ---------------------------------------------------------------------------
METRIC_LOAD = "expert load GB/s (FP4 expert blocks, ZCBLK01 experts pack -> HBM)"
WORKLOAD_LOAD = ("expert loading: the 256 FP4 experts of one DeepSeek-V4-Flash MoE layer "
                 "(4096 -> 2048 -> 4096, E2M1 + UE8M0-32, 13.4 MB of tensors each) as ZCBLK01 "
                 "blocks in an experts pack on local disk, read by the expert loader into one "
                 "HBM arena per step (reader threads + pinned staging + copy engines)")
TENSOR_NAMES = ("w1", "s1", "w3", "s3", "w2", "s2")


class _LazyExperts:
    """expert id -> the six ZCBLK01 tensors of that expert, generated on use
    (seeded random bytes); records int32-sum checksums of every tensor."""

    def __init__(self, ZB, ids, seed):
        self.ZB, self.ids, self.seed = ZB, list(ids), seed
        self.sums = {}

    def __len__(self):
        return len(self.ids)

    def __iter__(self):
        return iter(self.ids)

    def __getitem__(self, e):
        g = np.random.default_rng(self.seed + e)

        def packed(r, c):
            return g.integers(0, 256, size=(r, c // 2), dtype=np.uint8)

        def scales(r, c):
            return (127 + g.integers(-6, 1, size=(r, c // 32))).astype(np.uint8)

        arrs = (packed(INTER, HID), scales(INTER, HID), packed(INTER, HID), scales(INTER, HID),
                packed(HID, INTER), scales(HID, INTER))
        self.sums[e] = [int(a.view(np.int32).sum(dtype=np.int64)) for a in arrs]
        return self.ZB.deepseek_fp4_expert_tensors(f"layers.0.ffn.experts.{e}", *arrs)


def load_model_dir(rank: int, world: int):
    base = os.environ.get("WH_BENCH_DIR") or tempfile.gettempdir()
    return Path(base) / f"wh_expert_load_{os.environ.get('MASTER_PORT', 'local')}"


def write_load_model(ZB, d: Path, seed: int):
    d.mkdir(parents=True, exist_ok=True)
    lazy = _LazyExperts(ZB, range(E), seed)
    gate = ZB.BlockTensor("layers.0.ffn.gate.weight", 11, 2404, 9, (E, HID),
                          bytes(E * HID * 2))
    ZB.write_model(d / "dense_core.bin", [ZB.LayerSpec(0, [gate], lazy)], hidden_size=HID,
                   pack=True)
    (d / "sums.json").write_text(json.dumps({str(k): v for k, v in lazy.sums.items()}))


def load_cpu_sample(model: Path, ids, threads: int):
    """The reference's host path for the same experts: read each block's
    payload from the pack (pread, like its direct-I/O pread fallback) and parse
    it with the restated parser and suffix bridge; bytes/s of expert tensors."""
    import concurrent.futures as cf

    from oracle import zcblk as Z

    m = Z.load_manifest(model)

    def one(e):
        p, off, _db, pb = Z.expert_source(m, model, 0, e)
        fd = os.open(p, os.O_RDONLY)
        try:
            b = os.pread(fd, pb, off)
        finally:
            os.close(fd)
        w1, w3, w2 = Z.fp4_expert_from_block(b)
        return sum(v.weight_len + v.scale_len for v in (w1, w3, w2))

    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(threads) as ex:
        nbytes = sum(ex.map(one, ids))
    dt = time.perf_counter() - t0
    return nbytes / dt / 1e9, nbytes, dt


def h2d_peak_gbs(dev, nbytes: int = 1 << 30, reps: int = 5) -> float:
    """Pinned host -> device copy bandwidth of one large transfer (best of reps)."""
    import torch

    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, nbytes / (a.elapsed_time(b) * 1e-3) / 1e9)
    del src, dst
    return best


def run_expert_load(args):
    import torch

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    d = load_model_dir(rank, world)
    model = d / "dense_core.bin"
    if args.impl == "reference":
        res = None
        if rank == 0:
            if not model.exists():
                from wohper_b200 import zcblk as ZB

                write_load_model(ZB, d, 5000)
            threads = os.cpu_count() or 1
            vals = []
            for k in range(args.warmup + args.steps):
                v, nbytes, _dt = load_cpu_sample(model, range(E), threads)
                if k >= args.warmup:
                    vals.append(v)
            v = statistics.median(vals)
            res = {"metric": METRIC_LOAD, "value": round(v, 3), "unit": "GB/s", "n_gpus": world,
                   "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                   "impl": "reference", "scaling": "strong", "vs_baseline": None, "dtype": "u8",
                   "data": "synthetic (seeded random FP4 expert blocks)",
                   "config": {"workload": WORKLOAD_LOAD, "experts": E},
                   "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads,
                                    "kind": "port",
                                    "sample": "all 256 expert blocks per step: pread of each "
                                              "payload + the restated block parser"},
                   "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}}
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return res

    import wohper_b200 as W
    from wohper_b200 import zcblk as ZB

    ctx = W.Context(local)
    if rank == 0 and not model.exists():
        t0 = time.perf_counter()
        write_load_model(ZB, d, 5000)
        write_s = time.perf_counter() - t0
    else:
        write_s = None
    barrier(world)
    sums = json.loads((d / "sums.json").read_text())
    per = E // world
    ids = list(range(rank * per, (rank + 1) * per))
    man = ZB.ModelManifest(model)
    loader = ZB.ExpertLoader(ctx, man, threads=args.load_threads, direct_io=args.direct_io)
    arena = torch.empty(loader.arena_bytes(0, ids), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        loader.load(0, ids, arena)
        torch.cuda.synchronize()
    # size-independent parity: per-tensor int32 sums of the loaded bytes equal the
    # sums of the generated source arrays, for every expert
    _, experts = loader.load(0, ids, arena)
    torch.cuda.synchronize()
    bad = 0
    for e, ex in zip(ids, experts):
        got = [int(t.view(torch.int32).sum(dtype=torch.int64).item())
               for m in (ex.w1, ex.w3, ex.w2) for t in (m.packed_weight, m.ue8m0_scales)]
        bad += got != sums[str(e)]
    tensor_bytes = per * EXPERT_BYTES
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for k in range(args.steps):
            ev[k][0].record(stream)
            loader.load(0, ids, arena)
            ev[k][1].record(stream)
            torch.cuda.synchronize()
    barrier(world)
    ms_step = all_max(world, sum(a.elapsed_time(b) for a, b in ev)) / args.steps
    # end to end through the public API: open the manifest, load, synchronise
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for k in range(args.steps):
        ev2[k][0].record(stream)
        m2 = ZB.ModelManifest(model)
        loader.load(0, ids, arena)
        ev2[k][1].record(stream)
        torch.cuda.synchronize()
        m2.close()
    e2e_ms = all_max(world, sum(a.elapsed_time(b) for a, b in ev2)) / args.steps
    peak = h2d_peak_gbs(dev)
    achieved = tensor_bytes / (ms_step * 1e-3) / 1e9
    res = None
    if rank == 0:
        res = {
            "metric": METRIC_LOAD, "value": round(world * achieved, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (seeded random FP4 expert blocks written in the reference's "
                    "experts-pack format)",
            "config": {"workload": WORKLOAD_LOAD, "experts": E, "experts_per_rank": per,
                       "tensor_bytes_per_expert": EXPERT_BYTES,
                       "reader_threads": args.load_threads, "direct_io": bool(args.direct_io),
                       "l2": "inputs larger than L2 (3.4 GB per step from host memory)",
                       "file": "page cache warm (written just before)" if not args.direct_io
                               else "O_DIRECT reads",
                       "parallelism": f"expert shards x{world}" if world > 1 else "single GPU"},
            "parity": {"experts_checked": per, "mismatched": bad,
                       "check": "per-tensor int32 sums of the loaded HBM bytes vs the source"},
            "roofline": {"kernel": "copy engines (pinned staging -> HBM arena)", "bound": "h2d",
                         "achieved": round(achieved, 2), "peak": round(peak, 2),
                         "peak_kind": "measured live: one 1 GiB pinned cudaMemcpyAsync",
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "algorithmic_bytes": tensor_bytes, "traffic": None},
            "e2e": {"value": round(world * tensor_bytes / (e2e_ms * 1e-3) / 1e9, 2),
                    "unit": "GB/s", "ms_per_step": round(e2e_ms, 3),
                    "h2d_bytes_per_step": tensor_bytes, "d2h_bytes_per_step": 0,
                    "path": "wh_model_open + wh_expert_loader_load (C ABI) from the pack file"},
            "gpu_launches": 0,
            "copies_per_step": 6 * per,
            "clocks": clk.summary(),
        }
        if write_s is not None:
            res["config"]["pack_write_s"] = round(write_s, 2)
        if not args.no_cpu_baseline:
            v, nbytes, dt = load_cpu_sample(model, ids[:64], 1)
            res["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": 1,
                                   "kind": "port",
                                   "sample": f"64 experts ({nbytes / 1e9:.2f} GB) read with "
                                             "pread and parsed by the restated parser, one "
                                             "thread"}
    loader.close()
    man.close()
    ctx.close()
    barrier(world)
    if rank == 0 and not os.environ.get("WH_BENCH_DIR"):
        shutil.rmtree(d, ignore_errors=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return res


# ---------------------------------------------------------------------------
# BF16 lm_head top-k over the DeepSeek vocabulary
# ---------------------------------------------------------------------------
VOCAB = 129280
METRIC_LM = "lm_head top-k tokens/s (BF16 129280 x 4096 logits + top-k)"
WORKLOAD_LM = ("lm_head top-k: every logit of the BF16 lm_head of DeepSeek-V3/V4 shape "
               "(129280 x 4096, 1.06 GB) in the reference's dot_bf16_row order, then the "
               "top-k push_topk_candidate keeps, sorted; one hidden vector per step")
# DRAM bytes / algorithmic bytes of lm_logits_kernel from the ncu capture of the lmhead case
# (32768 rows: 268,467,200 read + 3,915,264 written / 268,582,912; bench.py --ncu-case lmhead),
# scaled to the full launch by rows
LM_TRAFFIC_RATIO = 272_382_464 / 268_582_912


def lm_head_cpu(w_np, xs, k, steps):
    """The oracle's restatement on all host threads: seconds per step."""
    import oracle as O

    O.lm_head_topk(w_np[:4096], xs[0], k)  # warm the library
    t0 = time.perf_counter()
    for i in range(steps):
        O.lm_head_topk(w_np, xs[i % len(xs)], k)
    return (time.perf_counter() - t0) / steps


def run_lm_head(args):
    import torch

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    k = max(args.lm_top_k, 1)
    g = torch.Generator(device=dev)
    g.manual_seed(700 + rank)
    w = (torch.randn(VOCAB, HID, device=dev, generator=g) * 0.02).to(torch.bfloat16).view(torch.int16)
    xs = [torch.randn(HID, device=dev, generator=g) for _ in range(8)]
    if args.impl == "reference":
        res = None
        if rank == 0:
            w_np = w.cpu().numpy().view(np.uint16)
            xs_np = [x.cpu().numpy() for x in xs]
            sec = lm_head_cpu(w_np, xs_np, k, max(args.steps, 1))
            v = 1.0 / sec
            res = {"metric": METRIC_LM, "value": round(v, 2), "unit": "tokens/s",
                   "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                   "higher_is_better": True, "impl": "reference", "scaling": "weak",
                   "vs_baseline": None, "dtype": "bf16 x f32, f32 accumulate",
                   "data": "synthetic (N(0, 0.02) bf16 weights, N(0, 1) hidden vectors)",
                   "config": {"workload": WORKLOAD_LM, "rows": VOCAB, "cols": HID, "top_k": k},
                   "cpu_baseline": {"value": round(v, 2), "unit": "tokens/s",
                                    "cores": os.cpu_count(), "kind": "port",
                                    "sample": f"{max(args.steps, 1)} full steps"},
                   "e2e": {"value": round(v, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}}
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return res

    import wohper_b200 as W

    ctx = W.Context(local)
    scratch = torch.empty(W.lib().wh_lm_head_scratch_bytes(VOCAB, k), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        W.lm_head_topk_score(ctx, w, xs[i % 8], k, scratch=scratch)
    ctx.sync()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            ev[i][0].record(stream)
            W.lm_head_topk_score(ctx, w, xs[i % 8], k, scratch=scratch)
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ctx.sync()
    ms_step = all_max(world, sum(a.elapsed_time(b) for a, b in ev)) / args.steps
    ctx.set_profiling(True)
    phases = []
    for i in range(5):
        W.lm_head_topk_score(ctx, w, xs[i % 8], k, scratch=scratch)
        phases.append(ctx.phase_times())
    ctx.set_profiling(False)
    ctx.sync()
    ph = np.median(np.array(phases), axis=0)  # logits, collect, select
    # end to end: x from pinned host memory, tokens + logits back to it
    xh = [x.cpu().pin_memory() for x in xs]
    xd = torch.empty(HID, device=dev)
    th = torch.empty(k, dtype=torch.int32).pin_memory()
    vh = torch.empty(k).pin_memory()
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for i in range(args.steps):
        ev2[i][0].record(stream)
        xd.copy_(xh[i % 8], non_blocking=True)
        t, v = W.lm_head_topk_score(ctx, w, xd, k, scratch=scratch)
        th[:t.numel()].copy_(t, non_blocking=True)
        vh[:v.numel()].copy_(v, non_blocking=True)
        ev2[i][1].record(stream)
    torch.cuda.synchronize()
    e2e_ms = all_max(world, sum(a.elapsed_time(b) for a, b in ev2)) / args.steps
    peak, peak_kind = peaks()
    alg = VOCAB * HID * 2 + HID * 4 + VOCAB * 4
    logits_ms = float(ph[0])
    achieved = alg / (logits_ms * 1e-3) / 1e9
    res = None
    if rank == 0:
        res = {
            "metric": METRIC_LM, "value": round(world * 1e3 / ms_step, 2), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 x f32, f32 accumulate (reference dot order)",
            "data": "synthetic (N(0, 0.02) bf16 weights, N(0, 1) hidden vectors)",
            "config": {"workload": WORKLOAD_LM, "rows": VOCAB, "cols": HID, "top_k": k,
                       "l2": "inputs larger than L2 (1.06 GB of weights per step)",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "phases_ms": {"logits": round(logits_ms, 4), "collect": round(float(ph[1]), 4),
                          "select": round(float(ph[2]), 4)},
            "roofline": {"kernel": "lm_logits_kernel", "bound": "hbm",
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "algorithmic_bytes": alg,
                         "traffic": int(alg * LM_TRAFFIC_RATIO) if LM_TRAFFIC_RATIO else None},
            "e2e": {"value": round(world * 1e3 / e2e_ms, 2), "unit": "tokens/s",
                    "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": HID * 4,
                    "d2h_bytes_per_step": k * 8,
                    "path": "pinned host x -> H2D -> wh_lm_head_topk (C ABI) -> D2H tokens + logits"},
            "gpu_launches": 3 * args.steps,
            "clocks": clocks,
        }
        if not args.no_cpu_baseline:
            w_np = w.cpu().numpy().view(np.uint16)
            sec = lm_head_cpu(w_np, [x.cpu().numpy() for x in xs], k, 3)
            res["cpu_baseline"] = {"value": round(1.0 / sec, 2), "unit": "tokens/s",
                                   "cores": os.cpu_count(), "kind": "port",
                                   "sample": "3 full steps (all 129280 rows, top-k) of the "
                                             "oracle's restatement on all host threads"}
    ctx.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return res


# DRAM bytes of one call (the three kernels) from the ncu capture of --ncu-case
# mla: 2,502,656 + 407,040 + 2,702,592 read, 0 written.  ncu empties the caches
# before each kernel, so the output kernel's key rows count as DRAM there; in
# the timed pipeline they are L2 hits.
MLA_TRAFFIC = 5_612_288
# cycles per step of a dependent FP32 addition chain (acc = acc + x * y with the
# products independent), measured on this pool's B200 with one thread timing a
# 2^20-step chain by clock64: 4.44 (4.56 for bare additions)
FADD_CHAIN_CYCLES = 4.44
METRIC_MLA = "MLA attention-core calls/s (one decode token, one DeepSeek-V4 layer, 64 heads)"
MLA_HEADS, MLA_HD, MLA_NOPE, MLA_POS, MLA_COMP = 64, 512, 448, 4095, 1024
WORKLOAD_MLA = ("MLA attention core of DeepSeek-V4-Flash (64 heads x 512 = 448 nope + 64 rope), "
                "ratio-4 layer at token 4095: 128-row sliding window + 1024 compressed rows, "
                "attention sink, YaRN inverse RoPE")


def mla_inputs(dev, seed):
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    q = torch.randn(MLA_HEADS, MLA_HD, device=dev, generator=g) * 0.05
    keys = torch.randn(MLA_POS + 1, MLA_HD, device=dev, generator=g)
    comp = torch.randn(MLA_COMP, MLA_HD, device=dev, generator=g)
    sink = torch.randn(MLA_HEADS, device=dev, generator=g)
    return q, keys, comp, sink


def mla_cpu(q, keys, comp, sink, fr, steps):
    """The oracle's scalar restatement on one host thread: seconds per call."""
    import oracle as O

    t0 = time.perf_counter()
    for _ in range(steps):
        O.mla_attention(q, keys, MLA_POS, 128, comp, sink, fr, MLA_NOPE)
    return (time.perf_counter() - t0) / steps


def run_mla(args):
    import torch

    import wohper_b200 as W

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    q, keys, comp, sink = mla_inputs(dev, 800 + rank)
    theta, yarn = W.deepseek_rope_for_layer(2)
    fr = W.rope_inv_freqs(MLA_HD - MLA_NOPE, theta, yarn)
    cfg = {"workload": WORKLOAD_MLA, "heads": MLA_HEADS, "head_dim": MLA_HD,
           "token_pos": MLA_POS, "window": 128, "compressed_rows": MLA_COMP,
           "l2": "flushed between calls (256 MiB memset outside the timed events)",
           "parallelism": f"replicas x{world}" if world > 1 else "single GPU"}
    if args.impl == "reference":
        res = None
        if rank == 0:
            host = [t.cpu().numpy() for t in (q, keys, comp, sink)]
            sec = mla_cpu(*host, fr, max(args.steps, 1))
            v = 1.0 / sec
            res = {"metric": METRIC_MLA, "value": round(v, 2), "unit": "calls/s",
                   "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                   "higher_is_better": True, "impl": "reference", "scaling": "weak",
                   "vs_baseline": None, "dtype": "f32", "data": "synthetic (N(0, 1) cache rows)",
                   "config": cfg,
                   "cpu_baseline": {"value": round(v, 2), "unit": "calls/s", "cores": 1,
                                    "kind": "port", "sample": f"{max(args.steps, 1)} full calls"},
                   "e2e": {"value": round(v, 2), "unit": "calls/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}}
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return res

    ctx = W.Context(local)
    out = torch.empty(MLA_HEADS, MLA_HD, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def call(qd):
        W.mla_attention(ctx, qd, keys, MLA_POS, fr, MLA_NOPE, compressed=comp, sink=sink,
                        out=out)

    for _ in range(args.warmup):
        flush.zero_()
        call(q)
    ctx.sync()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            call(q)
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms_step = all_max(world, sum(a.elapsed_time(b) for a, b in ev)) / args.steps
    # end to end: the query from pinned host memory, the output back to it
    qh = q.cpu().pin_memory()
    qd = torch.empty_like(q)
    oh = torch.empty(MLA_HEADS, MLA_HD).pin_memory()
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for i in range(args.steps):
        flush.zero_()
        ev2[i][0].record(stream)
        qd.copy_(qh, non_blocking=True)
        call(qd)
        oh.copy_(out, non_blocking=True)
        ev2[i][1].record(stream)
    torch.cuda.synchronize()
    e2e_ms = all_max(world, sum(a.elapsed_time(b) for a, b in ev2)) / args.steps
    peak, peak_kind = peaks()
    rows = 128 + MLA_COMP
    alg = rows * MLA_HD * 4 + 2 * MLA_HEADS * MLA_HD * 4 + MLA_HEADS * 4
    achieved = alg / (ms_step * 1e-3) / 1e9
    clocks = clk.summary()
    sm_mhz = (clocks or {}).get("sm_mhz") or 1965.0
    chain_us = (MLA_HD + rows) * FADD_CHAIN_CYCLES / sm_mhz
    res = None
    if rank == 0:
        res = {
            "metric": METRIC_MLA, "value": round(world * 1e3 / ms_step, 2), "unit": "calls/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 (reference operation order, no FMA)",
            "data": "synthetic (N(0, 1) cache rows, N(0, 0.05) queries)", "config": cfg,
            "roofline": {"kernel": "mla_scores_kernel + mla_weights_kernel + mla_output_kernel",
                         "bound": "hbm",
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "algorithmic_bytes": alg, "traffic": MLA_TRAFFIC,
                         "chain_floor_us": round(chain_us, 3),
                         "frac_of_chain_floor": round(chain_us / (ms_step * 1e3), 4),
                         "note": "latency-bound: the reference's in-order sums are "
                                 f"dependent chains of {MLA_HD} (scores) and {rows} "
                                 "(weighted sum) additions; chain_floor_us = those "
                                 "additions at the measured 4.44 cycles each and the "
                                 "sampled SM clock"},
            "e2e": {"value": round(world * 1e3 / e2e_ms, 2), "unit": "calls/s",
                    "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": q.numel() * 4,
                    "d2h_bytes_per_step": out.numel() * 4,
                    "path": "pinned host q -> H2D -> wh_mla_attention (C ABI) -> D2H output"},
            "gpu_launches": 3 * args.steps,
            "clocks": clocks,
        }
        if not args.no_cpu_baseline:
            host = [t.cpu().numpy() for t in (q, keys, comp, sink)]
            sec = mla_cpu(*host, fr, 3)
            res["cpu_baseline"] = {"value": round(1.0 / sec, 2), "unit": "calls/s", "cores": 1,
                                   "kind": "port",
                                   "sample": "3 full calls of the oracle's scalar restatement"}
    ctx.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return res


METRIC_MHC = "mHC hc_pre + hc_post token-calls/s (DeepSeek-V4 hyper-connections, one sub-block)"
MHC_HC, MHC_HIDDEN = 4, 4096
WORKLOAD_MHC = ("mHC of DeepSeek-V4 (hc_mult 4 x hidden 4096, 24 fn rows, 20 Sinkhorn rounds): "
                "hc_pre (RMS, fn mixes, Sinkhorn split, pooled input) then hc_post "
                "(redistribution over the 4 residual copies)")


def mhc_inputs(dev, seed, T):
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    rows, hc_dim = (2 + MHC_HC) * MHC_HC, MHC_HC * MHC_HIDDEN
    fn = torch.randn(rows, hc_dim, device=dev, generator=g) * 0.01
    scale = torch.tensor([0.3, 0.2, 0.5], device=dev)
    base = torch.randn(rows, device=dev, generator=g) * 0.1
    x = torch.randn(T, hc_dim, device=dev, generator=g)
    res = torch.randn(T, hc_dim, device=dev, generator=g)
    return fn, scale, base, x, res


def mhc_cpu(fn, scale, base, x, res, steps):
    """The oracle's scalar restatement on one host thread: seconds per token-call."""
    import oracle as O

    t0 = time.perf_counter()
    n = 0
    for _ in range(steps):
        for t in range(x.shape[0]):
            st, y, post, comb = O.hc_pre(fn, scale, base, x[t], MHC_HC, MHC_HIDDEN)
            O.hc_post(y, res[t], post, comb, MHC_HC, MHC_HIDDEN)
            n += 1
    return (time.perf_counter() - t0) / n


def run_mhc(args):
    import torch

    import wohper_b200 as W

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    T = max(args.mhc_tokens, 1)
    fn, scale, base, x, res = mhc_inputs(dev, 900 + rank, T)
    hc_dim = MHC_HC * MHC_HIDDEN
    cfg = {"workload": WORKLOAD_MHC, "hc_mult": MHC_HC, "hidden": MHC_HIDDEN, "tokens": T,
           "l2": "flushed between calls (256 MiB memset outside the timed events)",
           "parallelism": f"replicas x{world}" if world > 1 else "single GPU"}
    if args.impl == "reference":
        res_line = None
        if rank == 0:
            host = [t.cpu().numpy() for t in (fn, scale, base, x, res)]
            sec = mhc_cpu(*host, max(args.steps, 1))
            v = 1.0 / sec
            res_line = {"metric": METRIC_MHC, "value": round(v, 2), "unit": "token-calls/s",
                        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                        "higher_is_better": True, "impl": "reference", "scaling": "weak",
                        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
                        "cpu_baseline": {"value": round(v, 2), "unit": "token-calls/s",
                                         "cores": 1, "kind": "port",
                                         "sample": f"{max(args.steps, 1) * T} token-calls"},
                        "e2e": {"value": round(v, 2), "unit": "token-calls/s",
                                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return res_line

    ctx = W.Context(local)
    bufs = (torch.empty(T, MHC_HIDDEN, device=dev), torch.empty(T, MHC_HC, device=dev),
            torch.empty(T, MHC_HC, MHC_HC, device=dev))
    out = torch.empty(T, hc_dim, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def call(xd):
        y, post, comb = W.hc_pre(ctx, fn, scale, base, xd, MHC_HC, MHC_HIDDEN, out=bufs)
        W.hc_post(ctx, y, res, post, comb, MHC_HC, MHC_HIDDEN, out=out)

    for _ in range(args.warmup):
        flush.zero_()
        call(x)
    ctx.sync()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            call(x)
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms_step = all_max(world, sum(a.elapsed_time(b) for a, b in ev)) / args.steps
    xh = x.cpu().pin_memory()
    xd = torch.empty_like(x)
    oh = torch.empty(T, hc_dim).pin_memory()
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for i in range(args.steps):
        flush.zero_()
        ev2[i][0].record(stream)
        xd.copy_(xh, non_blocking=True)
        call(xd)
        oh.copy_(out, non_blocking=True)
        ev2[i][1].record(stream)
    torch.cuda.synchronize()
    e2e_ms = all_max(world, sum(a.elapsed_time(b) for a, b in ev2)) / args.steps
    peak, peak_kind = peaks()
    rows = (2 + MHC_HC) * MHC_HC
    alg = (rows * hc_dim * 4 + rows * 4 + 12 +
           T * (hc_dim * 4 + MHC_HIDDEN * 4 + (MHC_HC + MHC_HC * MHC_HC) * 4) +
           T * (MHC_HIDDEN * 4 + 2 * hc_dim * 4 + (MHC_HC + MHC_HC * MHC_HC) * 4))
    achieved = alg / (ms_step * 1e-3) / 1e9
    clocks = clk.summary()
    sm_mhz = (clocks or {}).get("sm_mhz") or 1965.0
    chain_us = hc_dim * FADD_CHAIN_CYCLES / sm_mhz
    res_line = None
    if rank == 0:
        res_line = {
            "metric": METRIC_MHC, "value": round(world * T * 1e3 / ms_step, 2),
            "unit": "token-calls/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (reference operation order, no FMA)",
            "data": "synthetic (N(0, 0.01) fn rows, N(0, 1) residual copies)", "config": cfg,
            "roofline": {"kernel": "hc_dots_kernel + hc_split_kernel + hc_post_kernel",
                         "bound": "hbm",
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "algorithmic_bytes": alg, "traffic": None,
                         "chain_floor_us": round(chain_us, 3),
                         "frac_of_chain_floor": round(chain_us / (ms_step * 1e3), 4),
                         "note": "latency-bound: the sum of squares and each fn-row dot are "
                                 f"chains of {hc_dim} dependent additions in the "
                                 "reference's order; chain_floor_us = one such chain at "
                                 "the measured 4.44 cycles an addition and the sampled "
                                 "SM clock"},
            "e2e": {"value": round(world * T * 1e3 / e2e_ms, 2), "unit": "token-calls/s",
                    "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": x.numel() * 4,
                    "d2h_bytes_per_step": out.numel() * 4,
                    "path": "pinned host x -> H2D -> wh_hc_pre + wh_hc_post (C ABI) -> D2H"},
            "gpu_launches": 3 * args.steps,
            "clocks": clocks,
        }
        if not args.no_cpu_baseline:
            host = [t.cpu().numpy() for t in (fn, scale, base, x, res)]
            sec = mhc_cpu(*host, 3)
            res_line["cpu_baseline"] = {"value": round(1.0 / sec, 2), "unit": "token-calls/s",
                                        "cores": 1, "kind": "port",
                                        "sample": f"{3 * T} token-calls of the oracle's scalar "
                                                  "restatement"}
    ctx.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return res_line


def run_ncu_case(args):
    """Small single-GPU workloads for ncu captures (no JSON bench line).

    fp8:   config-1 FP8 GEMV (4096 x 4096, one token), one launch per step.
    moe16: the config-2 MoE FFN step with 16 routed experts instead of 256
           (220 MB of weights; the kernels read the same 7 experts' bytes per
           token as at 256), router + moe_up + moe_down per step.
    grouped16: the config-3 batched path at 256 tokens and 16 experts (plus
           the shared one) of the config shape: router, dispatch, grouped up
           and down GEMMs, combine per step.
    lmhead: the BF16 lm_head top-50 on 32768 x 4096 (268 MB of weights),
           logits + candidates + selection per step.
    mla:   the MLA attention core at the bench's shape (10 MB of cache rows).
    mhc:   hc_pre + hc_post of one token at the bench's shape.
    moe-batch: one wh_moe_ffn layer of 256 V4-shape experts + shared with
           --batch tokens (softmax routing): the batched-decode grouped path
           (32 tokens: 16-token tiles) or, from 171 tokens, 112-token tiles.
    L2 is flushed (256 MiB memset) before every step."""
    import torch

    import wohper_b200 as W
    from tests import helpers as H

    ctx = W.Context(0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    n = args.warmup + args.steps
    if args.ncu_case == "mhc":
        fn, scale, base, x, res = mhc_inputs(torch.device("cuda", 0), 6, 1)
        for _ in range(n):
            flush.zero_()
            y, post, comb = W.hc_pre(ctx, fn, scale, base, x, MHC_HC, MHC_HIDDEN)
            W.hc_post(ctx, y, res, post, comb, MHC_HC, MHC_HIDDEN)
    elif args.ncu_case == "mla":
        q, keys, comp, sink = mla_inputs(torch.device("cuda", 0), 5)
        theta, yarn = W.deepseek_rope_for_layer(2)
        fr = W.rope_inv_freqs(MLA_HD - MLA_NOPE, theta, yarn)
        for _ in range(n):
            flush.zero_()
            W.mla_attention(ctx, q, keys, MLA_POS, fr, MLA_NOPE, compressed=comp, sink=sink)
    elif args.ncu_case == "lmhead":
        g = torch.Generator(device="cuda")
        g.manual_seed(3)
        wl = (torch.randn(32768, HID, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        wl = wl.view(torch.int16)
        x = torch.randn(HID, device="cuda", generator=g)
        for _ in range(n):
            flush.zero_()
            W.lm_head_topk_score(ctx, wl, x, 50)
    elif args.ncu_case == "fp8":
        w, s = H.fp8_weight(1, HID, HID)
        wd, sd = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda()
        x = torch.from_numpy(H.activations(2, 1, HID).reshape(-1)).cuda()
        for _ in range(n):
            flush.zero_()
            W.gemv_fp8_e4m3_ue8m0_tensorwise(ctx, wd, sd, x)
    elif args.ncu_case == "moe-batch":
        ne, T = E, args.batch
        stack = H.torch_fp4_experts(88, ne + 1, HID, INTER)
        gate = H.router_gate(89, ne, HID)

        def wexp(e):
            w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
            return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, INTER, HID, HID // 32),
                                         W.Fp4Matvec(w3, s3, INTER, HID, HID // 32),
                                         W.Fp4Matvec(w2, s2, HID, INTER, INTER // 32))

        layer = W.MoeLayer(ctx, [wexp(e) for e in range(ne)], wexp(ne),
                           torch.from_numpy(gate.view(np.int16)).cuda(), topk=TOPK, max_tokens=T)
        x = torch.from_numpy(H.activations(90, T, HID)).cuda()
        for _ in range(n):
            flush.zero_()
            layer.forward(x)
        layer.close()
    elif args.ncu_case == "grouped16":
        ne, T = 16, 256
        stack = H.torch_fp4_experts(5, ne + 1, HID, INTER)
        gate, xs = H.zipf_routing(9, H.router_gate(6, ne, HID), H.activations(7, T, HID))

        def wexp(e):
            w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
            return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, INTER, HID, HID // 32),
                                         W.Fp4Matvec(w3, s3, INTER, HID, HID // 32),
                                         W.Fp4Matvec(w2, s2, HID, INTER, INTER // 32))

        layer = W.MoeLayer(ctx, [wexp(e) for e in range(ne)], wexp(ne),
                           torch.from_numpy(gate.view(np.int16)).cuda(), topk=TOPK, max_tokens=T)
        x = torch.from_numpy(xs).cuda()
        y = torch.empty_like(x)
        for i in range(n):
            flush.zero_()
            layer.forward(x, y)
        layer.close()
    else:
        ne = 16
        stack = H.torch_fp4_experts(5, ne + 1, HID, INTER)
        gate = torch.from_numpy(H.router_gate(6, ne, HID).view(np.int16)).cuda()

        def wexp(e):
            w1, s1, w3, s3, w2, s2 = H.expert_views(stack, e)
            return W.DeepSeekV4Fp4Expert(W.Fp4Matvec(w1, s1, INTER, HID, HID // 32),
                                         W.Fp4Matvec(w3, s3, INTER, HID, HID // 32),
                                         W.Fp4Matvec(w2, s2, HID, INTER, INTER // 32))

        layer = W.MoeLayer(ctx, [wexp(e) for e in range(ne)], wexp(ne), gate, topk=TOPK,
                           max_tokens=1)
        xs = torch.from_numpy(H.activations(7, n, HID)).cuda()
        y = torch.empty(1, HID, device="cuda")
        for i in range(n):
            flush.zero_()
            layer.forward(xs[i:i + 1], y)
        layer.close()
    ctx.sync()
    ctx.close()
    print(json.dumps({"ncu_case": args.ncu_case, "steps": n}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ep", action="store_true",
                    help="config 2: skip the nested config-4 expert-parallel measurement")
    ap.add_argument("--batch", type=int, default=1, help="config 5: sequences per step")
    ap.add_argument("--tokens", type=int, default=0,
                    help="config 3: tokens per step (default 2048; 16384 is the compute-bound point)")
    ap.add_argument("--layers", type=int, default=V4_LAYERS, help="config 5: layers")
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5],
                    help="1: one FP8 GEMV 4096x4096; 2: one-token decode FFN (default); "
                         "3: 2048-token batched FFN; 4: expert-parallel layer over the ranks")
    ap.add_argument("--ep-transport", default="p2p", choices=["p2p", "nccl"],
                    help="config 4: rows over NVLink peer stores (p2p) or NCCL all-to-all")
    ap.add_argument("--workload", default="moe", choices=["moe", "expert-load", "lm-head", "mla", "mhc"],
                    help="moe: the MoE FFN step of --config (default); expert-load: one "
                         "layer's FP4 experts from an experts pack on disk into HBM; lm-head: "
                         "the BF16 lm_head top-k over the DeepSeek vocabulary; mla: the MLA "
                         "attention core of one DeepSeek-V4 layer at token 4095; mhc: hc_pre + "
                         "hc_post of one DeepSeek-V4 sub-block")
    ap.add_argument("--load-threads", type=int, default=8,
                    help="expert-load: reader threads of the expert loader")
    ap.add_argument("--direct-io", action="store_true",
                    help="expert-load: O_DIRECT reads (bypass the page cache)")
    ap.add_argument("--lm-top-k", type=int, default=50, help="lm-head: top_k")
    ap.add_argument("--mhc-tokens", type=int, default=1, help="mhc: tokens per call")
    ap.add_argument("--shared", default="fp4", choices=["fp4", "fp8"],
                    help="config 2: the shared expert's format (fp4, as BASELINE's config 2; "
                         "fp8: DeepSeek-V4's FP8 shared expert)")
    ap.add_argument("--ncu-case", choices=["fp8", "moe16", "grouped16", "moe-batch", "lmhead", "mla",
                                           "mhc"],
                    help="run a small workload for an ncu capture instead of the bench")
    args = ap.parse_args()
    if args.ncu_case:
        run_ncu_case(args)
        return
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    if args.tokens > 0:
        global T3
        T3 = args.tokens
    if args.workload == "expert-load":
        res = run_expert_load(args)
    elif args.workload == "lm-head":
        res = run_lm_head(args)
    elif args.workload == "mla":
        res = run_mla(args)
    elif args.workload == "mhc":
        res = run_mhc(args)
    elif args.config == 5:
        res = run_config5(args) if args.impl == "ours" else run_reference_config5(args)
    elif args.config == 1:
        res = run_config1(args) if args.impl == "ours" else run_reference_config1(args)
    elif args.config == 3:
        res = run_config3(args) if args.impl == "ours" else run_reference_moe_batch(args, 3)
    elif args.config == 4:
        res = run_config4(args) if args.impl == "ours" else run_reference_moe_batch(args, 4)
    else:
        res = run_reference(args) if args.impl == "reference" else run_ours(args)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
