"""Benchmark of the B200 hot path (driver contract: one JSON line on rank 0).

Workload (decode part): the op-level quantized
mul_mat sweep at batch-8 decode.  One step = one GGML_OP_MUL_MAT per weight of
the Qwen3-0.6B-shaped set {4096x1024, 1024x2048, 6144x1024, 1024x3072,
151936x1024} in each of Q8_0, Q4_0 and Q4_K (15 ops), activations f32 [8, K].
Metric: achieved decode mul_mat HBM GB/s = algorithmic bytes (quantized weight
bytes + M*K*4 + M*N*4 per op) / step time.  The 374 MB of weights exceed the
126 MB L2, so every step streams them from HBM (no flush needed).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Multi-GPU (torchrun, one process per GPU): every rank runs the same sweep on
its own GPU (independent replicas, no data-path collective); NCCL is used only
for the barrier and the max-over-ranks of the device time; value = the sum of
all ranks' bytes / the slowest rank's time ("scaling": "weak").
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [(4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (151936, 1024)]
TYPES = {"q8_0": 8, "q4_0": 2, "q4_k": 12}
BPE = {8: 34 / 32, 2: 18 / 32, 12: 144 / 256}
M = 8
SEED = 0x0A5A0002
METRIC = "decode mul_mat HBM GB/s (BASELINE metric part 2), Qwen3-0.6B weight sweep x {Q8_0,Q4_0,Q4_K}, M=8"


def op_bytes(qt: int, N: int, K: int, m: int = M) -> float:
    return N * K * BPE[qt] + m * K * 4 + m * N * 4


STEP_BYTES = sum(op_bytes(qt, N, K) for qt in TYPES.values() for (N, K) in SHAPES)


def make_weights(quantize, synth):
    ws = []
    for ti, (name, qt) in enumerate(TYPES.items()):
        for si, (N, K) in enumerate(SHAPES):
            x = synth(SEED + 16 * ti + si, N * K, 0.0, 0.02).reshape(N, K)
            ws.append((name, qt, N, K, quantize(qt, x)))
    return ws


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            # stdbuf: nvidia-smi block-buffers into a pipe; line buffering lets samples through
            self.proc = subprocess.Popen(
                ["stdbuf", "-oL", "nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=lambda: self.lines.extend(iter(self.proc.stdout.readline, "")), daemon=True)
        self.thread.start()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak_hbm() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic() -> float | None:
    p = os.path.join(ROOT, "profiles", "mmv_q8_0_lm_head_151936x1024_m8.json")
    if os.path.exists(p):
        try:
            return float(json.load(open(p))["dram_bytes_per_launch"])
        except (KeyError, ValueError):
            return None
    return None


# ---------------------------------------------------------------------------------------
def cpu_baseline(seconds: float = 12.0, kind_ref: bool = False) -> dict:
    """The CPU restatement of ggml's mul_mat (oracle, OpenMP over all host cores) on a
    bounded sample of the same workload: the four non-lm_head shapes of each type
    (plus the lm_head rows 0..4095), repeated for about `seconds`."""
    from oracle import oracle as oo

    cores = os.cpu_count() or 1
    sample = []
    for ti, (name, qt) in enumerate(TYPES.items()):
        for si, (N, K) in enumerate(SHAPES):
            n = min(N, 4096)
            w = oo.synth_normal(SEED + 16 * ti + si, n * K, 0.0, 0.02).reshape(n, K)
            sample.append((qt, n, K, oo.quantize(qt, w)))
    x = {K: oo.synth_normal(SEED ^ K, M * K).reshape(M, K) for K in {k for _, k in SHAPES}}
    nbytes, reps, t0 = 0.0, 0, time.perf_counter()
    while True:
        for qt, n, K, wq in sample:
            oo.mul_mat(wq, qt, K, n, x[K])
            nbytes += op_bytes(qt, n, K)
        reps += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{reps} passes over 15 ops (all shapes, lm_head cut to 4096 rows) x M=8, "
                      f"OpenMP {cores} threads, {dt:.1f} s"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # the reference's own ggml CPU path is unbuildable here (empty ggml submodule,
    # no Rust toolchain), so its CPU restatement in oracle/ is timed
    per_step = max(2.0, 60.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_baseline(seconds=per_step * 0.25)
    vals = [cpu_baseline(seconds=per_step)["value"] for _ in range(args.steps)]
    cb = cpu_baseline(seconds=per_step)
    v = statistics.median(vals)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": STEP_BYTES / (v * 1e9) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q8_0/q4_0/q4_K x f32 (int8 block dot, f32 accumulate)",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
        "config": {"workload": "configs[1] decode mul_mat sweep, M=8", "shapes": SHAPES, "types": list(TYPES),
                   "l2": "inputs larger than L2 (374 MB of weights per step)"},
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": cb["cores"], "kind": "port", "sample": cb["sample"]},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    import openasr_b200 as ob

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    stream = torch.cuda.Stream()
    be = ob.Backend(local)
    be.set_stream(stream)
    ws = make_weights(ob.quantize, ob.synth_normal)
    with torch.cuda.stream(stream):
        W = [(name, qt, N, K, be.upload_weight(q, qt, [K, N])) for (name, qt, N, K, q) in ws]
        xs = {K: torch.from_numpy(ob.synth_normal(SEED ^ K, M * K).reshape(M, K)).cuda() for K in {k for _, k in SHAPES}}
        outs = [torch.empty((M, N), dtype=torch.float32, device="cuda") for (_, _, N, _, _) in W]
        lm_idx = [i for i, w in enumerate(W) if w[0] == "q8_0" and w[2] == 151936][0]
        lm_qact = torch.empty(be.act_bytes(8, 1024, M), dtype=torch.uint8, device="cuda")
        # host side of the e2e leg: pinned activations in, pinned results out
        hx = {K: x.cpu().pin_memory() for K, x in xs.items()}
        hout = [torch.empty((M, N), dtype=torch.float32).pin_memory() for (_, _, N, _, _) in W]
    be.reserve_scratch(64 << 20)
    lm_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]

    def step(i_timed: int | None):
        for j, (name, qt, N, K, w) in enumerate(W):
            if j == lm_idx:
                be.quantize_act(qt, xs[K], lm_qact)
                if i_timed is not None:
                    lm_ev[i_timed][0].record(stream)
                be.mul_mat_qact(w, lm_qact, M, outs[j])
                if i_timed is not None:
                    lm_ev[i_timed][1].record(stream)
            else:
                be.mul_mat(w, xs[K], outs[j])

    def e2e_step():
        for K in xs:
            xs[K].copy_(hx[K], non_blocking=True)
        step(None)
        for j, o in enumerate(outs):
            hout[j].copy_(o, non_blocking=True)

    launches_per_step = 2 * len(W)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step(None)
        stream.synchronize()
        if world > 1:
            dist.barrier()
        sampler = ClockSampler(local)
        sampler.start()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record(stream)
        for i in range(args.steps):
            step(i)
        t1.record(stream)
        torch.cuda.synchronize()
        be.synchronize()
        clocks = sampler.stop()
        ms = t0.elapsed_time(t1) / args.steps
        lm_ms = sum(a.elapsed_time(b) for a, b in lm_ev) / args.steps
        # e2e: same metric through the public API with host buffers
        for _ in range(2):
            e2e_step()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])
    h2d = sum(x.numel() * 4 for x in xs.values())
    d2h = sum(o.numel() * 4 for o in outs)
    if rank == 0:
        peak, peak_kind = measured_peak_hbm()
        lm_bytes = op_bytes(8, 151936, 1024)
        achieved = lm_bytes / (lm_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": world * STEP_BYTES / (ms * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q8_0/q4_0/q4_K x f32 (int8 block dot, f32 accumulate)",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
            "config": {"workload": "configs[1] decode mul_mat sweep, M=8", "shapes": SHAPES, "types": list(TYPES),
                       "l2": "inputs larger than L2 (374 MB of weights per step)",
                       "parallelism": f"replicas x{world}"},
            "e2e": {"value": world * STEP_BYTES / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "hbm", "kernel": "mmv_q8_kernel (lm_head 151936x1024 Q8_0, M=8)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": ncu_traffic(), "algorithmic_bytes": lm_bytes,
                         "avg_launch_us": lm_ms * 1e3},
            "clocks": clocks,
        }
        line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    for w in W:
        w[4].free()
    be.close()
    if world > 1:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
