"""Benchmark of the B200 hot path (driver contract: one JSON line on rank 0).

Default workload (--workload rtfx): BASELINE.json's headline RTFx on the
configs[3]/[4] Whisper-large-v3-shaped Q4_K model, batch 8 per GPU.  The
utterances are configs[4]'s fixed job: 512 seeded utterances with lengths
U[5, 30] s, sharded round-robin over the N ranks (utterance u on rank u mod N).
A step runs mel + encoder + 224 greedy decoder steps on one batch of 8 of the
rank's utterances (the shard's batches in order, wrapping); after the K timed
steps the whole job (every rank its full shard) is timed once more as its own
leg: job RTFx = 512 utterances' audio / the slowest rank's time.

Qwen workload (--workload qwen [--batch 1|4|8]): the
Qwen3-ASR-0.6B-shaped Q8_0 decoder; one step = one oasr_b200_qwen_generate of
`batch` sequences per GPU (390-frame prompt standing for 30 s of audio, causal
prefill, 256 greedy tokens); metric RTFx = 30 s x sequences / device time.

Secondary workload (--workload mulmat, BASELINE.json configs[1], decode part): the op-level quantized
mul_mat sweep at batch-8 decode.  One step = one GGML_OP_MUL_MAT per weight of
the Qwen3-0.6B-shaped set {4096x1024, 1024x2048, 6144x1024, 1024x3072,
151936x1024} in each of Q8_0, Q4_0 and Q4_K (15 ops), activations f32 [8, K].
Metric: achieved decode mul_mat HBM GB/s = algorithmic bytes (quantized weight
bytes + M*K*4 + M*N*4 per op) / step time.  The 374 MB of weights exceed the
126 MB L2, so every step streams them from HBM (no flush needed).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Multi-GPU (torchrun, one process per GPU): every rank works on its own GPU
(no data-path collective, no NCCL); a gloo process group on the host carries
the barriers and the max-over-ranks of the device times; value = the sum of
all ranks' work / the slowest rank's time ("scaling": "weak").
"""
from __future__ import annotations

import argparse
import ctypes
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

    def wait_ready(self, timeout: float = 5.0) -> None:
        """Block until nvidia-smi has printed its first sample (it needs a few hundred ms
        to start), so that a short timed region that starts now is sampled."""
        t_end = time.time() + timeout
        while self.proc is not None and not self.lines and time.time() < t_end:
            time.sleep(0.01)

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
    """dram read + write bytes of one Qwen logits-head GEMV launch (Q8_0 151936 x 1024,
    M = 8), from its committed ncu summary."""
    return ncu_traffic_fa("mmv_q80_tc_lm_head_151936x1024_m8.md")


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


def run_reference_mulmat(args) -> None:
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


def run_b200_mulmat(args) -> None:
    import torch
    import torch.distributed as dist

    import openasr_b200 as ob

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    init_ranks(world)
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

    def step(_unused=None):
        for j, (name, qt, N, K, w) in enumerate(W):
            if j == lm_idx:
                be.quantize_act(qt, xs[K], lm_qact)
                be.mul_mat_qact(w, lm_qact, M, outs[j])
            else:
                be.mul_mat(w, xs[K], outs[j])

    def e2e_step():
        for K in xs:
            xs[K].copy_(hx[K], non_blocking=True)
        step(None)
        for j, o in enumerate(outs):
            hout[j].copy_(o, non_blocking=True)

    launches_per_step = 2 * len(W)
    # a step replays in ~0.2 ms: time at least 2500 of them (~0.5 s) so that the clock
    # sampler sees the timed region
    steps = max(args.steps, 2500)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step(None)
        stream.synchronize()
        # the device leg: one step (15 ops, 30 launches) captured once into a CUDA graph and
        # replayed, so the device time holds no host enqueue gaps (the e2e leg below keeps
        # the host-driven calls)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step(None)
        for _ in range(args.warmup):
            graph.replay()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        sampler = ClockSampler(local)
        sampler.start()
        sampler.wait_ready()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record(stream)
        for i in range(steps):
            graph.replay()
        t1.record(stream)
        torch.cuda.synchronize()
        be.synchronize()
        clocks = sampler.stop()
        ms = t0.elapsed_time(t1) / steps
        del graph
        # the roofline kernel alone: the lm_head GEMV on pre-quantized activations
        lm_w = W[lm_idx][4]
        be.quantize_act(8, xs[1024], lm_qact)
        lm_ms = graph_timed(torch, stream, lambda i: be.mul_mat_qact(lm_w, lm_qact, M, outs[lm_idx]), 20) / 1e3
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
        t = torch.tensor([ms, e2e_ms], dtype=torch.float64)
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
            "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q8_0/q4_0/q4_K x f32 (int8 block dot, f32 accumulate)",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
            "config": {"workload": "configs[1] decode mul_mat sweep, M=8", "shapes": SHAPES, "types": list(TYPES),
                       "l2": "inputs larger than L2 (374 MB of weights per step)",
                       "parallelism": f"replicas x{world}"},
            "e2e": {"value": world * STEP_BYTES / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * steps,
            "roofline": {"bound": "hbm", "kernel": "mmv_q80_tc_kernel (lm_head 151936x1024 Q8_0, M=8, pre-quantized "
                                                   "activations, graph-replayed alone)",
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


# ==================================================================================
# RTFx workload (default): BASELINE.json metric part 1 on configs[3]/[4]
# ==================================================================================
RTFX_METRIC = "RTFx (audio-s/s), Whisper-large-v3-shaped Q4_K, batch 8 per GPU, greedy 224 tokens"
N_NEW = 224
UTT_SEED = 0x0A5A0005


def graph_timed(torch, stream, fn, iters: int, replays: int = 3) -> float:
    """Mean device time (us) of one fn(i) call: `iters` calls captured into a CUDA graph
    (no host launch overhead between them), the graph replayed `replays` times between
    CUDA events on `stream`."""
    for i in range(3):
        fn(i)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(iters):
            fn(i)
    graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream.synchronize()
    e0.record(stream)
    for _ in range(replays):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) / (replays * iters) * 1e3


def init_ranks(world: int) -> None:
    """Host process group for the barriers and the timing reductions (gloo over
    127.0.0.1): the data path has no collective, so no NCCL communicator is made."""
    if world > 1:
        from datetime import timedelta

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=timedelta(seconds=600))


def gather_over_ranks(x: float) -> list[float]:
    """every rank's value (all ranks must call it)"""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [x]
    out = [torch.zeros(1, dtype=torch.float64) for _ in range(dist.get_world_size())]
    dist.all_gather(out, torch.tensor([x], dtype=torch.float64))
    return [float(t[0]) for t in out]


def reduce_over_ranks(dev_s: float, e2e_s: float, audio_s: float, device="cpu") -> tuple[float, float, float]:
    """Whole-job figures from every rank's own: the slowest rank's device and
    end-to-end times (max) and the audio seconds all ranks processed (sum).
    Every rank must call it (two collectives, same order); a single process
    returns its inputs."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return dev_s, e2e_s, audio_s
    t = torch.tensor([dev_s, e2e_s, audio_s], dtype=torch.float64, device=device)
    mx = t.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    tot = t.clone()
    dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    return float(mx[0]), float(mx[1]), float(tot[2])


JOB_UTTS = 512  # configs[4]: one job of 512 utterances


def job_lengths() -> list[int]:
    """the job's 512 utterance lengths, uniform in 5-30 s (seeded), 16 kHz samples."""
    rng = np.random.default_rng([UTT_SEED, JOB_UTTS])
    return [int(16000 * rng.uniform(5.0, 30.0)) for _ in range(JOB_UTTS)]


def job_shard(world: int, rank: int, B: int = 8) -> list[list[int]]:
    """utterance ids of this rank (round-robin: u on rank u mod world) in batches of B"""
    mine = list(range(rank, JOB_UTTS, world))
    return [mine[i:i + B] for i in range(0, len(mine), B)]


def job_pcm(u: int, n_samples: int, synth) -> np.ndarray:
    """seeded -20 dBFS Gaussian noise of utterance u (same bytes on every rank and arm)"""
    return synth(UTT_SEED + 7919 * (u + 1), n_samples, 0.0, 0.1)


def launches_per_batch(n_enc: int, n_dec: int, n_prompt: int, n_new: int, batch: int) -> int:
    """Kernel launches of one generate() (counted from model_whisper.cu, and equal to
    the committed launch list): mel 3; prelude 4 (2 im2col + 2 conv GEMMs) + batch
    positional adds; per encoder layer 12 (2 LayerNorm + quantize, 4 tensor-core GEMMs
    -- the QKV bias added in the QKV GEMM's store --, 3 f16 pre-pass + 1 tensor-core
    attention, attention-output quantize, GELU + quantize); final norm 1; 2 cross-K/V per decoder layer (GEMM + f16
    cast); per decoder step 1 embed + 1 first LayerNorm + 12 per layer (qkv GEMV, self
    attention, o GEMV, LayerNorm, cross-q GEMV, cross attention, cross-o GEMV,
    LayerNorm, fc1 GEMV, GELU + quantize, fc2 GEMV, LayerNorm) + logits + argmax +
    position advance; 1 token fill per prompt step."""
    enc = 3 + 4 + batch + n_enc * 12 + 1 + 2 * n_dec
    steps = n_prompt + n_new - 1
    return enc + steps * (1 + 1 + 12 * n_dec + 2 + 1) + n_prompt


def rtfx_cpu_sample(warmup_steps: int = 1, timed_steps: int = 8) -> dict:
    """The reference path's CPU arithmetic (oracle/, OpenMP over every host core) on a
    bounded sample of the workload: the full 32 + 32-layer whisper-large-v3-shaped Q4_K
    model built from the oracle's own quantizer and generator (nothing of
    liboasr_b200 is loaded), one utterance of the configs[4] job padded to 30 s:
    log-mel + encoder + cross-K/V once, then `timed_steps` greedy decoder steps.  The
    only extrapolation is over the step count: an utterance costs encoder +
    (4 prompt + 224 new - 1) decoder steps."""
    from openasr_b200 import models as om
    from oracle import oracle as oo
    from oracle import whisper_ref as wr

    cores = os.cpu_count() or 1
    cfg = om.WHISPER_LARGE_V3.replace(max_batch=1)
    t0 = time.perf_counter()
    pack = om.whisper_synthetic_pack(cfg, seed=0x0A5A0004, synth=oo.synth_normal, quantize=oo.quantize)
    t_pack = time.perf_counter() - t0
    lens = job_lengths()
    clip = job_pcm(0, lens[0], oo.synth_normal)
    ref = wr.WhisperRef(cfg, pack)
    t0 = time.perf_counter()
    enc = ref.encode(wr.log_mel(clip, cfg.n_mels))
    cross = ref.cross_kv(enc)
    t_enc = time.perf_counter() - t0
    state = ref.new_state()
    prompt = om.PROMPT[cfg.n_vocab]
    toks = list(prompt)
    step_s = []
    for pos in range(warmup_steps + timed_steps):
        t0 = time.perf_counter()
        logits = ref.decode_step(toks[pos], pos, cross, state)
        dt = time.perf_counter() - t0
        if pos >= len(prompt) - 1:
            toks.append(int(oo.argmax_first(logits)[0]))
        if pos >= warmup_steps:
            step_s.append(dt)
    t_step = float(np.mean(step_s))
    n_steps = len(prompt) + N_NEW - 1
    per_utt = t_enc + n_steps * t_step
    mean_audio = float(np.mean(lens)) / 16000.0
    return {"value": mean_audio / per_utt, "unit": "audio-s/s", "cores": cores, "kind": "port",
            "t_encoder_s": t_enc, "t_step_s": t_step, "step_times_s": step_s, "per_utterance_s": per_utt,
            "sample": (f"oracle (CPU restatement of the ggml path, OpenMP {cores} threads), full 32+32-layer model "
                       f"(pack built by the oracle in {t_pack:.0f} s, untimed): one 30 s-padded utterance, log-mel + "
                       f"encoder + cross-K/V {t_enc:.1f} s, {timed_steps} decoder steps {t_step * 1e3:.0f} ms each "
                       f"(after {warmup_steps} untimed); an utterance = encoder + {n_steps} steps = {per_utt:.0f} s; "
                       f"mean configs[4] audio {mean_audio:.1f} s")}


def run_reference(args) -> None:
    """The reference arm: the reference's own ggml CPU path cannot be built here (empty
    ggml submodule, no Rust toolchain), so its CPU restatement (oracle/) runs the same
    workload on the host cores.  A step is one full-depth decoder step of one utterance
    (what ms_per_step reports); the encoder runs once before the warm-up steps; value =
    the configs[4] mean audio / (encoder + 227 steps).  Under torchrun rank 0 alone
    runs and prints; the other ranks exit 0 without work."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cb = rtfx_cpu_sample(warmup_steps=args.warmup, timed_steps=args.steps)
    v = cb["value"]
    print(json.dumps({
        "impl": "reference", "metric": RTFX_METRIC, "value": v, "unit": "audio-s/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["t_step_s"] * 1e3, "higher_is_better": True,
        "scaling": "host (one CPU measurement at every N)", "vs_baseline": None,
        "dtype": "q4_K x q8_K int dot, f32 accumulate; f16 KV",
        "data": "synthetic (seeded N(0,0.02) Q4_K weights, -20 dBFS Gaussian-noise audio, lengths U[5,30] s)",
        "config": {"workload": "configs[3] model (whisper-large-v3-shaped Q4_K, 32+32 layers) on the configs[4] job's "
                               "utterances, greedy 224 tokens; a step = one decoder step of one utterance on the CPU",
                   "encoder_s": cb["t_encoder_s"], "per_utterance_s": cb["per_utterance_s"],
                   "l2": "inputs larger than L2"},
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": v, "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def _fa_roofline(be, torch, stream, n_layers_rot: int = 4, iters: int = 20) -> dict:
    """The dominant kernel of the decode step -- cross-attention flash-decode over the
    f16 cross-K/V of 8 utterances (fattn_heads_kernel, D 64, 20 heads, n_kv 1500) --
    timed alone on the benchmark stream from a CUDA graph of `iters` launches,
    rotating over 4 layers' K/V (246 MB > L2)."""
    S, H, N, D = 8, 20, 1500, 64
    kv = [torch.randn(S, N, 2 * H * D, device="cuda").half() for _ in range(n_layers_rot)]
    q = torch.randn(S, 1, H * D, device="cuda")
    out = torch.empty(S, 1, H * D, device="cuda")
    views = []
    for t in kv:
        k = t[:, :, : H * D].reshape(S, N, H, D).permute(0, 2, 1, 3)
        v = t[:, :, H * D:].reshape(S, N, H, D).permute(0, 2, 1, 3)
        views.append((k, v))
    qv = q.reshape(S, 1, H, D).permute(0, 2, 1, 3)
    ov = out.reshape(S, 1, H, D)

    def launch(i):
        be.flash_attn_ext(qv, views[i % n_layers_rot][0], views[i % n_layers_rot][1], None, 0.125, ov)

    us = graph_timed(torch, stream, launch, iters)
    nbytes = S * N * 2 * H * D * 2 + 2 * S * H * D * 4
    return {"us": us, "bytes": nbytes}


def whisper_step_bytes(cfg, B: int, n_prompt: int, n_new: int) -> dict:
    """Algorithmic bytes of one Whisper decode step at batch B: every decoder weight once
    (Q4_K decode tiles 144 B / 256 weights, the Q8_0 logits head 34 B / 32), the cross K/V
    of every layer (f16, 1500 frames x (K | V)), the self K/V rows up to the mean cache
    length of a batch's steps, the activations negligible."""
    d, L, V, T = cfg.d_model, cfg.n_dec_layers, cfg.n_vocab, cfg.n_audio_ctx
    per_layer = d * (3 * d + d + d + d + 4 * d) + 4 * d * d  # qkv, o, cross q, cross o, fc1, fc2
    weights = L * per_layer * 144 // 256 + V * d * 34 // 32
    cross = L * B * T * 2 * d * 2
    steps = n_prompt - 1 + n_new
    mean_kv = sum(p + 1 for p in range(steps)) / steps
    self_kv = int(L * B * mean_kv * 2 * d * 2)
    return {"weights": weights, "cross_kv": cross, "self_kv": self_kv, "total": weights + cross + self_kv}


def _step_roofline(model, torch, stream, lens, B, n_new, toks_dev) -> dict:
    """Per-step time of the Whisper decode graph: two generate calls from the same device
    mel (encoder + prompt + n steps), n = n_new and n = 32, timed with CUDA events on the
    bench stream; their difference over n_new - 32 steps is the step alone."""
    ev = lambda: torch.cuda.Event(enable_timing=True)
    ts = {}
    for n in (n_new, 32):
        model.generate_device(B, toks_dev, n_new=n)  # warm (graphs of this width exist)
        e0, e1 = ev(), ev()
        e0.record(stream)
        for _ in range(3):
            model.generate_device(B, toks_dev, n_new=n)
        e1.record(stream)
        torch.cuda.synchronize()
        ts[n] = e0.elapsed_time(e1) / 3 * 1e3
    return {"us": (ts[n_new] - ts[32]) / (n_new - 32), "batch_us": ts[n_new]}


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    import openasr_b200 as ob
    from openasr_b200 import models as om

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    init_ranks(world)
    B = 8
    cfg = om.WHISPER_LARGE_V3.replace(max_batch=B)
    t_setup = time.perf_counter()
    pack = om.whisper_synthetic_pack(cfg, seed=0x0A5A0004)
    stream = torch.cuda.Stream()
    be = ob.Backend(local)
    be.set_stream(stream)
    model = om.WhisperModel(be, cfg, pack)
    del pack

    # this rank's round-robin shard of the 512-utterance job, in batches of 8
    lens_all = job_lengths()
    shard = job_shard(world, rank, B)
    lens = [[lens_all[u] for u in b] for b in shard]
    audio_s = [sum(l) / 16000.0 for l in lens]
    pcm_host = [np.concatenate([job_pcm(u, lens_all[u], ob.synth_normal) for u in b]) for b in shard]
    with torch.cuda.stream(stream):
        pcm_dev = [torch.from_numpy(p).cuda() for p in pcm_host]
        pcm_pin = [torch.from_numpy(p).pin_memory() for p in pcm_host]
        toks_dev = torch.empty((B, N_NEW), dtype=torch.int32, device="cuda")
    t_setup = time.perf_counter() - t_setup
    nb = len(shard)

    def step_device(i):
        j = i % nb
        model.mel_device(pcm_dev[j], lens[j])
        model.generate_device(len(shard[j]), toks_dev, n_new=N_NEW)

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step_device(i)
        stream.synchronize()
        barrier()
        # ---- K timed steps: batches of the shard in order (wrapping) ----
        sampler = ClockSampler(local)
        sampler.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(args.warmup, args.warmup + args.steps):
            step_device(i)
        e1.record(stream)
        torch.cuda.synchronize()
        be.synchronize()
        dev_s = e0.elapsed_time(e1) / 1e3
        # ---- the configs[4] job: this rank's whole shard, once, through the serve loop ----
        # (continuous batching: finished slots refilled from the queue, pinned host PCM in,
        # host tokens out, every copy inside the timed region)
        barrier()
        job_s = float("nan")
        job_stats, job_tokens = None, 0
        if not args.no_job:
            flat = [u for b in shard for u in b]
            job_lens = np.ascontiguousarray([lens_all[u] for u in flat], np.int64)
            job_pin = torch.from_numpy(np.concatenate(pcm_host)).pin_memory()
            job_out = np.empty((len(flat), N_NEW), np.int32)
            job_n = np.zeros(len(flat), np.int32)
            job_stats = ob.backend.ServeStats()
            prompt = np.ascontiguousarray(om.PROMPT[cfg.n_vocab], np.int32)
            j0, j1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            j0.record(stream)
            be._check(ob.lib().oasr_b200_whisper_serve(
                model.handle, job_pin.data_ptr(), job_lens.ctypes.data, len(flat), prompt.ctypes.data, len(prompt),
                None, N_NEW, om.EOT, 1, 0, 8, job_out.ctypes.data, job_n.ctypes.data, ctypes.byref(job_stats)))
            j1.record(stream)
            torch.cuda.synchronize()
            be.synchronize()
            job_s = j0.elapsed_time(j1) / 1e3
            job_tokens = int(job_n.sum())
        clocks = sampler.stop()
        # ---- e2e: the public transcribe call on pinned host PCM -> host tokens, copies included ----
        barrier()
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0.record(stream)
        for i in range(args.warmup, args.warmup + args.steps):
            j = i % nb
            out = np.empty((len(shard[j]), N_NEW), np.int32)
            be._check(ob.lib().oasr_b200_whisper_transcribe(
                model.handle, pcm_pin[j].data_ptr(), np.ascontiguousarray(lens[j], np.int64).ctypes.data,
                len(shard[j]), np.ascontiguousarray(om.PROMPT[cfg.n_vocab], np.int32).ctypes.data, 4, N_NEW, om.EOT,
                0, out.ctypes.data))
        h1.record(stream)
        torch.cuda.synchronize()
        e2e_s = h0.elapsed_time(h1) / 1e3
        fa = _fa_roofline(be, torch, stream)
        model.mel_device(pcm_dev[0], lens[0])
        st = _step_roofline(model, torch, stream, lens[0], len(shard[0]), N_NEW, toks_dev)
    timed_audio = sum(audio_s[i % nb] for i in range(args.warmup, args.warmup + args.steps))
    dev_s, e2e_s, timed_audio = reduce_over_ranks(dev_s, e2e_s, timed_audio)
    job_times = gather_over_ranks(job_s)
    if rank == 0:
        peak, peak_kind = measured_peak_hbm()
        achieved = fa["bytes"] / (fa["us"] * 1e-6) / 1e9
        sb = whisper_step_bytes(cfg, len(shard[0]), len(om.PROMPT[cfg.n_vocab]), N_NEW)
        step_ach = sb["total"] / (st["us"] * 1e-6) / 1e9
        step_line = {"bound": "hbm", "achieved": step_ach, "peak": peak, "unit": "GB/s", "frac": step_ach / peak,
                     "step_us": st["us"], "algorithmic_bytes": sb,
                     "how": "one decode step of the batch-8 graph (32 layers + logits head + argmax): rank 0's "
                            "(generate 224 - generate 32) / 192 steps, CUDA events; bytes = every decoder weight "
                            "once + all cross K/V + self K/V at the mean cache length"}
        job_audio = sum(lens_all) / 16000.0
        line = {
            "metric": RTFX_METRIC, "value": timed_audio / dev_s, "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_s / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q4_K x q8_K int dot (f32 accumulate), fp16 tensor-core conv/attention, f16 KV",
            "data": "synthetic (seeded N(0,0.02) Q4_K weights, -20 dBFS Gaussian-noise audio, lengths U[5,30] s)",
            "config": {"workload": "configs[3] model (whisper-large-v3-shaped Q4_K, 32+32 layers, d 1280, vocab 51866) on "
                                   "configs[4]'s 512-utterance job sharded round-robin over the GPUs, batch 8 per GPU, "
                                   "greedy 224 tokens, mel+encoder+decoder on device; a step = one batch of 8 per GPU",
                       "batch_per_gpu": B, "utterances_per_step": B * world, "new_tokens": N_NEW,
                       "l2": "inputs larger than L2 (1.97 GB cross-K/V + 0.48 GB weights per decode step)",
                       "parallelism": f"independent replicas x{world} (utterances sharded round-robin per GPU)",
                       "setup_s": round(t_setup, 1)},
            "job": None if args.no_job else {
                "utterances": JOB_UTTS, "audio_s": job_audio, "utterances_per_gpu": len(shard) * B,
                "wall_s": max(job_times), "value": job_audio / max(job_times), "unit": "audio-s/s",
                "per_gpu_s": job_times, "imbalance": max(job_times) / min(job_times),
                "rank0_serve": {"steps": job_stats.steps, "admissions": job_stats.admissions,
                                "width_changes": job_stats.width_changes, "max_width": job_stats.max_width,
                                "tokens": job_tokens},
                "how": "every rank serves its whole round-robin shard once through oasr_b200_whisper_serve "
                       "(continuous batching, max width 8, greedy up to 224 tokens or EOT, pinned host PCM in and "
                       "host tokens out inside the timed region; CUDA events); RTFx = the job's audio / the "
                       "slowest rank's time"},
            "e2e": {"value": timed_audio / e2e_s, "unit": "audio-s/s",
                    "h2d_bytes_per_step": int(np.mean([pcm_host[i % nb].nbytes
                                                       for i in range(args.warmup, args.warmup + args.steps)])),
                    "d2h_bytes_per_step": B * N_NEW * 4},
            "gpu_launches": args.steps * launches_per_batch(32, 32, 4, N_NEW, B),
            "roofline": {"bound": "hbm", "kernel": "fattn_heads_kernel (cross-attention decode, 8 x 20 heads x 1500 "
                                                   "f16 K/V)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": ncu_traffic_fa(), "algorithmic_bytes": fa["bytes"],
                         "avg_launch_us": fa["us"], "how": "same kernel and shapes timed alone on the bench stream "
                                                           "after the timed region from a CUDA graph of 20 launches, "
                                                           "K/V rotated over 246 MB",
                         "step": step_line},
            "clocks": clocks,
        }
        if world == 1 and not args.no_job:
            cb = rtfx_cpu_sample()
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    model.close()
    be.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def ncu_traffic_fa(summary: str = "fattn_heads_cross_b8.md") -> float | None:
    """dram read + write bytes of one attention launch, from a committed ncu summary
    (the cross-attention's by default)."""
    p = os.path.join(ROOT, "profiles", summary)
    try:
        for line in open(p):
            if line.startswith("| dram_bytes_per_launch |"):
                return float(line.split("|")[2])
    except (OSError, ValueError):
        return None
    return None


def run_profile_case(args) -> None:
    """The small fixed cases the committed ncu captures of the model-internal kernels use:
    each kernel at the RTFx / configs[2] workloads' own per-layer shapes, depth cut to 2
    layers so the device holds about 1 GB.
      --case whisper    whisper-large-v3-shaped Q4_K (2 + 2 layers, batch 8, 30 s clips)
                        transcribing 8 tokens: conv stem gemm_f16_tc, encoder,
                        ln_quant_chunks / gelu_quant_chunks, the fused decoder GEMVs
                        (dgemv_kernel), cross- and self-attention, the Q8_0 logits head
                        (mmv_q80_tc, the first launch of that kernel) and argmax_chunks
      --case qwen_q8_0  Qwen3-ASR-0.6B-shaped (2 layers, batch 8, 390-frame prompt)
                        generating 8 tokens: qwen_qkv_post, swiglu_quant_chunks, the
                        151936-row logits head (mmv_q80_tc, first launch: the prefill's
                        last-row logits)
      --case qwen_q4_0  the same with Q4_0 linears: mmv_q8_kernel (the Q4_0 decode GEMV)"""
    import torch

    import openasr_b200 as ob
    from openasr_b200 import models as om

    torch.cuda.set_device(0)
    be = ob.Backend(0)
    out = {}
    if args.case == "whisper":
        cfg = om.WHISPER_LARGE_V3.replace(n_enc_layers=2, n_dec_layers=2, max_batch=8)
        m = om.WhisperModel(be, cfg, om.whisper_synthetic_pack(cfg, seed=0x0A5A0004))
        clips = [om.synthetic_audio(0x0A5A3000 + i, 16000 * 30) for i in range(8)]
        out["tokens"] = m.transcribe(clips, n_new=8)[:, :4].tolist()
        m.close()
    else:
        qc = om.QWEN3_ASR_0_6B.replace(n_layers=2, weight_type=ob.Q8_0 if args.case == "qwen_q8_0" else ob.Q4_0)
        q = om.QwenModel(be, qc, om.qwen_synthetic_pack(qc))
        emb = ob.synth_normal(0x0A5A3100, 8 * om.QWEN_PREFIX_FRAMES * qc.d_model, 0.0, 0.02).reshape(
            8, om.QWEN_PREFIX_FRAMES, qc.d_model)
        out["tokens"] = q.generate(emb, n_new=8)[:, :4].tolist()
        q.close()
    be.synchronize()
    be.close()
    print(json.dumps({"workload": "profile", "case": args.case, **out}), flush=True)


def run_kernels(args) -> None:
    """Per-kernel roofline table at the RTFx workload's own shapes (whisper-large-v3,
    batch 8 per GPU), each op timed alone with CUDA events on the launching stream:
    decode GEMVs (Q4_K, M = 8, rotated over 12 layers' weights = 155 MB > L2), the
    Q8_0 logits head (two copies, 141 MB), cross- and self-attention flash-decode,
    the encoder's Q4_K tensor-core GEMMs (M = 12000) and the encoder flash attention
    (8 x 20 heads x 1500 x 1500); then the Qwen decode GEMVs, GQA decode
    attention and causal prompt attention at batch 8.  Also the small, fixed command the
    committed ncu captures use."""
    import torch

    import openasr_b200 as ob

    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    be = ob.Backend(0)
    be.set_stream(stream)
    peak_hbm, hbm_kind = measured_peak_hbm()
    peak_tc, tc_kind = measured_peak_tensor()
    B, d, ffn, T, H = 8, 1280, 5120, 1500, 20
    rows = []

    def gemv_name(fam):
        dp4a = os.environ.get("OASR_B200_DECODE_GEMV") == "dp4a"
        if fam == "q4k":
            return "mmv_q4k_kernel (dp4a)" if dp4a else "mmv_q4k_tc_kernel (mma.sync s8)"
        return "mmv_q8_kernel (dp4a)" if dp4a else "mmv_q80_tc_kernel (mma.sync s8)"

    def timed(fn, iters):
        return graph_timed(torch, stream, fn, iters)

    def add(name, shape, us, amount, unit):
        if unit == "GB/s":
            ach, pk, kind = amount / (us * 1e-6) / 1e9, peak_hbm, hbm_kind
        else:
            ach, pk, kind = amount / (us * 1e-6) / 1e12, peak_tc, tc_kind
        rows.append({"kernel": name, "shape": shape, "us": round(us, 2), "achieved": round(ach, 1), "unit": unit,
                     "peak": pk, "peak_kind": kind, "frac": round(ach / pk, 4)})

    with torch.cuda.stream(stream):
        # decode GEMVs: one weight per role and layer, activations pre-quantized (q8_K)
        n_rot = 12
        roles = [("qkv", d, 3 * d), ("o", d, d), ("cross_q", d, d), ("cross_o", d, d), ("fc1", d, ffn),
                 ("fc2", ffn, d)]
        for role, K, N in roles:
            ws = [be.upload_weight(ob.quantize(ob.Q4_K, ob.synth_normal(0xD0 + 97 * j + N + K, N * K, 0.0, 0.02)
                                               .reshape(N, K)), ob.Q4_K, [K, N]) for j in range(n_rot)]
            x = torch.randn(B, K, device="cuda")
            qa = torch.empty(be.act_bytes(ob.Q4_K, K, B), dtype=torch.uint8, device="cuda")
            be.quantize_act(ob.Q4_K, x, qa)
            y = torch.empty(B, N, device="cuda")
            us = timed(lambda i: be.mul_mat_qact(ws[i % n_rot], qa, B, y), 48)
            add(gemv_name("q4k"), f"{role} Q4_K N={N} K={K} M={B}", us, N * K * 144 / 256 + B * K + B * N * 4, "GB/s")
            del ws
        # logits head (Q8_0, tied token embedding)
        V = 51866
        lm = [be.upload_weight(ob.quantize(ob.Q8_0, ob.synth_normal(0xE0 + j, V * d, 0.0, 0.02).reshape(V, d)),
                               ob.Q8_0, [d, V]) for j in range(2)]
        x = torch.randn(B, d, device="cuda")
        qa = torch.empty(be.act_bytes(ob.Q8_0, d, B), dtype=torch.uint8, device="cuda")
        be.quantize_act(ob.Q8_0, x, qa)
        y = torch.empty(B, V, device="cuda")
        us = timed(lambda i: be.mul_mat_qact(lm[i % 2], qa, B, y), 20)
        add(gemv_name("q80"), f"logits Q8_0 N={V} K={d} M={B}", us, V * d * 34 / 32 + B * d + B * V * 4, "GB/s")
        del lm
        # cross-attention flash-decode (the dominant decode kernel)
        fa = _fa_roofline(be, torch, stream)
        add("fattn_heads_kernel", f"cross S={B} H={H} n_kv={T} D=64 f16 K/V", fa["us"], fa["bytes"], "GB/s")
        # self-attention flash-decode at position 128 of the 448-slot cache
        P, nkv = 448, 128
        kc = torch.randn(B, P, d, device="cuda").half()
        vc = torch.randn(B, P, d, device="cuda").half()
        kv = kc[:, :nkv].reshape(B, nkv, H, 64).permute(0, 2, 1, 3)
        vv = vc[:, :nkv].reshape(B, nkv, H, 64).permute(0, 2, 1, 3)
        q = torch.randn(B, 1, H, 64, device="cuda").permute(0, 2, 1, 3)
        o = torch.empty(B, 1, H, 64, device="cuda")
        us = timed(lambda i: be.flash_attn_ext(q, kv, vv, None, 0.125, o), 50)
        add("fattn_heads_kernel", f"self S={B} H={H} n_kv={nkv} D=64 f16 K/V", us, 2 * B * nkv * d * 2 + 2 * B * d * 4,
            "GB/s")
        del kc, vc
        # encoder GEMMs: Q4_K weights x q8_K activations on the tensor cores, M = 8 x 1500
        Menc = B * T
        for role, K, N in [("qkv", d, 3 * d), ("o", d, d), ("fc1", d, ffn), ("fc2", ffn, d)]:
            w = be.upload_weight(ob.quantize(ob.Q4_K, ob.synth_normal(0xF0 + N + K, N * K, 0.0, 0.02).reshape(N, K)),
                                 ob.Q4_K, [K, N])
            x = torch.randn(Menc, K, device="cuda")
            qa = torch.empty(be.act_bytes(ob.Q4_K, K, Menc), dtype=torch.uint8, device="cuda")
            be.quantize_act(ob.Q4_K, x, qa)
            y = torch.empty(Menc, N, device="cuda")
            us = timed(lambda i: be.mul_mat_qact(w, qa, Menc, y), 10)
            add("mmq_q4k_tc_kernel", f"encoder {role} Q4_K N={N} K={K} M={Menc}", us, 2.0 * Menc * N * K, "TFLOP/s")
            del w, x, qa, y
        # Q8_0 prefill GEMMs on tcgen05 kind::i8 (configs[1] shapes at M = 1500)
        for N, K in [(4096, 1024), (6144, 1024), (1024, 3072)]:
            Mp = 1500
            w = be.upload_weight(ob.quantize(ob.Q8_0, ob.synth_normal(0xF8 + N + K, N * K, 0.0, 0.02).reshape(N, K)),
                                 ob.Q8_0, [K, N])
            x = torch.randn(Mp, K, device="cuda")
            qa = torch.empty(be.act_bytes(ob.Q8_0, K, Mp), dtype=torch.uint8, device="cuda")
            be.quantize_act(ob.Q8_0, x, qa)
            y = torch.empty(Mp, N, device="cuda")
            us = timed(lambda i: be.mul_mat_qact(w, qa, Mp, y), 10)
            add("mmq_q80_tc_kernel", f"prefill Q8_0 N={N} K={K} M={Mp}", us, 2.0 * Mp * N * K, "TFLOP/s")
            del w, x, qa, y
        # Q4_0 on the same kernel (its nibbles expanded to int8 at upload), one configs[1] shape
        N, K, Mp = 4096, 1024, 1500
        w = be.upload_weight(ob.quantize(ob.Q4_0, ob.synth_normal(0xF4 + N + K, N * K, 0.0, 0.02).reshape(N, K)),
                             ob.Q4_0, [K, N])
        x = torch.randn(Mp, K, device="cuda")
        qa = torch.empty(be.act_bytes(ob.Q4_0, K, Mp), dtype=torch.uint8, device="cuda")
        be.quantize_act(ob.Q4_0, x, qa)
        y = torch.empty(Mp, N, device="cuda")
        us = timed(lambda i: be.mul_mat_qact(w, qa, Mp, y), 10)
        add("mmq_q80_tc_kernel (Q4_0 expanded)", f"prefill Q4_0 N={N} K={K} M={Mp}", us, 2.0 * Mp * N * K, "TFLOP/s")
        del w, x, qa, y
        # encoder self-attention: f16 pre-pass + tcgen05 flash attention
        qkv = torch.randn(B, T, 3 * d, device="cuda")
        qe = qkv[:, :, :d].reshape(B, T, H, 64).permute(0, 2, 1, 3)
        ke = qkv[:, :, d:2 * d].reshape(B, T, H, 64).permute(0, 2, 1, 3).half()
        ve = qkv[:, :, 2 * d:].reshape(B, T, H, 64).permute(0, 2, 1, 3).half()
        oe = torch.empty(B, T, H, 64, device="cuda")
        us = timed(lambda i: be.flash_attn_ext(qe, ke, ve, None, 0.125, oe), 10)
        add("fa_prep_tile_kernel+fattn_tc_kernel", f"encoder S={B} H={H} {T}x{T} D=64", us, 4.0 * B * H * T * T * 64,
            "TFLOP/s")
        del qkv
        # Qwen3-ASR-0.6B decode (configs[2], batch 8): Q8_0 GEMVs rotated over 4 layers' weights
        for role, N, K in [("qwen qkv", 4096, 1024), ("qwen gate|up", 6144, 1024), ("qwen down", 1024, 3072),
                           ("qwen o", 1024, 2048), ("qwen lm_head", 151936, 1024)]:
            n_rot = 2 if N > 100000 else 4
            ws = [be.upload_weight(ob.quantize(ob.Q8_0, ob.synth_normal(0x100 + 16 * j + N + K, N * K, 0.0, 0.02)
                                               .reshape(N, K)), ob.Q8_0, [K, N]) for j in range(n_rot)]
            x = torch.randn(B, K, device="cuda")
            qa = torch.empty(be.act_bytes(ob.Q8_0, K, B), dtype=torch.uint8, device="cuda")
            be.quantize_act(ob.Q8_0, x, qa)
            y = torch.empty(B, N, device="cuda")
            us = timed(lambda i: be.mul_mat_qact(ws[i % n_rot], qa, B, y), 20 if N > 100000 else 48)
            add(gemv_name("q80"), f"{role} Q8_0 N={N} K={K} M={B}", us, N * K * 34 / 32 + B * K + B * N * 4, "GB/s")
            del ws
        # Qwen GQA decode attention at the mid-generation KV length
        fq = _qwen_fa_roofline(be, torch, stream, B, 390 + 128)
        add("fattn_gqa_kernel<2>", f"qwen decode S={B} H=16 HKV=8 n_kv={fq['n_kv']} D=128", fq["us"], fq["bytes"],
            "GB/s")
        # Qwen causal prompt attention on the tensor cores (8 x 390 rows, GQA, D 128)
        Tq = 390
        qq = torch.randn(B, 16, Tq, 128, device="cuda")
        kq = torch.randn(B, 8, Tq, 128, device="cuda").half()
        vq = torch.randn(B, 8, Tq, 128, device="cuda").half()
        oq = torch.empty(B, Tq, 16, 128, device="cuda")
        us = timed(lambda i: be.flash_attn_causal(qq, kq, vq, 1.0 / float(np.sqrt(128.0)), oq), 10)
        add("fa_prep_tile_kernel+fattn_tc_kernel<128,causal>", f"qwen prompt S={B} H=16 HKV=8 {Tq}x{Tq} D=128", us,
            2.0 * B * 16 * Tq * (Tq + 1) * 128, "TFLOP/s")
    # resident weight upload (raw pack bytes from pageable host memory through the pinned
    # staging ring, plane split, decode tiles and scale copies built on the device): the
    # Qwen lm_head shape, 165 MB of Q8_0 blocks; wall time of the synchronous call
    import time
    raw = np.random.default_rng(5).integers(0, 256, (151936, 1024 // 32 * 34), dtype=np.uint8)
    best = float("inf")
    for _ in range(3):
        t0 = time.perf_counter()
        w = be.upload_weight(raw, ob.Q8_0, [1024, 151936])
        best = min(best, time.perf_counter() - t0)
        w.free()
    rows.append({"kernel": "oasr_b200_weight_upload (staged H2D + split_blocks_kernel + tile build)",
                 "shape": "Q8_0 151936x1024 (165.3 MB raw)", "us": round(best * 1e6, 1),
                 "achieved": round(raw.nbytes / best / 1e9, 2), "unit": "GB/s host->device (raw bytes / wall time)",
                 "peak": None, "peak_kind": None, "frac": None})
    print(json.dumps({"workload": "kernels", "n_gpus": 1, "kernels": rows}), flush=True)
    be.close()


# ==================================================================================
# Qwen workload (--workload qwen)
# ==================================================================================
QWEN_METRIC = "RTFx (audio-s/s), Qwen3-ASR-0.6B-shaped Q8_0 decoder, 390-frame prompt, greedy 256 tokens"
QWEN_NEW = 256
QWEN_SEED = 0x0A5A0003


def qwen_launches_per_batch(n_layers: int, n_new: int, n_tok: int = 390) -> int:
    """Kernel launches of one oasr_b200_qwen_generate (counted from model_qwen.cu):
    prefill = first RMSNorm + per layer (q|k|v, o, gate|up and down GEMMs, q/k-norm +
    RoPE + KV write, attention, quantize, RMSNorm, SwiGLU = 10; the tensor-core attention
    of 64+ rows adds its 3 f16 staging kernels) less the last layer's trailing RMSNorm +
    head (RMSNorm, logits, argmax) + 1 advance; decode step = embed + RMSNorm + 9 per
    layer + logits + argmax + advance (equal to the committed launch list); the causal
    mask is built once per prompt length."""
    attn_extra = 3 if n_tok >= 64 else 0
    prefill = 1 + (10 + attn_extra) * n_layers - 1 + 3 + 1
    step = 2 + 9 * n_layers + 3
    return prefill + (n_new - 1) * step


def qwen_cpu_baseline() -> dict:
    """The oracle (CPU restatement) on a bounded sample: the full-width decoder at 1 and
    2 layers, the 390-frame prefill and 2 decode steps of one sequence, extrapolated
    linearly in layers to 28 and in steps to 255."""
    from oracle import oracle as oo
    from oracle import qwen_ref as qr
    from openasr_b200 import models as om

    cores = os.cpu_count() or 1
    emb = om.qwen_synthetic_prefix(0x0A5A3700, 1, om.QWEN_PREFIX_FRAMES, 1024)[0]
    times = {}
    for L in (1, 2):
        cfg = om.QWEN3_ASR_0_6B.replace(n_layers=L, max_batch=1, max_prefill=om.QWEN_PREFIX_FRAMES)
        ref = qr.QwenRef(cfg, om.qwen_synthetic_pack(cfg, seed=QWEN_SEED, synth=oo.synth_normal, quantize=oo.quantize))
        cache = ref.new_cache(1)
        t0 = time.perf_counter()
        tok = int(oo.argmax_first(ref.prefill(emb, cache))[0])
        t1 = time.perf_counter()
        for i in range(2):
            tok = int(oo.argmax_first(ref.step([tok], om.QWEN_PREFIX_FRAMES + i, cache)[0])[0])
        t2 = time.perf_counter()
        times[L] = (t1 - t0, (t2 - t1) / 2)
    pre_layer = times[2][0] - times[1][0]
    step_layer = times[2][1] - times[1][1]
    pre = times[1][0] - pre_layer + 28 * pre_layer
    step = times[1][1] - step_layer + 28 * step_layer
    per_seq = pre + (QWEN_NEW - 1) * step
    return {"value": om.QWEN_PREFIX_SECONDS / per_seq, "unit": "audio-s/s", "cores": cores, "kind": "port",
            "sample": (f"oracle (CPU restatement of ggml semantics, OpenMP {cores} threads) on the full-width decoder "
                       f"at 1 and 2 layers: 390-frame prefill {times[1][0]:.2f}/{times[2][0]:.2f} s, decode step "
                       f"{times[1][1]:.3f}/{times[2][1]:.3f} s; extrapolated to 28 layers and 255 steps = "
                       f"{per_seq:.1f} s per sequence (30 s of audio)")}


def run_reference_qwen(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cb = qwen_cpu_baseline()
    v = cb["value"]
    print(json.dumps({
        "impl": "reference", "metric": QWEN_METRIC, "value": v, "unit": "audio-s/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": args.batch * 30.0 / v * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q8_0 x q8_0 int dot, f32 accumulate; f16 KV",
        "data": "synthetic (seeded N(0,0.02) Q8_0 weights, N(0,1) 390-frame prompt embeddings)",
        "config": {"workload": f"configs[2]: qwen3-asr-0.6b-shaped decoder, batch {args.batch}, 390-frame prompt, "
                               f"greedy {QWEN_NEW} tokens", "l2": "inputs larger than L2"},
        "cpu_baseline": cb,
        "e2e": {"value": v, "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def _qwen_fa_roofline(be, torch, stream, S: int, n_kv: int, n_rot: int = 8, iters: int = 40) -> dict:
    """The decode step's attention (fattn_gqa_kernel<2>: GQA 16 q / 8 kv heads, D 128) over
    the mid-generation KV length, through the public flash_attn_ext entry point on views
    of the model's cache layout [seq][kv head][max_pos][128], timed alone on the bench
    stream from a CUDA graph of `iters` launches, rotating over 8 layers' caches (> L2)."""
    P, HKV, H, D = 2048, 8, 16, 128
    caches = [(torch.randn(S, HKV, P, D, device="cuda").half(), torch.randn(S, HKV, P, D, device="cuda").half())
              for _ in range(n_rot)]
    q = torch.randn(S, H, 1, D, device="cuda")
    out = torch.empty(S, 1, H, D, device="cuda")
    scale = 1.0 / float(np.sqrt(np.float32(D)))

    def launch(i):
        k, v = caches[i % n_rot]
        be.flash_attn_ext(q, k[:, :, :n_kv], v[:, :, :n_kv], None, scale, out)

    us = graph_timed(torch, stream, launch, iters)
    return {"us": us, "bytes": S * HKV * n_kv * D * 2 * 2 + 2 * S * H * D * 4, "n_kv": n_kv}


def run_b200_qwen(args) -> None:
    import torch
    import torch.distributed as dist

    import openasr_b200 as ob
    from openasr_b200 import models as om

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    init_ranks(world)
    B, T, NEW = args.batch, om.QWEN_PREFIX_FRAMES, args.new_tokens
    cfg = om.QWEN3_ASR_0_6B.replace(max_batch=B, max_prefill=T)
    t_setup = time.perf_counter()
    stream = torch.cuda.Stream()
    be = ob.Backend(local)
    be.set_stream(stream)
    model = om.QwenModel(be, cfg, om.qwen_synthetic_pack(cfg, seed=QWEN_SEED))
    t_setup = time.perf_counter() - t_setup
    n_steps = args.warmup + args.steps
    emb_host = [om.qwen_synthetic_prefix(0x0A5A3700 + 1000 * rank + i, B, T, cfg.d_model) for i in range(n_steps)]
    with torch.cuda.stream(stream):
        emb_dev = [torch.from_numpy(e).cuda() for e in emb_host]
        emb_pin = [torch.from_numpy(e).pin_memory() for e in emb_host]
        toks_dev = torch.empty((B, NEW), dtype=torch.int32, device="cuda")
        for i in range(args.warmup):
            model.generate_device(emb_dev[i], B, T, toks_dev, NEW)
        stream.synchronize()
        if world > 1:
            dist.barrier()
        sampler = ClockSampler(local)
        sampler.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(args.warmup, n_steps):
            model.generate_device(emb_dev[i], B, T, toks_dev, NEW)
        e1.record(stream)
        torch.cuda.synchronize()
        be.synchronize()
        clocks = sampler.stop()
        dev_s = e0.elapsed_time(e1) / 1e3
        # e2e: the public generate call from pinned host embeddings to host tokens
        if world > 1:
            dist.barrier()
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0.record(stream)
        for i in range(args.warmup, n_steps):
            out = np.empty((B, NEW), np.int32)
            be._check(ob.lib().oasr_b200_qwen_generate(model.handle, emb_pin[i].data_ptr(), 0, B, T, NEW,
                                                       om.QWEN_EOS, 0, out.ctypes.data, 0))
        h1.record(stream)
        torch.cuda.synchronize()
        e2e_s = h0.elapsed_time(h1) / 1e3
        fa = _qwen_fa_roofline(be, torch, stream, B, T + QWEN_NEW // 2)
        # one decode step alone: (generate NEW - generate 32) / (NEW - 32) steps, CUDA events
        qs = {}
        for n in (NEW, 32):
            model.generate_device(emb_dev[0], B, T, toks_dev, n)
            q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            q0.record(stream)
            for _ in range(3):
                model.generate_device(emb_dev[0], B, T, toks_dev, n)
            q1.record(stream)
            torch.cuda.synchronize()
            qs[n] = q0.elapsed_time(q1) / 3 * 1e3
        step_us = (qs[NEW] - qs[32]) / (NEW - 32) if NEW > 32 else None
    audio = om.QWEN_PREFIX_SECONDS * B * args.steps
    dev_s, e2e_s, audio = reduce_over_ranks(dev_s, e2e_s, audio)
    if rank == 0:
        peak, peak_kind = measured_peak_hbm()
        achieved = fa["bytes"] / (fa["us"] * 1e-6) / 1e9
        # algorithmic bytes of one decode step: every Q8_0 weight once (28 layers of q|k|v,
        # o, gate|up, down, and the tied 151936-row head; 34 B per 32 weights) + the K/V of the
        # B sequences at the mean cache length (f16, 8 kv heads x 128, K and V)
        d, L = cfg.d_model, cfg.n_layers
        kvw = cfg.n_kv_heads * cfg.head_dim
        per_layer = d * (cfg.n_heads * cfg.head_dim + 2 * kvw) + cfg.n_heads * cfg.head_dim * d + 3 * d * cfg.ffn
        wbytes = (L * per_layer + cfg.n_vocab * d) * 34 // 32
        mean_kv = T + (NEW - 1) / 2
        kvbytes = int(L * B * mean_kv * 2 * kvw * 2)
        step_line = None
        if step_us:
            sa = (wbytes + kvbytes) / (step_us * 1e-6) / 1e9
            step_line = {"bound": "hbm", "achieved": sa, "peak": peak, "unit": "GB/s", "frac": sa / peak,
                         "step_us": step_us, "algorithmic_bytes": {"weights": wbytes, "kv": kvbytes,
                                                                   "total": wbytes + kvbytes},
                         "how": f"one decode step of the batch-{B} graph (28 layers + logits head + argmax): rank "
                                f"0's (generate {NEW} - generate 32) / {NEW - 32} steps, CUDA events; bytes = every "
                                "weight once + K/V at the mean cache length"}
        tokens = B * NEW * args.steps * world
        line = {
            "metric": QWEN_METRIC.replace(f"greedy {QWEN_NEW}", f"greedy {NEW}"), "value": audio / dev_s,
            "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_s / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q8_0 x q8_0 int dot (f32 accumulate), f16 KV",
            "data": "synthetic (seeded N(0,0.02) Q8_0 weights, N(0,1) 390-frame prompt embeddings)",
            "config": {"workload": f"configs[2]: qwen3-asr-0.6b-shaped decoder (28 layers, d 1024, 16/8 heads of 128, "
                                   f"ffn 3072, vocab 151936), batch {B} per GPU, 390-frame prompt (30 s of audio), "
                                   f"greedy {NEW} tokens, prefill + decode on device",
                       "batch_per_gpu": B, "sequences_per_step": B * world, "new_tokens": NEW,
                       "tokens_per_s": tokens / dev_s,
                       "l2": "inputs larger than L2 (633 MB of Q8_0 weights per decode step)",
                       "parallelism": f"independent replicas x{world} (sequences sharded per GPU)",
                       "setup_s": round(t_setup, 1)},
            "e2e": {"value": audio / e2e_s, "unit": "audio-s/s", "h2d_bytes_per_step": int(emb_host[0].nbytes),
                    "d2h_bytes_per_step": B * NEW * 4},
            "gpu_launches": args.steps * qwen_launches_per_batch(cfg.n_layers, NEW, T),
            "roofline": {"bound": "hbm", "kernel": f"fattn_gqa_kernel<2> (GQA decode attention, {B} x 8 kv "
                                                   f"heads x {fa['n_kv']} f16 K/V positions)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind,
                         # the committed capture is of this exact shape (8 sequences, 518 positions)
                         "traffic": ncu_traffic_fa("fattn_gqa_decode_qwen_b8.md")
                         if (B, fa["n_kv"]) == (8, 518) else None,
                         "algorithmic_bytes": fa["bytes"],
                         "avg_launch_us": fa["us"], "how": "same kernel and shapes through flash_attn_ext, timed alone "
                                                           "on the bench stream from a CUDA graph of 40 launches, "
                                                           "caches rotated over 8 layers",
                         "step": step_line},
            "clocks": clocks,
        }
        line["cpu_baseline"] = qwen_cpu_baseline()
        print(json.dumps(line), flush=True)
    model.close()
    be.close()
    if world > 1:
        dist.destroy_process_group()


def measured_peak_tensor() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        j = json.load(open(p))
        return float(j["bf16_tflops"]), "measured (bf16 burst)"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["rtfx", "qwen", "mulmat", "kernels", "profile"], default="rtfx")
    ap.add_argument("--batch", type=int, default=8, help="sequences per GPU (qwen workload: 1, 4 or 8)")
    ap.add_argument("--case", choices=["whisper", "qwen_q8_0", "qwen_q4_0"], default="whisper",
                    help="profile workload: which small model case to run")
    ap.add_argument("--no-job", action="store_true",
                    help="rtfx workload: skip the 512-utterance job leg and the CPU sample (profiling runs)")
    ap.add_argument("--new-tokens", type=int, default=256,
                    help="qwen workload: greedy tokens per sequence (256 = configs[2]; fewer only to profile)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.steps is None:
        args.steps = 8 if args.workload in ("rtfx", "qwen") else 20
    if args.workload == "profile":
        run_profile_case(args)
    elif args.workload == "kernels":
        run_kernels(args)
    elif args.workload == "rtfx":
        (run_reference if args.impl == "reference" else run_b200)(args)
    elif args.workload == "qwen":
        (run_reference_qwen if args.impl == "reference" else run_b200_qwen)(args)
    elif args.impl == "reference":
        run_reference_mulmat(args)
    else:
        run_b200_mulmat(args)


if __name__ == "__main__":
    main()
