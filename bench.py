#!/usr/bin/env python3
"""Benchmark: batch-1 greedy decode of chpe-qwen-engine's forwardDecode loop.

Default workload (the configuration the metric is quoted on
at 1/2/4/8 B200): Qwen2.5-72B in the 4-bit flat-cell format (group-128 FP16
scales), random-init seeded synthetic archive, a 2048-token prompt decoded
token by token (untimed), then W warm-up and K timed greedy steps.  A step is
one token through all 80 layers + LM head.  With N > 1 (torchrun, one rank per
GPU) the model is tensor parallel over the N GPUs; `value` is tokens of the
one sequence per second (strong scaling).  --model picks another config
(3b-fp16 = config 1, 3b-w4 / 3b-w2 = config 2, 9b-w4 = config 3, 72b-fp16 =
the FP16 half of config 5); the 3B models run as independent replicas for
N > 1.  --sweep prints config 2's isolated GEMV sweep instead.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--model M] [--impl ours|reference]
  python bench.py --sweep [--model 3b-w4|3b-w2|3b-fp16]

value: tok/s with weights resident in HBM, device time (CUDA events on the
engine stream) of K back-to-back greedy steps (each step's token is the
previous argmax, fed back on the device), max over ranks.  e2e: the same steps
through the C ABI with a pinned host->device copy of each token and a
device->host copy of each step's logits and result, wall time, max over ranks.
--impl reference times the CPU restatement of the reference engine (the Zig
reference cannot be built here) on all host threads, rank 0 only, at the
GPU arm's positions over a KV cache prefilled to the same context; both arms
print the same `config`.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch-1 greedy decode tok/s (weight stream vs HBM roofline)"

# Workloads: synthetic archive, architecture preset, prompt
# length decoded before timing, and the layer count of the model.
MODELS = {
    "3b-w4": dict(synth="SYNTH_3B_W4", arch="ARCH_3B", prompt=512, name="qwen2.5-3b-w4-dense-cell",
                  dtype="u4->f32"),
    "3b-w2": dict(synth="SYNTH_3B_W2", arch="ARCH_3B", prompt=512, name="qwen2.5-3b-w2-dense-cell",
                  dtype="u2->f32"),
    "3b-fp16": dict(synth="SYNTH_3B_FP16_RAW", arch="ARCH_3B", prompt=32, name="qwen2.5-3b-fp16-raw",
                    dtype="f16->f32"),
    "9b-w4": dict(synth="SYNTH_9B_W4", arch="ARCH_9B", prompt=1024, name="qwen3.5-9b-w4-flat-cell",
                  tp=True, dtype="u4->f32"),
    "72b-w4": dict(synth="SYNTH_72B_W4", arch="ARCH_72B", prompt=2048, name="qwen2.5-72b-w4-flat-cell",
                   tp=True, dtype="u4->f32"),
    # FP16 raw tiles laid out by the 72B tensor map, whose tile counts are
    # sized for 4-bit cells: the reference reads a quarter of each projection
    "72b-fp16": dict(synth="SYNTH_72B_FP16_RAW", arch="ARCH_72B", prompt=2048,
                     name="qwen2.5-72b-fp16-raw-reference-map", tp=True, dtype="f16->f32"),
}
# layers, kv heads, head dim per architecture (KV bytes of a step)
KV_GEOM = {0: (36, 2, 128), 1: (32, 4, 256), 2: (80, 8, 128)}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


def cpu_isa() -> str:
    try:
        flags = open("/proc/cpuinfo").read()
        isa = [f for f in ("avx512f", "avx2", "amx_tile") if f" {f}" in flags]
        model = [l.split(":", 1)[1].strip() for l in flags.splitlines() if l.startswith("model name")]
        return (model[0] if model else platform.processor()) + " [" + ",".join(isa) + "]"
    except Exception:
        return platform.processor()


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        for line in (self.out or "").splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def dist_setup(n):
    if n <= 1:
        return 0, 1, 0, None
    import torch.distributed as dist
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", n))
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=600))
    return rank, world, local, dist


def max_over_ranks(dist, v: float) -> float:
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(dist, v: float) -> float:
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(dist):
    if dist is not None:
        dist.barrier()


def kv_bytes_per_step(arch: int, pos: float) -> float:
    """FP16 K and V the attention of one step at position `pos` reads
    (positions 0..pos of every layer and kv head)."""
    L, KV, HD = KV_GEOM[arch]
    return float(L * KV * HD * 2 * 2) * (pos + 1)


def common_config(M, prompt: int, warmup: int, steps: int, world: int, tp: bool) -> dict:
    """The workload both arms run (the same dict in both JSON lines)."""
    p0 = prompt + warmup
    return {"workload": M["name"], "prompt": prompt, "positions": f"{p0}..{p0 + steps - 1}",
            "parallelism": f"tp{world}" if tp else f"replicas x{world}",
            "kv": "paged FP16 (GPU), f32 (CPU); CPU context prefilled to the same length",
            "l2": "inputs larger than L2 (the weights of a step exceed 126 MB)"}


def prefilled_oracle(archive, arch: int, ctx: int, extra: int, threads: int):
    """The oracle (C restatement of the reference engine) with its KV cache
    filled at positions 0..ctx-1 by seeded rows, so its steps attend over
    the same context length as the GPU arm's."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_py as O
    e = O.OracleEngine(archive, arch, ctx + extra + 2, threads=threads)
    L, KV, HD = KV_GEOM[arch]
    rng = np.random.default_rng(5)
    for l in range(L):
        if ctx:
            e.kv_load(l, 0, rng.standard_normal((ctx, KV * HD), dtype=np.float32),
                      rng.standard_normal((ctx, KV * HD), dtype=np.float32))
    return e


def oracle_sample(archive, arch: int, pos0: int, warmup: int, max_steps: int, threads: int,
                  budget_s: float) -> tuple[float, int, int]:
    """Times oracle decode steps at positions pos0+warmup.. after `warmup`
    untimed steps, stopping after max_steps or once budget_s has passed
    (at least one step).  Returns (tok/s, steps timed, first timed position)."""
    e = prefilled_oracle(archive, arch, pos0, warmup + max_steps, threads)
    toks = np.random.default_rng(1).integers(0, 151936, warmup + max_steps + 1)
    for i in range(warmup):
        e.forward_decode(int(toks[i]), pos0 + i)
    p = pos0 + warmup
    n = 0
    t0 = time.perf_counter()
    while n < max_steps:
        e.forward_decode(int(toks[warmup + n]), p + n)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    e.close()
    return n / dt, n, p


def run_reference(args, rank, world, dist):
    import chpe_qwen_engine_b200 as chpe
    if rank != 0:
        return
    M = MODELS[args.model]
    tp = world > 1 and M.get("tp", False)
    archive = chpe.synth_archive(getattr(chpe, M["synth"]), 0, seed=0)
    arch = getattr(chpe, M["arch"])
    threads = os.cpu_count() or 1
    # the GPU arm's positions: the prompt, then its warm-up steps, then the
    # timed steps; the CPU warms up on one step and times up to K within ~90 s
    v, n, p = oracle_sample(archive, arch, args.prompt + args.warmup - 1, 1, args.steps, threads, 90.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": n, "warmup": args.warmup, "ms_per_step": 1000.0 / v,
        "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
        "dtype": M["dtype"], "data": "synthetic (seeded archive, random-init weights)",
        "config": common_config(M, args.prompt, args.warmup, args.steps, world, tp),
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{n} decode steps at positions {p}..{p + n - 1} over a KV cache "
                                   f"prefilled to the same context as the GPU arm; CPU restatement of "
                                   f"src/chpe_engine.zig, rows split over {threads} threads "
                                   f"(the reference itself is single-threaded) ({cpu_isa()})"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


class nvtx_range:
    """An NVTX range around the timed steps (a profiler can restrict its
    capture to it: ncu --nvtx --nvtx-include "chpe_timed/")."""

    def __init__(self, name: str):
        self.name = name

    def __enter__(self):
        try:
            import torch
            torch.cuda.nvtx.range_push(self.name)
            self.pushed = True
        except Exception:
            self.pushed = False
        return self

    def __exit__(self, *exc):
        if self.pushed:
            import torch
            torch.cuda.nvtx.range_pop()
        return False


def shared_archive_path(chpe, cfg: int, rank: int, dist) -> str:
    """Rank 0 writes the seeded archive once to a local file that every rank
    maps read-only (one copy in the page cache, not one per rank)."""
    import shutil
    import tempfile
    need = chpe.synth_lib().chpe_synth_bytes(cfg, 0) + (1 << 30)
    dirs = [d for d in ("/dev/shm", tempfile.gettempdir(), ROOT) if os.path.isdir(d)]
    dirs = [d for d in dirs if shutil.disk_usage(d).free > need] or [ROOT]
    path = os.path.join(dirs[0], f"chpe_bench_{cfg}.chpe")
    if rank == 0 and not (os.path.exists(path) and os.path.getsize(path) == need - (1 << 30)):
        chpe.synth_write(path, cfg, 0, seed=0)
    barrier(dist)
    return path


def run_ours(args, rank, world, local, dist):
    import chpe_qwen_engine_b200 as chpe
    M = MODELS[args.model]
    dev = local if world > 1 else 0
    cfg = getattr(chpe, M["synth"])
    arch = getattr(chpe, M["arch"])
    max_seq = args.prompt + args.warmup + 2 * args.steps + 64
    tp = world > 1 and M.get("tp", False)
    if tp:
        # tensor parallel: rank r of `world` GPUs over one shared archive file
        path = shared_archive_path(chpe, cfg, rank, dist)
        archive = None
        eng = chpe.Engine.tensor_parallel(path, arch, rank, world, max_seq_len=max_seq, device=dev)
    else:
        archive = chpe.synth_archive(cfg, 0, seed=0)
        eng = chpe.Engine.from_bytes(archive, arch, max_seq_len=max_seq, device=dev)
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, 151936, args.prompt).astype(np.uint32)
    eng.forward_tokens(prompt)  # positions 0..prompt-1, untimed
    eng.bench_greedy(args.warmup)  # warm-up steps
    barrier(dist)
    with ClockSampler(dev) as cs, nvtx_range("chpe_timed"):
        ms = eng.bench_greedy(args.steps)
    barrier(dist)
    ms_max = max_over_ranks(dist, ms)
    # replicas decode `world` independent streams; tensor parallel decodes one
    value = (1 if tp else world) * args.steps / (ms_max / 1000.0)

    # e2e through the C ABI with host buffers
    host_toks = rng.integers(0, 151936, args.steps).astype(np.uint32)
    eng.forward_tokens(prompt)
    barrier(dist)
    wall_ms, _ = eng.bench_host(host_toks)
    wall_ms = max_over_ranks(dist, wall_ms)
    e2e = (1 if tp else world) * args.steps / (wall_ms / 1000.0)

    hbm, peak_kind = peaks()
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tf):
        traffic = json.load(open(tf)).get(f"gateup_{args.model}_bytes_per_launch")
    per_role = {}
    step_bytes = 0.0
    if not tp:
        # whole-step algorithmic bytes (all roles)
        for role, name in ((chpe.ROLE_QKV, "qkv"), (chpe.ROLE_ATTN, "attention"), (chpe.ROLE_O, "o"),
                           (chpe.ROLE_GATEUP, "gateup"), (chpe.ROLE_DOWN, "down"),
                           (chpe.ROLE_LMHEAD, "lmhead")):
            m, b, n = eng.bench_kernel(role, rounds=2)
            launches_per_step = n // 2
            step_bytes += b * launches_per_step
            per_role[name] = {"avg_us": round(m * 1000, 2), "launches_per_step": launches_per_step,
                              "bytes_per_launch": b,
                              "gbs": round(b / (m / 1000) / 1e9, 1) if b else None}
        # roofline of the dominant kernel (fused RMSNorm + gate/up + SwiGLU
        # GEMV): every layer's launch, 4 rounds, after the roles above warmed
        # the clocks
        kms, kbytes, klaunch = eng.bench_kernel(chpe.ROLE_GATEUP, rounds=4)
        achieved = kbytes / (kms / 1000.0) / 1e9
        roof = {"kernel": eng.op_kernel_name(chpe.ROLE_GATEUP) + " fused RMSNorm+gate/up+SwiGLU",
                "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "peak_kind": peak_kind, "traffic": traffic, "bytes_per_launch": kbytes,
                "avg_launch_us": kms * 1000}
    # Per-role device time inside whole steps launched op by op with CUDA
    # events between the ops (no graph, no overlap between kernels; with
    # tensor parallelism every rank together, max over ranks).
    names = {chpe.ROLE_QKV: "qkv", chpe.ROLE_ATTN: "attention", chpe.ROLE_O: "o",
             chpe.ROLE_GATEUP: "gateup", chpe.ROLE_DOWN: "down", chpe.ROLE_LMHEAD: "lmhead"}
    acc = {}
    reps = 3
    for _ in range(reps):
        ms_ops, roles = eng.profile_step()
        for m, r in zip(ms_ops, roles):
            if int(r) in names:
                a = acc.setdefault(names[int(r)], [0.0, 0])
                a[0] += float(m)
                a[1] += 1
    per_role_step = {name: round(max_over_ranks(dist, tot / cnt) * 1000, 2) for name, (tot, cnt) in acc.items()}
    ms_step = ms_max / args.steps
    if tp:
        # one role cannot run alone across ranks (its exchanges wait on the
        # others): the roofline here is the whole step's weight stream per GPU
        for name, us in per_role_step.items():
            per_role[name] = {"avg_us": us, "launches_per_step": acc[name][1] // reps,
                              "bytes_per_launch": None, "gbs": None}
        mine = eng.step_weight_bytes()
        step_bytes = sum_over_ranks(dist, mine)
        per_gpu = max_over_ranks(dist, mine) / (ms_step / 1000.0) / 1e9
        roof = {"kernel": "whole decode step per GPU (all kernels, exchanges included)", "bound": "hbm",
                "achieved": per_gpu, "peak": hbm, "unit": "GB/s", "frac": per_gpu / hbm,
                "peak_kind": peak_kind, "traffic": None, "bytes_per_launch": step_bytes / world,
                "avg_launch_us": ms_step * 1000}
    # KV read by the timed steps (their average position), FP16
    p0 = args.prompt + args.warmup
    kvb = kv_bytes_per_step(arch, p0 + (args.steps - 1) / 2.0)
    cpu = None
    if rank == 0 and archive is None:
        archive = np.memmap(path, dtype=np.uint8, mode="r")
    if rank == 0:
        # a bounded sample (~25 s) of the same workload on the host: the oracle
        # at the timed positions over a KV cache prefilled to the same context
        threads = os.cpu_count() or 1
        v_cpu, n_cpu, p_cpu = oracle_sample(archive, arch, p0 - 1, 1, 8, threads, 25.0)
        cpu = {"value": v_cpu, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{n_cpu} decode steps at positions {p_cpu}..{p_cpu + n_cpu - 1} over a KV "
                         f"cache prefilled to the same context; CPU restatement of src/chpe_engine.zig, "
                         f"rows split over {threads} threads (the reference is single-threaded) "
                         f"({cpu_isa()})"}
    if rank != 0:
        return
    total = step_bytes + kvb
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": M["dtype"],
        "data": "synthetic (seeded archive, random-init weights)",
        "config": common_config(M, args.prompt, args.warmup, args.steps, world, tp),
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": eng.vocab * 4 + 24},
        "roofline": roof,
        "cpu_baseline": cpu,
        "clocks": cs.summary(),
        "gpu_launches": eng.kernels_per_step() * args.steps,
        "detail": {
            "algorithmic_bytes_per_token": total,
            "weight_bytes_per_token": step_bytes,
            "kv_bytes_per_token": kvb,
            "step_gbs": total / (ms_step / 1000) / 1e9,
            "step_frac_of_measured_hbm": total / (ms_step / 1000) / 1e9 / hbm / (world if tp else 1),
            "weight_stream_gbs": step_bytes / (ms_step / 1000) / 1e9,
            "per_role": per_role,
            "per_role_in_step_us": per_role_step,
        },
    }
    print(json.dumps(line), flush=True)


def run_verify(args):
    """Config 4: Qwen3.5-9B 4-bit batch-M speculative verification against a
    2048-token context (the prompt decoded first).  Each timed call scores M
    candidates at the same position (rolling back between calls), through the
    batched tcgen05 step and, for comparison, as M sequential decode steps;
    one greedy decode step is timed at the same position."""
    import chpe_qwen_engine_b200 as chpe
    M = args.verify
    ctx = args.prompt if args.prompt_given else 2048
    a = chpe.synth_archive(chpe.SYNTH_9B_W4, 0, seed=0)
    eng = chpe.Engine.from_bytes(a, chpe.ARCH_9B, ctx + 2 * args.steps + 64)
    rng = np.random.default_rng(1)
    eng.forward_tokens(rng.integers(0, 151936, ctx).astype(np.uint32))
    cand = rng.integers(0, 151936, M).astype(np.uint32)

    def timed(n):
        for _ in range(args.warmup):
            eng.verify(cand, ctx)
        t0 = time.perf_counter()
        for _ in range(n):
            eng.verify(cand, ctx)
        return (time.perf_counter() - t0) / n

    with ClockSampler(0) as cs:
        t_batched = timed(args.steps)
        batched = eng.last_verify_batched()
        os.environ["CHPE_VERIFY_BATCHED"] = "0"
        t_seq = timed(max(1, args.steps // 2))
        del os.environ["CHPE_VERIFY_BATCHED"]
    # per-role device time of the batched step, ops launched one by one
    ms_role, by_role = eng.profile_verify(M, ctx)
    hbm, _ = peaks()
    names = ["other", "qkv", "attention", "o", "gateup", "down", "lmhead", "embed"]
    roles = {names[i]: {"ms": round(float(ms_role[i]), 4),
                        "gbs": round(by_role[i] / (ms_role[i] / 1000) / 1e9, 1) if by_role[i] else None}
             for i in range(8) if ms_role[i] > 0}
    wbytes = float(by_role.sum())
    eng.forward_decode(int(cand[0]), ctx)  # sets the graph position
    ms1 = eng.bench_greedy(args.steps) / args.steps
    print(json.dumps({
        "metric": f"batch-{M} speculative verify: candidate tokens scored per second", "unit": "tok/s",
        "value": M / t_batched, "impl": "ours", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "batched_tensor_core_path": batched,
        "why_not_batched": "" if batched else eng.verify_batched_unavailable(M),
        "ms_per_verify": t_batched * 1000, "ms_per_verify_sequential": t_seq * 1000,
        "ms_per_decode_step": ms1, "verify_over_decode_step": t_batched * 1000 / ms1,
        "timing": "wall time of chpe_verify calls (host round trip included); decode step: CUDA events",
        "batched_step_per_role": roles, "batched_step_weight_bytes": wbytes,
        "batched_step_ops_ms": float(ms_role.sum()),
        "batched_step_weight_frac_of_measured_hbm": wbytes / (float(ms_role.sum()) / 1000) / 1e9 / hbm,
        "config": {"workload": "qwen3.5-9b-w4-flat-cell", "context": ctx, "candidates": M},
        "clocks": cs.summary()}), flush=True)


def run_sweep(args):
    """Config 2's isolated GEMV sweep on the 3B dense-cell archive: every
    launch of a role (one per layer) timed alone from a cold L2."""
    import chpe_qwen_engine_b200 as chpe
    M = MODELS[args.model]
    arch = getattr(chpe, M["arch"])
    eng = chpe.Engine.from_bytes(chpe.synth_archive(getattr(chpe, M["synth"]), 0, seed=0), arch, 64)
    eng.forward_tokens(np.array([1, 2], np.uint32))
    hbm, peak_kind = peaks()
    shapes = [("o", chpe.ROLE_O, "2048x2048"), ("gateup", chpe.ROLE_GATEUP, "2048x(2x11008) fused SwiGLU"),
              ("down", chpe.ROLE_DOWN, "11008x2048"), ("lmhead", chpe.ROLE_LMHEAD, "2048x151936 tied"),
              ("qkv", chpe.ROLE_QKV, "2048x(2048+256+256) fused RMSNorm")]
    rows = {}
    for name, role, shape in shapes:
        m, b, n = eng.bench_kernel_cold(role, rounds=max(1, args.steps // 8))
        g = b / (m / 1000) / 1e9
        rows[name] = {"shape_in_x_out": shape, "kernel": eng.op_kernel_name(role), "avg_us": round(m * 1000, 2),
                      "bytes_per_launch": b, "gbs": round(g, 1), "frac": round(g / hbm, 3), "launches": n}
    print(json.dumps({"sweep": M["name"], "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
                      "timing": "CUDA events around each launch, a 256 MiB buffer written before it (cold L2)",
                      "shapes": rows}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="72b-w4", choices=sorted(MODELS))
    ap.add_argument("--verify", type=int, default=0, choices=[0, 4, 8],
                    help="config 4: batch-M speculative verification on the 9B archive at a 2048 context")
    ap.add_argument("--sweep", action="store_true",
                    help="config 2's isolated GEMV sweep (3B archives): per-shape GB/s from a cold L2")
    ap.add_argument("--prompt", type=int, default=None,
                    help="prompt tokens decoded before timing (default: the model's config)")
    ap.add_argument("--kernel-only", default=None,
                    choices=["qkv", "attention", "o", "gateup", "down", "lmhead", "flat-aligned", "flat-stream",
                             "flat-rowblk", "bgemm4", "bgemm8"],
                    help="profiling case: build the engine (max_seq_len 64) and only launch this "
                         "op of every layer, --steps rounds after one warm-up round; flat-aligned / "
                         "flat-stream: one flat GEMV over 2064 contiguous 4-bit cells of the 3B "
                         "archive (35 MB) read as 8192 columns (aligned cells: the tensor-core mode, "
                         "or with CHPE_FLAT_MMA=0 the FFMA aligned mode) or 29568 columns (the 72B "
                         "down width: column owners, or with CHPE_FLAT_COLOWN=0 the stream mode); "
                         "flat-rowblk: the same cells as 2280 rows x 29568 columns (the row-block "
                         "tensor-core kernel); --steps launches")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    args.prompt_given = args.prompt is not None
    if args.prompt is None:
        args.prompt = MODELS[args.model]["prompt"]
    if args.verify:
        run_verify(args)
        return
    if args.sweep:
        if args.model not in ("3b-w4", "3b-w2", "3b-fp16"):
            args.model = "3b-w4"
        run_sweep(args)
        return
    if args.kernel_only in ("bgemm4", "bgemm8"):
        # the batched tcgen05 GEMM alone: the 9472 embedding cells of the 3B
        # archive (165 MB, beyond L2) read as a 75776 x 4096 tensor, NT
        # tokens, --steps launches through the probe entry point
        import chpe_qwen_engine_b200 as chpe
        nt = 4 if args.kernel_only == "bgemm4" else 8
        eng = chpe.Engine.from_bytes(chpe.synth_archive(chpe.SYNTH_3B_W4, 0, seed=0), chpe.ARCH_3B, 64)
        rows, cols = 75776, 4096
        x = np.random.default_rng(3).standard_normal((nt, cols)).astype(np.float32)
        for _ in range(max(1, args.steps)):
            y = eng.probe_bgemm(0, 9472, x, rows, cols)
        print(json.dumps({"kernel": "bgemm_w4_kernel", "nt": nt, "rows": rows, "cols": cols,
                          "y00": float(y[0][0])}))
        return
    if args.kernel_only in ("flat-aligned", "flat-stream", "flat-rowblk"):
        import chpe_qwen_engine_b200 as chpe
        eng = chpe.Engine.from_bytes(chpe.synth_archive(chpe.SYNTH_3B_W4, 0, seed=0), chpe.ARCH_3B, 64)
        tile0, ntiles = 9497, 2064  # layer 0 down, gate, up: contiguous 4-bit cells
        cols = 8192 if args.kernel_only == "flat-aligned" else 29568
        rows = ntiles * 32768 // cols
        if args.kernel_only == "flat-rowblk":
            rows -= rows % 8  # whole 8-row units: the row-block tensor-core kernel
        x = np.random.default_rng(3).standard_normal(cols).astype(np.float32)
        for _ in range(max(1, args.steps)):
            y = eng.probe_gemv_linear(tile0, ntiles, x, rows, cols)
        print(json.dumps({"kernel": args.kernel_only, "rows": rows, "cols": cols,
                          "kernel_name": "gemv_rowblk_kernel" if args.kernel_only == "flat-rowblk"
                          else "gemv_flat_tma_kernel", "y0": float(y[0])}))
        return
    if args.kernel_only:
        import chpe_qwen_engine_b200 as chpe
        roles = {"qkv": chpe.ROLE_QKV, "attention": chpe.ROLE_ATTN, "o": chpe.ROLE_O,
                 "gateup": chpe.ROLE_GATEUP, "down": chpe.ROLE_DOWN, "lmhead": chpe.ROLE_LMHEAD}
        M = MODELS[args.model]
        # --prompt given explicitly: decode that many tokens first, so the
        # attention kernel runs at that context length
        ctx = args.prompt if args.prompt_given else 0
        eng = chpe.Engine.from_bytes(chpe.synth_archive(getattr(chpe, M["synth"]), 0, seed=0),
                                     getattr(chpe, M["arch"]), ctx + 64)
        if ctx:
            eng.forward_tokens(np.random.default_rng(1).integers(0, 151936, ctx).astype(np.uint32))
        ms, b, n = eng.bench_kernel(roles[args.kernel_only], rounds=max(1, args.steps))
        print(json.dumps({"kernel": args.kernel_only, "avg_us": ms * 1000, "bytes_per_launch": b,
                          "gbs": b / (ms / 1000) / 1e9 if b else None, "launches": n}))
        return
    rank, world, local, dist = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world, dist)
        else:
            run_ours(args, rank, world, local, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
