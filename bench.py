#!/usr/bin/env python3
"""Benchmark: DF-SSM greedy decode tok/s on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg1] [--impl ours|reference]

A step is one greedy decode step of the whole batch: embedding gather, all layers
(in_proj + conv + SSM + gate + out_proj), final norm, LM head and argmax.  Before the
timed region every sequence consumes its 16-token prompt and W warm-up steps; then
exactly K steps are timed with CUDA events between a barrier + synchronize on each side.
Weights, embedding and state stream from HBM every step (>= 482 MB/step for cfg1, far
above the 126 MB L2), so no explicit L2 flush is needed.

Configs (synthetic weights of the stated shapes, seed 0):
  cfg0  2-layer 1.3B width, batch 1           cfg1  48-layer 1.3B, batch 1 (default)
  cfg2  48-layer 1.3B, batch 32               cfg4  64-layer 2.7B, batch 256 split over ranks
  --prefill T  instead of decode steps, time K prompt prefills (reset + dfssm_prefill of a [batch, T]
        random prompt; metric prompt tok/s)
  cfg3  isolated scaffold GEMM (1-bit x int8 -> int32, dfssm_scaffold_gemm) at the 1.3B in_proj and
        out_proj shapes for M in {1, 8, 32, 128, 512}; one JSON line with the sweep
Multi-GPU: one process per GPU, each with a full weight replica and its own sequences;
no collective on the data path (NCCL only for the barrier and the max-over-ranks time).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "cfg0": dict(shape="1.3b", layers=2, batch=1, scaling="weak"),
    "cfg1": dict(shape="1.3b", layers=48, batch=1, scaling="weak"),
    "cfg2": dict(shape="1.3b", layers=48, batch=32, scaling="weak"),
    "cfg4": dict(shape="2.7b", layers=64, batch=256, scaling="strong"),
    "cfg3": dict(shape="1.3b", layers=0, batch=0, scaling="weak"),
}
CFG3_SHAPES = (("in_proj", 8512, 2048), ("out_proj", 2048, 4096))
CFG3_M = (1, 8, 32, 128, 512)
METRIC = "decode tok/s at Mamba-2 1.3B shape, batch 1/32 per B200; HBM GB/s vs 8 TB/s"
PROMPT_LEN = 16


def step_bytes(d, batch: int) -> dict:
    """Algorithmic HBM bytes of one decode step (read once each): packed scaffold + fp16 scales +
    int8 LoRA (+ scales) + conv/SSM params + norms per layer, final norm, int8 embedding + per-row
    scale, and per sequence the fp32 SSM and conv state read and written."""
    def proj(n, k):
        return n * k // 8 + 2 * n + 16 * n + 2 * n + 16 * k + 32
    per_layer = (proj(d.n_in, d.d_model) + proj(d.d_model, d.d_inner) + d.d_xbc * 4 * 2 + d.d_xbc * 2
                 + 3 * d.nheads * 4 + d.d_inner * 4 + d.d_model * 4)
    weights = d.n_layer * per_layer + d.d_model * 4
    emb = d.vocab * d.d_model + d.vocab * 4
    state_seq = d.n_layer * 2 * (d.nheads * d.headdim * d.d_state * 4 + 3 * d.d_xbc * 4)
    return dict(weights=weights, embedding=emb, state=batch * state_seq, total=weights + emb + batch * state_seq)


def rank_batch(cfg: dict, world: int) -> tuple:
    """(sequences per rank, sequences of the whole job): weak scaling keeps the config's batch per
    rank, strong scaling splits the config's batch over the ranks."""
    if cfg["scaling"] == "weak":
        return cfg["batch"], cfg["batch"] * world
    if cfg["batch"] % world:
        raise SystemExit(f"batch {cfg['batch']} not divisible by {world} ranks")
    return cfg["batch"] // world, cfg["batch"]


def rank_rows(rank: int, per_rank: int) -> slice:
    """This rank's contiguous slice of the job's sequences (no data-path collective needed)."""
    return slice(rank * per_rank, (rank + 1) * per_rank)


def max_over_ranks(value: float, world: int, device) -> float:
    """Max of a per-rank timing over all ranks (all_reduce MAX on the process group's backend)."""
    if world <= 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join("/tmp", f"dfssm_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.remove(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_run(cfg: dict, steps: int, warmup: int, threads: int, batch: int) -> dict:
    """Times the reference's own CPU engine (oracle/_ref, built from inference/cpu/cpu_inference.c)
    in a child process with `threads` OpenMP/BLAS threads; falls back to "unavailable"."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ref_cpu
    from dfssm_b200 import synthetic
    d = synthetic.make_dims(cfg["shape"], 1)
    key = ref_cpu.shape_key(d)
    if not os.path.exists(ref_cpu.lib_path(key)):
        return {"unavailable": f"oracle/_ref/libcpu_inference_{key}.so not built"}
    if not ref_cpu.cpu_supports_reference():
        return {"unavailable": "host CPU lacks AVX-512 VNNI needed by the reference cpu_inference.c"}
    env = dict(os.environ, OMP_NUM_THREADS=str(threads), OPENBLAS_NUM_THREADS=str(threads),
               MKL_NUM_THREADS=str(threads), OMP_PROC_BIND="close")
    cmd = [sys.executable, os.path.join(ROOT, "oracle", "ref_cpu.py"), "--shape", cfg["shape"], "--layers",
           str(cfg["layers"]), "--batch", str(batch), "--prompt", str(PROMPT_LEN), "--steps", str(steps),
           "--warmup", str(warmup)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=1800)
    if r.returncode != 0:
        return {"unavailable": f"reference CPU run failed: {r.stderr.strip().splitlines()[-1:]}"}
    return json.loads(r.stdout.strip().splitlines()[-1])


def cpu_model_name() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def physical_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference_arm(args, cfg, rank, world):
    if rank != 0:
        return
    # the whole job's sequences: per-GPU batch x ranks (weak scaling) or the global batch (strong)
    batch = rank_batch(cfg, world)[1]
    threads = physical_threads()
    res = cpu_reference_run(cfg, args.steps, args.warmup, threads, batch)
    if "unavailable" in res:
        print(json.dumps({"impl": "reference", "unavailable": res["unavailable"]}))
        return
    value = res["tok_per_s"]
    from dfssm_b200 import synthetic
    dims = synthetic.make_dims(cfg["shape"], cfg["layers"])
    sample = f"{args.steps} greedy steps x batch {batch} after a {PROMPT_LEN}-token prompt, {cfg['layers']}-layer {cfg['shape']}"
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["seconds"] / args.steps * 1e3, "higher_is_better": True,
            "scaling": cfg["scaling"], "vs_baseline": None, "dtype": "int8/fp32 (AVX-512 VNNI)",
            "data": "synthetic (seeded random weights and prompts)", "impl": "reference",
            "config": workload_config(args.config, cfg, rank_batch(cfg, world)[0], batch,
                                      step_bytes(dims, rank_batch(cfg, world)[0])["total"]),
            "engine": {"impl": "reference inference/cpu/cpu_inference.c (HEADDIM 64), cpu_inference_driver loop",
                       "parallelism": "rank 0 decodes every sequence of the job on the host cores"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "reference",
                             "sample": sample, "cpu": cpu_model_name()},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_scaffold_bench(args, rank, world):
    """cfg3: times dfssm_scaffold_gemm (activation permute + 1-bit x int8 tensor-core or dp4a
    GEMM) per shape and M.  Each timed call reads a different copy of the packed weights (copies
    totalling > 126 MB of L2), so every call streams its weights from HBM."""
    import torch
    from dfssm_b200 import _lib
    if rank != 0:
        return
    lib = _lib.load()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)  # a non-default stream: the timed calls are captured
    s_ptr = ctypes.c_void_p(stream.cuda_stream)
    rng = np.random.default_rng(0)
    peak_hbm, peak_kind = load_peaks()
    sweep = []
    clocks = ClockSampler(dev.index)
    clocks.start()
    for name, N, K in CFG3_SHAPES:
        wbytes = N * K // 8
        ncopy = max(2, -(-160 * 2**20 // wbytes))
        packed = torch.from_numpy(rng.integers(0, 2**32, size=(ncopy, N, K // 32), dtype=np.uint64)
                                  .astype(np.uint32).view(np.int32)).to(dev)
        for M in CFG3_M:
            q = torch.from_numpy(rng.integers(-128, 128, size=(M, K), dtype=np.int8)).to(dev)
            acc = torch.empty(M, N, dtype=torch.int32, device=dev)
            ws = torch.empty(max(1, lib.dfssm_scaffold_gemm_workspace(M, K)), dtype=torch.uint8, device=dev)

            def call(i):
                _lib.check(lib.dfssm_scaffold_gemm(ctypes.c_void_p(packed[i % ncopy].data_ptr()),
                                                   ctypes.c_void_p(q.data_ptr()), M, N, K,
                                                   ctypes.c_void_p(acc.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                                   s_ptr))
            torch.cuda.synchronize()
            for i in range(args.warmup):
                call(i)
            torch.cuda.synchronize()
            # the K timed calls replay as one CUDA graph: device time of the operator, without the
            # host's per-call launch overhead (which exceeds the kernels at small M)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(args.steps):
                    call(i)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):  # replay() launches on the current stream
                g.replay()
                torch.cuda.synchronize()
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / args.steps
            ops = 2.0 * M * N * K
            sweep.append({"proj": name, "M": M, "N": N, "K": K, "us": us, "tops": ops / us / 1e6,
                          "weight_gbs": wbytes / us / 1e3,
                          "path": "tcgen05 i8" if M >= 64 else ("mma.sync s8" if M >= 8 else "dp4a")})
    clk = clocks.stop()
    best = next(r for r in sweep if r["proj"] == "in_proj" and r["M"] == 512)
    small = next(r for r in sweep if r["proj"] == "in_proj" and r["M"] == 1)
    line = {"metric": "scaffold GEMM (1-bit x int8 -> int32) int8 TOP/s, 1.3B in_proj, M=512", "value": best["tops"],
            "unit": "TOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": best["us"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 x 1-bit -> int32",
            "data": "synthetic (random sign bits and int8 activations)",
            "config": {"workload": "cfg3", "shapes": [list(s) for s in CFG3_SHAPES], "M": list(CFG3_M),
                       "l2": "weights rotate over copies totalling > 160 MB"},
            "roofline": {"bound": "hbm", "kernel": "scaffold GEMM, in_proj M=1", "achieved": small["weight_gbs"],
                         "peak": peak_hbm, "unit": "GB/s", "frac": small["weight_gbs"] / peak_hbm,
                         "peak_kind": peak_kind, "traffic": None,
                         "note": "M <= 32 streams the packed weights (HBM-bound); tensor use grows with M"},
            "sweep": sweep, "gpu_launches": 2 * args.steps * len(sweep), "clocks": clk, "cpu_baseline": None,
            "e2e": None}
    print(json.dumps(line))


def run_prefill_bench(args, cfg, m, batch, world, rank, local, dims):
    """K timed prompt prefills (reset + dfssm_prefill of one [batch, T] prompt each), device time,
    max over ranks; prompts of T > 64 tokens run in 64-token chunks."""
    import torch
    import torch.distributed as dist
    T = args.prefill
    prompt = torch.from_numpy(np.random.default_rng(1 + rank).integers(0, dims.vocab, (batch, T))).to(
        device=f"cuda:{local}", dtype=torch.int32)
    for _ in range(args.warmup):
        m.reset_state()
        m.prefill(prompt)
    stream = torch.cuda.current_stream()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        m.reset_state()
        m.prefill(prompt)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world, torch.device("cuda", local))
    m.check_finite()
    if rank == 0:
        print(json.dumps({
            "metric": "prompt prefill tok/s", "value": batch * world * T * args.steps / (ms / 1e3), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 x 1-bit -> int32 scaffold, fp16 activations, fp32 state",
            "data": "synthetic (seeded random weights of the named shape and random prompts)",
            "config": {"workload": args.config, "shape": cfg["shape"], "layers": cfg["layers"],
                       "batch_per_gpu": batch, "prompt": T, "mode": m.mode}}))
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--config", default="cfg1", choices=list(CONFIGS))
    ap.add_argument("--batch", type=int, default=None, help="override the config's batch (per GPU for weak scaling)")
    ap.add_argument("--layers", type=int, default=None, help="override the config's layer count (small profiling cases)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="auto", choices=["auto", "graph", "eager", "persistent"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="skip the sub-records (batch-32 and cfg4 lines)")
    ap.add_argument("--cfg4", action="store_true", help="add the cfg4 batch-256 strong-split sub-record at N = 1 too")
    ap.add_argument("--kernel-times", type=int, default=0, metavar="K",
                    help="after the timed region, replay K more steps under the CUDA activity profiler and print "
                         "each kernel's warm mean duration and its time per step (stderr, rank 0)")
    ap.add_argument("--prefill", type=int, default=0, metavar="T",
                    help="time K prompt prefills of T tokens per sequence instead of decode steps")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["batch"] = args.batch
    if args.layers:
        cfg["layers"] = args.layers
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)

    if args.config == "cfg3":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "cfg3 is a GPU operator microbench; the "
                                  "reference CPU engine has no stand-alone scaffold GEMM entry point"}))
            return
        run_scaffold_bench(args, rank, world)
        return
    if args.impl == "reference":
        if args.prefill:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference has no prompt prefill: its "
                                  "drivers feed a prompt one decode step per token"}))
            return
        run_reference_arm(args, cfg, rank, world)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from dfssm_b200 import synthetic
    from dfssm_b200.model import DFSSMModel

    batch, job_batch = rank_batch(cfg, world)
    dims = synthetic.make_dims(cfg["shape"], cfg["layers"])
    w = synthetic.make_weights(dims, seed=0)
    if args.prefill:
        m = DFSSMModel(w, device=f"cuda:{local}", batch_size=batch, mode=args.mode)
        run_prefill_bench(args, cfg, m, batch, world, rank, local, dims)
        return

    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v for v in vis.split(",") if v.strip()]
    phys = int(ids[local]) if ids and local < len(ids) and ids[local].strip().isdigit() else local
    rec, m = decode_record(args, args.config, cfg, w, dims, world, rank, local, phys, keep=True)
    batch = rec["batch"]

    # ---------------- end-to-end through the public host-buffer API (tokens in/out via pinned host memory)
    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    tok_h = torch.empty(batch, dtype=torch.int32).pin_memory().numpy()
    nxt_h = torch.empty(batch, dtype=torch.int32).pin_memory().numpy()
    tok_h[:] = m._tok_out[:batch].cpu().numpy()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.step_host(tok_h, nxt_h)
        tok_h[:] = nxt_h
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(e2e_s, world, torch.device("cuda", local))
    m.check_finite()
    mode = m.mode
    m.close()
    del m

    tokens_total = batch * world * args.steps
    e2e_value = tokens_total / e2e_s

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_steps = 128 if cfg["layers"] <= 48 and batch == 1 else 4
        threads = physical_threads()
        res = cpu_reference_run(cfg, cpu_steps, 2, threads, 1)
        if "unavailable" not in res:
            cpu = {"value": res["tok_per_s"], "unit": "tok/s", "cores": threads, "kind": "reference",
                   "sample": f"{cpu_steps} greedy steps, batch 1, after a {PROMPT_LEN}-token prompt "
                             f"({cfg['layers']}-layer {cfg['shape']}); the reference CPU path decodes one sequence",
                   "cpu": cpu_model_name()}
        else:
            cpu = {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference", "sample": res["unavailable"]}

    # ---------------- sub-records timed in the same process: the other half of the metric (batch 32 per
    # GPU) and, on multi-GPU runs, the batch-256 2.7B decode split over the ranks (strong scaling)
    subs = {}
    if args.config == "cfg1" and not args.no_sub:
        del w
        subs["cfg2_batch32"] = decode_record(args, "cfg2", dict(CONFIGS["cfg2"]), None, None, world, rank, local, phys)[0]
    if (args.gpus > 1 or world > 1 or args.cfg4) and args.config != "cfg4" and not args.no_sub:
        subs["cfg4_batch256_strong"] = decode_record(args, "cfg4", dict(CONFIGS["cfg4"]), None, None, world, rank,
                                                     local, phys, steps=min(args.steps, 32))[0]

    if rank == 0:
        line = {
            "metric": METRIC, "value": rec["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True,
            "scaling": cfg["scaling"], "vs_baseline": None,
            "dtype": "int8 x 1-bit -> int32 scaffold, fp16 activations, fp32 state",
            "data": "synthetic (seeded random weights of the named shape and random prompts)",
            "config": rec["config"],
            "engine": {"mode": mode, "parallelism": f"sequence-sharded dp{world} (no collective)"},
            "roofline": rec["roofline"],
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 4 * batch,
                    "d2h_bytes_per_step": 4 * batch},
            "gpu_launches": rec["gpu_launches"] + sum(r["gpu_launches"] for r in subs.values()),
            "clocks": rec["clocks"],
            "cpu_baseline": cpu,
        }
        for k, r in subs.items():
            line[k] = {kk: r[kk] for kk in ("value", "unit", "ms_per_step", "steps", "scaling", "config", "engine",
                                            "roofline", "gpu_launches", "clocks")}
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def persistent_launches(batch: int) -> int:
    """Launches of the persistent step kernel per step: one per group of up to 4 sequences."""
    return -(-batch // 4)


def workload_config(name: str, cfg: dict, batch: int, job_batch: int, total_bytes: float) -> dict:
    """The workload keys, identical in both arms (the reference arm runs the same workload)."""
    return {"workload": name, "shape": cfg["shape"], "layers": cfg["layers"], "batch_per_gpu": batch,
            "global_batch": job_batch, "prompt": PROMPT_LEN,
            "l2": "no flush: each step streams >= %.0f MB from HBM (> 126 MB L2)" % (total_bytes / 1e6)}


def kernel_times(m, steps: int, label: str) -> None:
    """Per-kernel warm durations of `steps` decode steps (graph replays included), from the CUDA activity
    records of torch.profiler; printed to stderr.  Outside every timed region."""
    import collections
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            m.step(None, logits=False)
        torch.cuda.synchronize()
    ev = sorted((e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA),
                key=lambda e: e.time_range.start)
    if not ev:
        print(f"kernel times ({label}): no CUDA activity records", file=sys.stderr)
        return
    agg = collections.defaultdict(list)
    for e in ev:
        agg[e.name.split("(")[0][:64]].append(e.time_range.end - e.time_range.start)
    span = (ev[-1].time_range.end - ev[0].time_range.start) / steps
    busy = sum(sum(v) for v in agg.values()) / steps
    print(f"kernel times ({label}): {span:.1f} us per step from first start to last end, kernels "
          f"{busy:.1f} us per step (sum of durations)", file=sys.stderr)
    for n, v in sorted(agg.items(), key=lambda kv: -sum(kv[1])):
        print(f"  {n:64s} launches/step {len(v) / steps:6.1f}  mean {sum(v) / len(v):8.2f} us  "
              f"per step {sum(v) / steps:8.1f} us  share {sum(v) / steps / busy:6.1%}", file=sys.stderr)


def decode_record(args, name, cfg, w, dims, world, rank, local, phys, keep=False, steps=None):
    """Builds the engine for one decode workload, consumes the prompts and W warm-up steps, then
    times K greedy steps with CUDA events between a barrier + synchronize on each side (max over
    ranks).  Returns (record, engine if keep else None)."""
    import torch
    import torch.distributed as dist
    from dfssm_b200 import synthetic
    from dfssm_b200.model import DFSSMModel
    steps = steps or args.steps
    batch, job_batch = rank_batch(cfg, world)
    if w is None:
        dims = synthetic.make_dims(cfg["shape"], cfg["layers"])
        w = synthetic.make_weights(dims, seed=0)
    prompts = synthetic.make_prompts(dims.vocab, job_batch, PROMPT_LEN, seed=0)
    my_prompts = prompts[rank_rows(rank, batch)]
    m = DFSSMModel(w, device=f"cuda:{local}", batch_size=batch, mode=args.mode)
    del w
    stream = torch.cuda.current_stream()
    m.reset_state()
    m.prefill(torch.from_numpy(my_prompts))
    for _ in range(args.warmup):
        m.step(None, logits=False)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = ClockSampler(phys)
    clocks.start()
    time.sleep(0.3)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        m.step(None, logits=False)
    e1.record(stream)
    barrier()
    clk = clocks.stop()
    ms_max = max_over_ranks(e0.elapsed_time(e1), world, torch.device("cuda", local))
    m.check_finite()
    if getattr(args, "kernel_times", 0) and rank == 0:
        kernel_times(m, args.kernel_times, f"{name} batch {batch} ({m.mode})")
    sb = step_bytes(dims, batch)
    peak, peak_kind = load_peaks()
    step_ms = ms_max / steps
    achieved = sb["total"] / (step_ms / 1e3) / 1e9
    n_launch = {"graph": 5 * dims.n_layer + 4, "eager": 5 * dims.n_layer + 4,
                "persistent": persistent_launches(batch)}[m.mode]
    traffic = None
    tf = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if os.path.exists(tf):
        with open(tf) as f:
            tj = json.load(f)
        ent = tj.get(f"{name}:{m.mode}:b{batch}")
        if ent:
            traffic = ent["bytes_per_launch"]
    rec = {"value": batch * world * steps / (ms_max / 1e3), "unit": "tok/s", "ms_per_step": step_ms, "steps": steps,
           "scaling": cfg["scaling"], "batch": batch,
           "config": workload_config(name, cfg, batch, job_batch, sb["total"]),
           "engine": {"mode": m.mode, "parallelism": f"sequence-sharded dp{world} (no collective)"},
           "roofline": {"bound": "hbm", "kernel": "whole decode step" if m.mode != "persistent" else "persistent step kernel",
                        "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                        "peak_kind": peak_kind, "bytes_per_step": sb["total"], "traffic": traffic},
           "gpu_launches": n_launch * steps, "clocks": clk}
    if keep:
        return rec, m
    m.close()
    del m
    torch.cuda.empty_cache()
    return rec, None

if __name__ == "__main__":
    main()
