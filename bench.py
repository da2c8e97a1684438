#!/usr/bin/env python
"""Dual-AR frames/s of the sm_100a path (and of the reference's CPU path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

Workload: BASELINE config 2 (C2), the full-size S2-Pro-shaped f16 Dual-AR
(36 Slow-AR layers, 4 Fast-AR layers, d 2560, vocab 155,776, 10 codebooks x
4096), random-init weights written as a seeded synthetic GGUF, 512-token
seeded prompt, greedy decode of 256 frames at batch 1.  The same run then
measures config 4 (C4: 64 sequences, prompts of 128..1024 tokens, 512 frames,
T 0.8 / top-p 0.9 / top-k 30 with per-sequence Philox) and nests that line
under "batch64" (--no-batch64 skips it; --workload C1..C5 runs one config).

One step = one generate_codes call (prefill + 256 frames).  Reported:
  value      frames/s of the decode loop, device time (CUDA events on the
             library's stream around the frame graphs), weights and prompt
             already resident; whole-job = all ranks' frames / max rank time.
  e2e        frames/s through the C ABI with host buffers: prompt upload,
             prefill, every frame, codes download, wall clock bracketed by
             barrier + device synchronize, max over ranks.
  roofline   the dominant kernel: the persistent decode engine running the
             Slow-AR step program (36 layers + masked LM head), timed live
             with CUDA events on the library's stream after the timed steps;
             achieved = algorithmic bytes of one launch (the step's weights +
             the KV rows it attends) / median launch time, against
             MEASURED_PEAKS.json.  The Fast-AR pass program is listed beside it.
  cpu_baseline  the CPU oracle (port of the reference's algorithm) on a
             bounded sample of the same workload, rank 0, N = 1 only.
Nested lines (N = 1): "q8_0" (C3) and "q4_k" (C5), the quantized batch-1
configurations, timed over min(steps, 5) steps each (--no-quant skips them).
Multi-GPU (torchrun, N > 1): the headline line is the Slow-AR tensor-parallel
run (all ranks decode one utterance, heads and FFN columns sharded, NCCL
allreduce per residual add; "scaling": "strong"); the independent-replica run
(every rank decodes its own utterance, weak scaling, no data-path collective)
is nested under "replicas".  --replicas makes the replica run the headline.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from fish_s2pro_b200 import configs  # noqa: E402

METRIC = "Dual-AR frames/sec (batch 1)"
METRIC_BATCH = "Dual-AR frames/sec (batch 64)"
# arithmetic of the linears: f16 weights, or ggml blocks dequantised in
# registers; activations and accumulation are f32 throughout
WTYPE = {configs.GGML_F16: "f16", configs.GGML_Q8_0: "q8_0", configs.GGML_Q4_K: "q4_k"}
UNIT = "frames/s"
# DRAM traffic of one Slow-AR step program over its algorithmic bytes, from an
# ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of the 4-layer
# C2S step: 845,365,248 B for 829,445,120 algorithmic bytes.  Every layer
# streams its own weights once, so the ratio carries over to 36 layers.
ENGINE_TRAFFIC_RATIO = 845365248 / 829445120


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="C2")
    ap.add_argument("--frames", type=int, default=None, help="override frames per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernel-profile", action="store_true")
    ap.add_argument("--prompt-len", type=int, default=None,
                    help="override the prompt length (profiling runs only)")
    ap.add_argument("--model-dir", default=None, help="GGUF cache (default: synth.default_model_dir())")
    ap.add_argument("--no-batch64", action="store_true",
                    help="skip the batch-64 (C4) measurement that the default C2 run adds to its line")
    ap.add_argument("--tp", action="store_true",
                    help="under torchrun: all ranks form one tensor-parallel Slow-AR decoding one "
                         "utterance (strong scaling); the default under torchrun")
    ap.add_argument("--replicas", action="store_true",
                    help="under torchrun: independent replicas (weak scaling) as the headline line")
    ap.add_argument("--no-serving", action="store_true",
                    help="skip the nested continuous-batching line of the default run")
    ap.add_argument("--no-codec", action="store_true",
                    help="skip the nested codec-decode line (codes -> PCM) of the default run")
    ap.add_argument("--codec-only", action="store_true",
                    help="measure only the codec decode line (profiling)")
    ap.add_argument("--no-quant", action="store_true",
                    help="skip the nested C3 (Q8_0) and C5 (Q4_K) lines of the default N = 1 run")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

class Dist:
    def __init__(self, gpus: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{self.local}")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{self.local}")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def bcast_bytes(self, b: bytes | None) -> bytes:
        """Rank 0's bytes on every rank."""
        if not self.pg:
            return b
        obj = [b]
        self.pg.broadcast_object_list(obj, src=0)
        return obj[0]

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def device_sync():
    import torch
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = Path(f"/tmp/s2d_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        sm, mx, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        load = [s for s, p in zip(sm, power) if p > 300] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power)}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d.get("bf16_tflops", 1590.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# CPU oracle timing (port of the reference's algorithm)
# ---------------------------------------------------------------------------

def oracle_frames(model_path, wl, frames: int, warmup: int, prompt_len: int, seed: int = 0):
    """The reference's generate_codes loop (generate.rs:117-221) on the CPU
    oracle in reference-faithful mode (per-step f32 weight re-expansion,
    per-codebook Fast-AR prefix recomputation, full-vocabulary LM head and
    sort).  Returns (seconds per timed frame, threads, prefill seconds)."""
    from oracle import oracle as o
    m = wl.model
    om = o.OracleModel(model_path, max_seq_len=prompt_len + frames + warmup + 4, mode=1)
    gp = wl.gen_params(greedy=True)
    prompt = wl.prompt()[:, :prompt_len]
    flat = prompt.T.reshape(-1).astype(np.int32)
    bias = o.build_semantic_bias(m.vocab, m.sem_begin, m.sem_end, gp["im_end_id"])
    rng = o.SeededRng(seed)
    t0 = time.perf_counter()
    hidden, logits = om.eval(flat)
    t_prefill = time.perf_counter() - t0
    main = o.sample_token(o.apply_semantic_bias(logits, bias, True, gp["im_end_id"]),
                          gp["temperature"], gp["top_p"], gp["top_k"], None, rng)
    times = []
    for f in range(warmup + frames):
        t = time.perf_counter()
        sem = main - m.sem_begin if m.sem_begin <= main <= m.sem_end else 0
        cbs = om.generate_codebooks(hidden, sem, gp["temperature"], gp["top_p"], gp["top_k"], rng)
        step = [main] + (cbs if m.sem_begin <= main <= m.sem_end else [0] * m.num_codebooks)
        hidden, logits = om.eval(step)
        main = o.sample_token(o.apply_semantic_bias(logits, bias, True, gp["im_end_id"]),
                              gp["temperature"], gp["top_p"], gp["top_k"], None, rng)
        if f >= warmup:
            times.append(time.perf_counter() - t)
    om.close()
    return sum(times) / len(times), o.get_threads(), t_prefill


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------

def ensure_model(d, wl, model_dir, lib_path=None) -> Path:
    """The workload's synthetic GGUF, written once per host (local rank 0)
    with the writer at lib_path (default: the package's, see synth._load)."""
    from fish_s2pro_b200 import synth
    if d.local == 0:
        synth.cached_gguf(wl.model, model_dir, lib_path)
    d.barrier()
    return synth.cached_gguf(wl.model, model_dir, lib_path)


def run_ours(args, d: Dist, wl_name=None, use_tp=False, steps=None, warmup=None, cpu_baseline=True):
    """Batch-1 generation of workload wl_name (default args.workload): one
    utterance per rank (replicas) or, with use_tp under torchrun, one
    utterance over all ranks (Slow-AR tensor parallelism)."""
    from fish_s2pro_b200 import (FastArWeights, GenerateParams, PromptTensor, SeededRng,
                                 SlowArState, build, generate_codes)
    build.build_runtime()
    wl_name = wl_name or args.workload
    wl = {**configs.WORKLOADS, **configs.PROFILING}[wl_name]
    if args.prompt_len:
        wl = configs.Workload(wl.model, args.prompt_len, wl.frames, wl.prompt_seed, wl.im_end_id)
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    frames = args.frames or wl.frames
    m = wl.model
    path = ensure_model(d, wl, args.model_dir)
    tp = None
    if use_tp and d.world > 1:
        from fish_s2pro_b200 import nccl_unique_id
        tp = (d.world, d.rank, d.bcast_bytes(nccl_unique_id() if d.rank == 0 else None))
    st = SlowArState.open(path, max_seq_len=wl.prompt_len + frames + 8, device=d.local, tp=tp)
    spec = st.graph_spec()
    fw = FastArWeights.from_state(st)
    # replicas decode their own prompts; tensor-parallel ranks share one
    prompt = configs.Workload(m, wl.prompt_len, frames, wl.prompt_seed + (0 if tp else d.rank),
                              wl.im_end_id).prompt()
    gp = wl.gen_params(greedy=True)
    gp["max_new_tokens"] = frames
    gp["min_tokens_before_end"] = 2 * frames + 2
    params = GenerateParams(frames, gp["temperature"], gp["top_p"], gp["top_k"],
                            gp["min_tokens_before_end"])
    pt = PromptTensor(prompt.shape[0], prompt.shape[1], prompt.reshape(-1))

    def one(seed):
        return generate_codes(st, gp["im_end_id"], spec, pt, params, fw, SeededRng(seed))

    for i in range(warmup):
        one(i)
    clocks = Clocks(d.local)
    d.barrier()
    device_sync()
    clocks.start()
    t0 = time.perf_counter()
    results = [one(100 + i) for i in range(steps)]
    device_sync()
    t1 = time.perf_counter()
    d.barrier()
    ck = clocks.stop()
    wall = d.max(t1 - t0)
    decode_s = d.max(sum(r.profile.decode_ms for r in results) / 1e3)
    prefill_ms = d.max(statistics.mean(r.profile.prefill_ms for r in results))
    my_frames = sum(r.n_frames for r in results)
    frames_total = my_frames if tp else d.sum(my_frames)
    launches = sum(r.profile.prefill_kernels + r.profile.kernels_per_frame *
                   r.profile.frame_launches for r in results)
    value = frames_total / decode_s
    e2e = frames_total / wall
    pk = peaks()
    bpf = configs.weight_bytes_per_frame(m)
    # the engine's programs, timed live after the timed steps on the state
    # they left (n_past = prompt + frames): median of 7 launches each
    kern = {}
    if not args.no_kernel_profile and not tp:  # the engine is single-GPU
        n_past = st.n_past()
        kv_pos = configs.kv_bytes_per_position(m)
        passes = m.num_codebooks - 1
        for prog, name, nbytes in ((0, "slow_step", bpf["slow"] + bpf["lm_head"] + kv_pos * (n_past + 1)),
                                   (2, "fast_pass", bpf["fast"] / passes)):
            ms = statistics.median(st.profile_engine(prog, trace=False)[0] for _ in range(7))
            kern[name] = {"ms": ms, "bytes": nbytes, "gbs": nbytes / ms / 1e6}
        try:  # the frame's whole Fast-AR in one launch (all passes, heads and samplers)
            ms = statistics.median(st.profile_engine(-1, trace=False)[0] for _ in range(7))
            kern["fast_frame"] = {"ms": ms, "bytes": bpf["fast"], "gbs": bpf["fast"] / ms / 1e6}
        except RuntimeError:
            pass
    top = kern.get("slow_step")
    p_avg = wl.prompt_len + frames / 2
    frame_bytes = sum(bpf.values()) + configs.kv_bytes_per_position(m) * p_avg
    # HBM bytes each GPU streams per second: a replica streams whole frames;
    # a tensor-parallel rank its share of the Slow-AR and KV plus the
    # replicated LM head and Fast-AR
    if tp:
        rank_bytes = ((bpf["slow"] + configs.kv_bytes_per_position(m) * p_avg) / d.world
                      + bpf["lm_head"] + bpf["fast"] + bpf["embed_rows"])
        gpu_gbs = rank_bytes * value / 1e9
    else:
        gpu_gbs = frame_bytes * value / d.world / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": d.world,
        "steps": steps, "warmup": warmup,
        "ms_per_step": round(wall / steps * 1e3, 2),
        "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
        "dtype": WTYPE[m.linear_type],
        "data": f"synthetic (seeded random-init S2-Pro-shaped GGUF, seeded {wl.prompt_len}-id prompt)",
        "config": {"workload": f"{wl_name}: full-size {WTYPE[m.linear_type]} S2-Pro-shaped Dual-AR, "
                               f"{wl.prompt_len}-token prompt, greedy {frames} frames, batch 1",
                   "global_batch": 1 if tp else d.world, "seq_len": wl.prompt_len + frames,
                   "parallelism": (f"tp{d.world} (Slow-AR heads and FFN columns sharded; the wo "
                                   "and w2 partial sums exchanged inside the persistent engine "
                                   "over NVLink peer stores; Fast-AR replicated)") if tp
                                  else f"replicas x{d.world} (independent utterances)",
                   "l2": f"inputs larger than L2 (each frame streams {frame_bytes / 1e9:.2f} GB of "
                         f"{WTYPE[m.linear_type]} weights and KV rows; L2 is 0.126 GB)"},
        "e2e": {"value": round(e2e, 2), "unit": UNIT,
                "h2d_bytes_per_step": int(prompt.nbytes),
                "d2h_bytes_per_step": int(m.num_codebooks * frames * 4 + 40)},
        "gpu_launches": int(launches),
        "prefill_ms": round(prefill_ms, 2),
        "frame_bytes": int(frame_bytes),
        "frame_gbs": round(gpu_gbs, 1),
        "frame_roofline_frac": round(gpu_gbs / pk["hbm_gbs"], 3),
        "roofline": ({"bound": "hbm", "kernel": f"engine_kernel, Slow-AR step program ({m.slow_layers} "
                                                "layers + masked LM head)",
                      "achieved": round(top["gbs"], 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                      "frac": round(top["gbs"] / pk["hbm_gbs"], 3),
                      "traffic": (int(top["bytes"] * ENGINE_TRAFFIC_RATIO)
                                  if m.linear_type == configs.GGML_F16 else None),
                      "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the 4-layer "
                                        "C2S Slow-AR step (1.019 x its algorithmic bytes), scaled to "
                                        "this step's algorithmic bytes",
                      "peak_source": pk["source"],
                      "bytes_per_launch": int(top["bytes"]),
                      "kernels": {k: {"us": round(v["ms"] * 1e3, 2), "gbs": round(v["gbs"], 1),
                                      "bytes": int(v["bytes"])} for k, v in kern.items()}}
                     if top else
                     {"bound": "hbm", "kernel": "whole frame on each rank (tensor-parallel Slow-AR: the "
                                                "rank's weight and KV shard, replicated LM head and Fast-AR)",
                      "achieved": round(gpu_gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                      "frac": round(gpu_gbs / pk["hbm_gbs"], 3), "traffic": None,
                      "peak_source": pk["source"]}),
        "clocks": ck,
    }
    if cpu_baseline and d.rank == 0 and d.world == 1 and not args.no_cpu_baseline:
        spf, cores, _ = oracle_frames(path, wl, frames=2, warmup=0, prompt_len=16)
        line["cpu_baseline"] = {
            "value": round(1.0 / spf, 4), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"2 decode frames after a 16-token prefill of the same {wl_name} model, "
                      "reference-faithful CPU oracle (f32 re-expansion per step, Fast-AR "
                      "prefix recomputation, full-vocab LM head and sort)"}
    st.close()
    return line


def run_serving(args, d: Dist, wl, n_req=128, frames=64, slots=64, kv_pages=640):
    """Continuous batching (TtsScheduler over s2d_serve_*) on the C4 model:
    n_req requests with C4's prompt lengths (uniform 128..1024) arrive at
    once and share `slots` slots of the batched frame; each generates
    `frames` frames (T 0.8, top-p 0.9, top-k 30, per-request SeededRng).  The
    KV pool holds kv_pages pages of 64 positions, fewer than slots requests
    of the longest prompt need, so admission also waits for pages.  The timed
    region is the whole run: every admission prefill, every frame, every
    collection (host copies included).  Each rank serves its own requests."""
    from fish_s2pro_b200 import GenerateParams, PromptTensor, SeededRng, SlowArState, TtsScheduler, build
    build.build_runtime()
    m = wl.model
    path = ensure_model(d, wl, args.model_dir)
    st = SlowArState.open(path, max_seq_len=wl.prompt_len + frames + 8, device=d.local, max_batch=slots,
                          kv_pages=kv_pages)
    gp = wl.gen_params(greedy=False)
    params = GenerateParams(frames, gp["temperature"], gp["top_p"], gp["top_k"], 2 * frames + 2)
    reqs = []
    for j in range((n_req + slots - 1) // slots):
        ps = configs.Workload(m, wl.prompt_len, frames, wl.prompt_seed + 1000 * d.rank + j, wl.im_end_id,
                              batch=slots, prompt_len_min=wl.prompt_len_min).batch_prompts()
        reqs += [PromptTensor(p.shape[0], p.shape[1], p.reshape(-1)) for p in ps]
    reqs = reqs[:n_req]

    def serve(rs):
        sch = TtsScheduler(st, gp["im_end_id"], params, frames_per_step=4)
        for i, r in enumerate(rs):
            sch.submit(r, SeededRng(7 + i))
        return sch, sch.run()

    serve(reqs[:8])  # capture the frame graph
    clocks = Clocks(d.local)
    d.barrier()
    device_sync()
    clocks.start()
    t0 = time.perf_counter()
    sch, out = serve(reqs)
    device_sync()
    t1 = time.perf_counter()
    d.barrier()
    ck = clocks.stop()
    wall = d.max(t1 - t0)
    my_frames = sum(r.result.n_frames for r in out.values())
    frames_total = d.sum(my_frames)
    lat = sorted(r.latency_s for r in out.values())
    line = {
        "metric": METRIC_BATCH, "value": round(frames_total / wall, 1), "unit": UNIT, "n_gpus": d.world,
        "steps": 1, "warmup": 1, "ms_per_step": round(wall * 1e3, 2), "dtype": WTYPE[m.linear_type],
        "scaling": "weak",
        "requests_per_s": round(d.sum(len(out)) / wall, 2),
        "latency_s": {"mean": round(statistics.mean(lat), 3), "p50": round(lat[len(lat) // 2], 3),
                      "p95": round(lat[min(len(lat) - 1, int(0.95 * len(lat)))], 3)},
        "queue_s_mean": round(statistics.mean(r.queue_s for r in out.values()), 3),
        "e2e": {"value": round(frames_total / wall, 1), "unit": UNIT,
                "h2d_bytes_per_step": int(sum(r.data.nbytes for r in reqs)),
                "d2h_bytes_per_step": int(my_frames * m.num_codebooks * 4)},
        "config": {"workload": f"serving: continuous batching on the C4 model, {n_req} requests arriving at "
                               f"once (prompts {wl.prompt_len_min}..{wl.prompt_len} tokens), {frames} frames each, "
                               f"{slots} slots, KV pool of {kv_pages} pages of 64 positions, T 0.8 / top-p 0.9 / "
                               "top-k 30, per-request SeededRng; prefills, frames and collection all timed",
                   "global_batch": slots * d.world, "parallelism": f"replicas x{d.world}"},
        "clocks": ck,
    }
    st.close()
    return line


def codec_flops_per_frame() -> float:
    """Algorithmic FLOPs of one code frame's decode (2 per multiply-add of
    every contraction, each counted once): post module, upsample, decoder
    (codec.rs:986, 2302, 1941).  The attention is counted at the full
    128-frame window."""
    H, F, E = 1024, 3072, 4096
    post = 8 * 2 * (H * 3 * H + H * H + 2 * H * F + F * H) + 8 * 2 * 2 * 128 * H
    up = 2 * (H * 2 * H) + 2 * 2 * (2 * H * E) + 2 * (2 * H * (2 * H)) + 2 * 4 * (2 * H * E)
    dec = 2 * 4 * 7 * H * 1536
    rows, cin = 4, 1536
    for r, c in zip((8, 8, 4, 2), (768, 384, 192, 96)):
        dec += 2 * rows * cin * 2 * r * c          # transposed conv, kernel 2 x stride
        rows *= r
        dec += 3 * 2 * rows * (7 * c * c + c * c)  # three residual units
        cin = c
    dec += 2 * rows * 7 * 96
    return float(post + up + dec)


def run_codec(args, d: Dist, frames=512, steps=None, warmup=None):
    """The codec decode (codes -> 44.1 kHz PCM, CodecDecoder over
    include/s2d_codec.h) of `frames` code frames (2,048 samples each) on a
    synthetic codec of the real shapes.  One step = one decode; `value`
    times it on device codes with CUDA events (s2d_codec_decode_waveform_device),
    `e2e` through decode_waveform with host codes in and host samples out.
    Each rank decodes its own codes (replicas)."""
    import torch
    from fish_s2pro_b200 import CodecDecoder, build, codec_synth
    from fish_s2pro_b200.codec import codec_lib
    build.build_runtime()
    steps = max(10, min(args.steps, 30)) if steps is None else steps
    warmup = max(3, min(args.warmup, 3)) if warmup is None else warmup
    if d.local == 0:  # one writer per host; the others find the file after the barrier
        codec_synth.cached_codec_gguf(args.model_dir)
    d.barrier()
    path = codec_synth.cached_codec_gguf(args.model_dir)
    c = CodecDecoder.open(path, device=d.local)
    rng = np.random.default_rng(1234 + d.rank)
    codes = np.concatenate([rng.integers(0, 4096, frames), rng.integers(0, 1024, 9 * frames)]).astype(np.int32)
    codes_dev = torch.from_numpy(codes).to(f"cuda:{d.local}")
    out = torch.empty(frames * 2048, dtype=torch.float32, device=f"cuda:{d.local}")
    # a stream of our own (not the legacy default stream, whose handle 0
    # would select the codec's internal stream): the decode and the events share it
    stream = torch.cuda.Stream(device=d.local)
    device_sync()
    lib = codec_lib()

    def step():
        rc = lib.s2d_codec_decode_waveform_device(c.handle, codes_dev.data_ptr(), 10, frames, out.data_ptr(),
                                                  stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(lib.s2d_codec_last_error(c.handle).decode())

    for _ in range(warmup):
        step()
    device_sync()
    clocks = Clocks(d.local)
    d.barrier()
    device_sync()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    device_sync()
    d.barrier()
    ck = clocks.stop()
    ms = d.max(e0.elapsed_time(e1) / steps)
    if lib.s2d_codec_sync(c.handle) != 0:
        raise RuntimeError(lib.s2d_codec_last_error(c.handle).decode())
    # end to end through the public call: codes from the host, samples back
    c.decode_waveform(codes, 10, frames)
    device_sync()
    d.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        w = c.decode_waveform(codes, 10, frames)
    t1 = time.perf_counter()
    d.barrier()
    e2e_s = d.max((t1 - t0) / steps)
    samples = frames * 2048
    flops = codec_flops_per_frame() * frames
    pk = peaks()
    line = {
        "metric": "codec_samples_per_s", "value": round(d.sum(samples) / (ms / 1e3)), "unit": "samples/s",
        "n_gpus": d.world, "steps": steps, "warmup": warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "dtype": "f16 tensor-core GEMMs, f32 accumulation",
        "realtime_factor": round(d.sum(samples) / (ms / 1e3) / 44100.0, 1),
        "e2e": {"value": round(d.sum(samples) / e2e_s), "unit": "samples/s", "h2d_bytes_per_step": int(codes.nbytes),
                "d2h_bytes_per_step": int(w.samples.nbytes)},
        "roofline": {"bound": "tensor", "achieved": round(flops / (ms / 1e3) / 1e12, 1), "peak": pk["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(flops / (ms / 1e3) / 1e12 / pk["bf16_tflops"], 3),
                     "traffic": None,
                     "note": f"whole decode: {flops / 1e12:.2f} TFLOP of contractions per step over the step's "
                             f"device time, of {pk['source']} dense bf16 peak"},
        "config": {"workload": f"codec decode of {frames} code frames ({samples} samples, "
                               f"{samples / 44100:.1f} s of 44.1 kHz audio) on a seeded synthetic codec of the "
                               "s2-pro shapes; workspace > L2 (no flush needed)",
                   "parallelism": f"replicas x{d.world}"},
        "clocks": ck,
    }
    # the reference-audio encoder (PCM -> prompt codes), end to end through
    # encode_reference_audio: 10 s of audio in, codes out
    if c.has_encoder:
        n_audio = 441000
        audio = (0.3 * np.sin(np.arange(n_audio) * 0.031) +
                 0.05 * np.random.default_rng(7 + d.rank).standard_normal(n_audio)).astype(np.float32)
        for _ in range(2):
            r = c.encode_reference_audio(audio)
        d.barrier()
        t0 = time.perf_counter()
        enc_steps = 5
        for _ in range(enc_steps):
            r = c.encode_reference_audio(audio)
        t1 = time.perf_counter()
        d.barrier()
        enc_s = d.max((t1 - t0) / enc_steps)
        line["encode"] = {
            "metric": "encode_samples_per_s", "value": round(d.sum(n_audio) / enc_s), "unit": "samples/s",
            "ms_per_call": round(enc_s * 1e3, 3), "realtime_factor": round(d.sum(n_audio) / enc_s / 44100.0, 1),
            "steps": enc_steps,
            "config": {"workload": f"encode_reference_audio of {n_audio} samples (10 s) -> {r.quantizer_frames} "
                                   "frames x 10 codes, host PCM in and host codes out (wall clock, synchronised)"},
            "e2e": {"value": round(d.sum(n_audio) / enc_s), "unit": "samples/s", "h2d_bytes_per_step": int(audio.nbytes),
                    "d2h_bytes_per_step": int(r.codes.nbytes + r.final_residual_l2.nbytes)},
        }
    if d.rank == 0 and d.world == 1 and not args.no_cpu_baseline:
        # the float64 numpy oracle on one code frame, all host threads (BLAS)
        from oracle import codec_oracle as co
        w64 = co.CodecWeights(path)
        one = codes.reshape(10, frames)[:, :1].reshape(-1)
        co.decode_waveform(one, 10, 1, w64)  # converts the weights once
        t0 = time.perf_counter()
        n_cpu = 2
        for _ in range(n_cpu):
            co.decode_waveform(one, 10, 1, w64)
        dt = (time.perf_counter() - t0) / n_cpu
        line["cpu_baseline"] = {"value": round(2048 / dt, 1), "unit": "samples/s", "cores": os.cpu_count(),
                                "kind": "port", "sample": "one code frame (2,048 samples) through the float64 "
                                                          "numpy codec oracle, twice"}
        if "encode" in line:
            clip = np.asarray(audio[:4096])
            co.encode_reference_audio(clip, w64)  # converts the encoder weights once
            t0 = time.perf_counter()
            co.encode_reference_audio(clip, w64)
            dt = time.perf_counter() - t0
            line["encode"]["cpu_baseline"] = {
                "value": round(4096 / dt, 1), "unit": "samples/s", "cores": os.cpu_count(), "kind": "port",
                "sample": "4,096 samples (2 code frames) through the float64 numpy encoder oracle, once"}
    c.close()
    return line


def run_batch(args, d: Dist, wl, name=None, steps=None, warmup=None):
    """Batched workload (C4): every rank generates for `wl.batch` independent
    prompts at once through s2d_generate_codes_batch; one step = one call
    (every sequence's prefill + `frames` frames of all sequences)."""
    from fish_s2pro_b200 import (RNG_PHILOX, FastArWeights, GenerateParams, PromptTensor,
                                 SeededRng, SlowArState, build, generate_codes_batch)
    build.build_runtime()
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    frames = args.frames or wl.frames
    m = wl.model
    path = ensure_model(d, wl, args.model_dir)
    B = wl.batch
    st = SlowArState.open(path, max_seq_len=wl.prompt_len + frames + 8, device=d.local, max_batch=B)
    spec = st.graph_spec()
    fw = FastArWeights.from_state(st)
    ps = configs.Workload(m, wl.prompt_len, frames, wl.prompt_seed + d.rank, wl.im_end_id,
                          batch=B, prompt_len_min=wl.prompt_len_min).batch_prompts()
    pts = [PromptTensor(p.shape[0], p.shape[1], p.reshape(-1)) for p in ps]
    gp = wl.gen_params(greedy=False)
    params = GenerateParams(frames, gp["temperature"], gp["top_p"], gp["top_k"], 2 * frames + 2)

    def one(key):
        return generate_codes_batch(st, gp["im_end_id"], spec, pts, params, fw,
                                    [SeededRng(0) for _ in ps], rng_kind=RNG_PHILOX, philox_key=key)

    for i in range(warmup):
        one(i)
    clocks = Clocks(d.local)
    d.barrier()
    device_sync()
    clocks.start()
    t0 = time.perf_counter()
    results = [one(100 + i) for i in range(steps)]
    device_sync()
    t1 = time.perf_counter()
    d.barrier()
    ck = clocks.stop()
    wall = d.max(t1 - t0)
    decode_s = d.max(sum(r[0].profile.decode_ms for r in results) / 1e3)
    prefill_ms = d.max(statistics.mean(r[0].profile.prefill_ms for r in results))
    my_frames = sum(x.n_frames for r in results for x in r)
    frames_total = d.sum(my_frames)
    launches = sum(r[0].profile.prefill_kernels + r[0].profile.kernels_per_frame *
                   r[0].profile.frame_launches for r in results)
    value = frames_total / decode_s
    e2e = frames_total / wall
    pk = peaks()
    bpf = configs.weight_bytes_per_frame(m)
    kv_pos = configs.kv_bytes_per_position(m)
    lens = [p.shape[1] for p in ps]
    # one batched frame step: the weights once, every sequence's KV rows
    step_bytes = bpf["slow"] + bpf["lm_head"] + bpf["fast"] + kv_pos * sum(n + frames / 2 for n in lens)
    step_s = decode_s / (steps * frames)
    achieved = step_bytes / step_s / 1e9
    h2d = int(sum(p.nbytes for p in ps))
    breakdown = {} if args.no_kernel_profile else {
        k: round(v, 3) for k, v in st.profile_batch(B).items()}
    line = {
        "metric": METRIC_BATCH, "value": round(value, 1), "unit": UNIT, "n_gpus": d.world,
        "steps": steps, "warmup": warmup,
        "ms_per_step": round(wall / steps * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": WTYPE[m.linear_type],
        "data": f"synthetic (seeded random-init S2-Pro-shaped GGUF, {B} seeded prompts)",
        "config": {"workload": f"{name or args.workload}: full-size {WTYPE[m.linear_type]} S2-Pro-shaped Dual-AR, {B} sequences, "
                               f"prompt lengths {min(lens)}..{max(lens)} (uniform "
                               f"{wl.prompt_len_min}..{wl.prompt_len}), {frames} frames each, "
                               f"T {gp['temperature']} top-p {gp['top_p']} top-k {gp['top_k']}, "
                               "per-sequence Philox4x32-10",
                   "global_batch": B * d.world, "seq_len": max(lens) + frames,
                   "parallelism": f"replicas x{d.world}, batch {B} per GPU",
                   "l2": "inputs larger than L2 (each frame step streams ~15 GB of weights and ~8 GB of KV)"},
        "e2e": {"value": round(e2e, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": int(B * m.num_codebooks * frames * 4 + B * 40)},
        "gpu_launches": int(launches),
        "prefill_ms": round(prefill_ms, 2),
        "ms_per_frame_step": round(step_s * 1e3, 3),
        "roofline": {"bound": "hbm", "kernel": "batched frame step (all kernels: cuBLAS GEMMs over the "
                                               "stacked rows, rows attention, samplers)",
                     "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 3), "traffic": None,
                     "peak_source": pk["source"], "bytes_per_launch": int(step_bytes),
                     "frame_ms_by_kernel": breakdown},
        "clocks": ck,
    }
    st.close()
    return line


def run_reference(args, d: Dist):
    """The reference's CPU implementation (oracle port, reference-faithful),
    rank 0 only, on the same workload: each step is one decode frame after a
    short prefill."""
    wl = configs.WORKLOADS[args.workload]
    if d.rank != 0:
        return None
    # the model file comes from the oracle's build of the synthetic writer, so
    # that this process maps only oracle/ libraries
    synth_lib = ROOT / "oracle" / "libs2o_synth.so"
    if not synth_lib.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle")], check=True, capture_output=True)
    path = ensure_model(d, wl, args.model_dir, lib_path=synth_lib)
    prompt_len = 16
    spf, cores, t_prefill = oracle_frames(path, wl, frames=max(args.steps, 1),
                                          warmup=args.warmup, prompt_len=prompt_len)
    v = round(1.0 / spf, 4)
    return {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": d.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(spf * 1e3, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init S2-Pro-shaped GGUF)",
        "config": {"workload": f"{args.workload}: full-size {WTYPE[wl.model.linear_type]} S2-Pro-shaped "
                               f"Dual-AR, greedy, batch 1 (CPU sample: {prompt_len}-token prompt instead "
                               f"of {wl.prompt_len}, one decode frame per step)",
                   "global_batch": 1, "seq_len": prompt_len + args.steps + args.warmup,
                   "parallelism": "host threads"},
        "impl": "reference",
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{args.steps} timed decode frames after {args.warmup} "
                                   f"warm-up frames and a {prompt_len}-token prefill "
                                   f"({t_prefill:.1f} s), reference-faithful CPU oracle"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


class _Single:
    """One process and no process group (the CPU reference arm)."""
    world = 1
    rank = 0
    local = 0

    def barrier(self):
        pass

    def max(self, v: float) -> float:
        return v

    def sum(self, v: float) -> float:
        return v


def main():
    args = parse()
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return 0
        line = run_reference(args, _Single())
        print(json.dumps(line), flush=True)
        return 0
    d = Dist(args.gpus)
    if args.codec_only:
        try:
            line = run_codec(args, d)
            if d.rank == 0:
                print(json.dumps(line), flush=True)
        finally:
            d.close()
        return 0
    nested_keys = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "dtype",
                   "scaling", "prefill_ms", "e2e", "gpu_launches", "roofline", "config", "clocks")
    try:
        wl = {**configs.WORKLOADS, **configs.PROFILING}[args.workload]
        use_tp = d.world > 1 and (args.tp or not args.replicas) and wl.batch == 1
        line = run_batch(args, d, wl) if wl.batch > 1 else run_ours(args, d, use_tp=use_tp)
        default_c2 = args.workload == "C2"
        # under torchrun the tensor-parallel run heads the line; the replica
        # run (the same workload, one utterance per rank) is nested beside it
        if use_tp and default_c2:
            r = run_ours(args, d, use_tp=False, cpu_baseline=False)
            line["replicas"] = {k: r[k] for k in nested_keys if k in r}
        # the headline metric is frames/s at batch 1 and batch 64: the default
        # C2 run also measures the batch-64 workload (C4) and nests its line
        if default_c2 and not args.no_batch64:
            try:
                b = run_batch(args, d, configs.C4, name="C4", steps=min(args.steps, 10),
                              warmup=min(args.warmup, 3))
                line["batch64"] = {k: b[k] for k in nested_keys + ("ms_per_frame_step",) if k in b}
            except Exception as e:  # the batch-1 line stands on its own
                line["batch64"] = {"metric": METRIC_BATCH, "error": repr(e)[:300]}
        # continuous batching on the batch-64 model (requests joining and leaving)
        if default_c2 and not args.no_serving:
            try:
                line["serving"] = run_serving(args, d, configs.C4)
            except Exception as e:
                line["serving"] = {"metric": METRIC_BATCH, "error": repr(e)[:300]}
        # the codec decode after the token loop (codes -> PCM)
        if default_c2 and not args.no_codec:
            try:
                line["codec"] = run_codec(args, d)
            except Exception as e:
                line["codec"] = {"metric": "codec_samples_per_s", "error": repr(e)[:300]}
        # the quantized batch-1 configurations, on one GPU, over a few steps
        if default_c2 and d.world == 1 and not args.no_quant:
            for key, name in (("q8_0", "C3"), ("q4_k", "C5")):
                try:
                    q = run_ours(args, d, wl_name=name, steps=min(args.steps, 5),
                                 warmup=min(args.warmup, 3), cpu_baseline=False)
                    line[key] = {k: q[k] for k in nested_keys if k in q}
                    line[key]["parity"] = ("quantized parity is pinned to the oracle's restatement of "
                                           "ggml's published block format only")
                except Exception as e:
                    line[key] = {"metric": METRIC, "error": repr(e)[:300]}
        if d.rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        d.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
