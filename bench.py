#!/usr/bin/env python
"""Benchmark of soraku-TTS's per-frame decode loop on B200.

Metric: decode frames/s at batch 1 with CFG (cond + uncond
rows), RTF, and the HBM roofline fraction.  Workload at N=1: config 2 of
BASELINE.json -- 96 text tokens (+ BOS) and a 144-frame reference block,
600 decoded frames (context 242 -> 842 cond, 146 -> 746 uncond), CFG 1.5,
temperature 0.9, top-k 50, top-p 0.95; random-init weights (seed 42) of the
28-layer talker.  EOS is masked (min_new_frames = max_new_frames) so every
utterance decodes exactly 600 frames.

One step = one utterance: its prefill (timed separately, reported as
prefill_ms) and its 600 decode frames.  ``value`` is decode frames/s from
CUDA events around the decode graph replays, with the prompt already resident
on the device; each frame streams ~2.1 GB (weights + KV), far more than L2,
so no L2 flush is needed between frames.  ``e2e`` is the same metric through
FastGenerator.generate with host buffers: prefill, decode and every
host<->device copy inside the wall-clock region.

With --gpus N (torchrun, one process per GPU) every rank decodes its own
utterance (replicas, no data-path collective); ``value`` is the sum of all
ranks' frames over the slowest rank's time (weak scaling).  NCCL carries only
the timing reduction.

--impl reference times the reference's native FP32 CPU algorithm (the
oracle port in oracle/model_np.py; the reference is Python and cannot be
installed on the GPU box) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "decode frames/s & RTF per B200 (bs1 CFG), HBM GB/s % peak; batched fr/s @1-8"
FRAME_RATE = 12.5  # codec frames per second of audio
WORKLOADS = {
    "config2": dict(n_text=96, n_ref=144, frames=600),
    "config1": dict(n_text=48, n_ref=72, frames=150),
    # 64 requests with ragged prompts decoded together (128 CFG rows), split
    # by request over the GPUs
    "config4": dict(requests=64, frames=250, text=(16, 96), ref=(24, 144)),
}
SAMPLING = dict(cfg_scale=1.5, temperature=0.9, top_k=50, top_p=0.95)
BOS_TEXT = 151643
KV_BYTES_PER_POS_ROW = 229_376  # 28 layers x 2 (K,V) x 8 heads x 128 x 4 B


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config2")
    ap.add_argument("--frames", type=int, default=0, help="override decoded frames per utterance")
    ap.add_argument("--fpg", type=int, default=8, help="frames per graph replay")
    ap.add_argument("--cpu-frames", type=int, default=24, help="frames per CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--no-prefetch", action="store_true")
    ap.add_argument("--kernel-only", action="store_true", help="time only the dominant kernel (for ncu captures)")
    ap.add_argument("--profile-frame", action="store_true",
                    help="config4 only: prefill every request, then one NVTX range 'prefill' around the last "
                         "request's prefill and one range 'decode' around a single frame (for ncu --nvtx "
                         "captures); prints no JSON line")
    ap.add_argument("--requests", type=int, default=0, help="override the number of requests (config4)")
    return ap.parse_args()


def make_inputs(seed: int, n_text: int, n_ref: int):
    rng = np.random.default_rng(seed)
    ids = np.concatenate([[BOS_TEXT], rng.integers(0, BOS_TEXT, n_text)]).astype(np.int64)[None]
    uncond = np.array([[BOS_TEXT]], dtype=np.int64)
    prompt = rng.integers(0, 2048, size=(n_ref, 16)).astype(np.int64)
    return ids, uncond, prompt


def bytes_per_frame(weights_bytes: int, n_text: int, n_ref: int, frames: int) -> float:
    """Algorithmic HBM bytes per frame averaged over the utterance: every
    weight once (both CFG rows share the pass) + the KV cache read."""
    lc0 = 1 + n_text + 1 + n_ref
    lu0 = 1 + 1 + n_ref
    mean_pos = (lc0 + lu0) + (frames - 1)  # sum over both rows of the mean cached length
    return weights_bytes + KV_BYTES_PER_POS_ROW * mean_pos


def measured_peak_hbm():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join("/tmp", f"skb_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


GATEUP_PROFILE = os.path.join(HERE, "profiles", "gemv_swiglu_m2_trunk_gateup.md")


def time_gateup_kernel(params, n_layers: int, reps: int = 10):
    """The dominant decode kernel timed alone: the trunk gate/up SwiGLU GEMV
    (M = 2 CFG rows, 2 x 3072 x 1024 FP32 weights) over every layer's weights
    back to back (28 x 25.2 MB, far more than L2), recorded as a CUDA graph so
    host launch overhead stays out of the CUDA-event timing.  Returns (ms per
    launch, algorithmic bytes per launch)."""
    import torch

    from soraku_tts_b200 import kernels as K

    x = torch.randn(2, 1024, device="cuda")
    k_su = K.swiglu_gemv(2, 3072, 1024)
    layers = [(params[f"trunk.layers.{i}.mlp.gate_proj.weight"], params[f"trunk.layers.{i}.mlp.up_proj.weight"])
              for i in range(n_layers)]
    for wg, wu in layers:
        k_su(x, wg, wu)
    torch.cuda.synchronize()
    kgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(kgraph):
        for wg, wu in layers:
            k_su(x, wg, wu)
    kgraph.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ka.record(stream)
    for _ in range(reps):
        kgraph.replay()
    kb.record(stream)
    torch.cuda.synchronize()
    k_ms = ka.elapsed_time(kb) / (reps * len(layers))
    del kgraph
    k_bytes = 2 * 3072 * 1024 * 4 + 2 * 1024 * 4 + 2 * 3072 * 4
    return k_ms, k_bytes


def profiled_traffic():
    """DRAM bytes (read + write) per launch of the gate/up GEMV from the
    committed ncu summary (its line 'dram_bytes_per_launch: N'), else None."""
    try:
        with open(GATEUP_PROFILE) as f:
            for line in f:
                if line.strip().startswith("dram_bytes_per_launch:"):
                    return int(line.split(":", 1)[1].strip().replace(",", ""))
    except OSError:
        pass
    return None


def kernel_only_main(args):
    """--kernel-only: just the dominant kernel's timing on random weights of
    the trunk's gate/up shape (a small command for ncu captures)."""
    import torch

    torch.cuda.set_device(0)
    n_layers = 28
    g = torch.Generator(device="cuda")
    g.manual_seed(42)
    params = {}
    for i in range(n_layers):
        for nm in ("gate_proj", "up_proj"):
            params[f"trunk.layers.{i}.mlp.{nm}.weight"] = torch.randn(3072, 1024, device="cuda", generator=g) * 0.02
    k_ms, k_bytes = time_gateup_kernel(params, n_layers)
    peak, peak_kind = measured_peak_hbm()
    gbs = k_bytes / (k_ms * 1e-3) / 1e9
    print(json.dumps({"kernel": "rgemv_kernel swiglu M=2 3072x1024", "launch_ms": round(k_ms, 5),
                      "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4), "peak_kind": peak_kind}), flush=True)
    return 0


# ----------------------------------------------------------------- reference
def run_reference(args, wl):
    """The reference's native FP32 algorithm on the host cores (oracle port)."""
    import torch
    from threadpoolctl import threadpool_info

    from oracle.model_np import OracleModel
    from soraku_tts_b200.config import ModelDims
    from soraku_tts_b200.weights import random_state_dict, rope_inv_freq

    dims = ModelDims()
    sd = random_state_dict(dims, 42)
    orc = OracleModel(sd, dims, rope_inv_freq(dims).numpy())
    del sd
    n = args.cpu_frames
    ids, uncond, prompt = make_inputs(1000, wl["n_text"], wl["n_ref"])
    decode_s, prefill_s = [], []
    for step in range(args.warmup + args.steps):
        t = {}
        orc.generate(input_ids=ids[0], prompt_codes=prompt, uncond_input_ids=uncond[0], max_new_frames=n,
                     min_new_frames=n, seed=step, timings=t, **SAMPLING)
        if step >= args.warmup:
            decode_s.append(t["decode_s"])
            prefill_s.append(t["prefill_s"])
    fps = n * len(decode_s) / sum(decode_s)
    threads = max([p.get("num_threads", 1) for p in threadpool_info()] + [1])
    del torch
    return fps, statistics.mean(decode_s), statistics.mean(prefill_s), threads


def reference_main(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    fps, dec_s, pre_s, threads = run_reference(args, wl)
    sample = (f"{args.cpu_frames} decode frames per step of {args.workload} (context from "
              f"{2 + wl['n_text'] + wl['n_ref']} positions), after its 2-branch prefill")
    line = {
        "metric": METRIC, "value": round(fps, 4), "unit": "frames/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dec_s * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "frames_per_step": args.cpu_frames,
                   "prefill_ms": round(pre_s * 1e3, 1), "rtf": round(FRAME_RATE / fps, 4),
                   "model": "soraku-TTS v2 talker (Qwen3 28L d1024) + depth head, random-init seed 42"},
        "impl": "reference",
        "cpu_baseline": {"value": round(fps, 4), "unit": "frames/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(fps, 4), "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------- b200
def b200_main(args, wl):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    from soraku_tts_b200 import _lib
    from soraku_tts_b200.config import ModelDims
    from soraku_tts_b200.fast_generate import FastGenerator
    from soraku_tts_b200.model import SorakuModel

    frames = args.frames or wl["frames"]
    fpg = args.fpg
    if frames % fpg:
        raise SystemExit(f"--frames {frames} must be a multiple of --fpg {fpg}")
    dims = ModelDims()
    model = SorakuModel.random(dims, 42, f"cuda:{local}")
    weights_bytes = sum(t.numel() * 4 for k, t in model.params.items() if k != "trunk.embed_tokens.weight")
    gen = FastGenerator(model, device=torch.device("cuda", local), frames_per_graph=fpg,
                        use_pdl=not args.no_pdl, l2_prefetch=not args.no_prefetch)
    ids, uncond, prompt = make_inputs(1000 + rank, wl["n_text"], wl["n_ref"])
    gkw = dict(max_new_frames=frames, min_new_frames=frames, **SAMPLING)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        from soraku_tts_b200.batching import max_over_ranks as mor

        return mor(v, device="cuda")

    # warm-up through the public API (builds the engine and its graph)
    for w in range(args.warmup):
        gen.generate(input_ids=torch.from_numpy(ids), prompt_codes=torch.from_numpy(prompt),
                     uncond_input_ids=torch.from_numpy(uncond), seed=w, **gkw)
    eng = gen._engine
    stream = torch.cuda.current_stream()

    # ---- device-resident decode throughput (value)
    clocks = ClockSampler(local)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    pev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    clocks.start()
    t_wall0 = time.perf_counter()
    for s in range(args.steps):
        eng.set_sampling(0, cfg=SAMPLING["cfg_scale"], temperature=0.9, temperature_q0=0.9, top_k=50, top_p=0.95,
                         top_k_q0=50, top_p_q0=0.95, seed=100 + s, min_new_frames=frames, eos_rule=1)
        pev[s][0].record(stream)
        eng.prefill(0, ids, uncond, prompt)
        pev[s][1].record(stream)
        ev[s][0].record(stream)
        for _ in range(frames // fpg):
            eng.step(True)
        ev[s][1].record(stream)
    barrier()
    t_wall = time.perf_counter() - t_wall0
    clk = clocks.stop()
    dec_ms = [a.elapsed_time(b) for a, b in ev]
    pre_ms = [a.elapsed_time(b) for a, b in pev]
    dec_total_s = max_over_ranks(sum(dec_ms) / 1e3)
    value = world * args.steps * frames / dec_total_s
    codes_check = eng.read_codes(0, 0, frames).clone()
    assert codes_check.shape == (frames, 16) and int(codes_check.max()) < 2048 and int(codes_check.min()) >= 0

    # ---- end to end through the public API with host buffers
    barrier()
    t0 = time.perf_counter()
    for s in range(args.steps):
        codes, info = gen.generate(input_ids=torch.from_numpy(ids), prompt_codes=torch.from_numpy(prompt),
                                   uncond_input_ids=torch.from_numpy(uncond), seed=200 + s, **gkw)
        assert info["num_frames"] == frames
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = world * args.steps * frames / e2e_s
    h2d = int(ids.nbytes + uncond.nbytes + prompt.nbytes)
    d2h = int(frames * 16 * 8)

    k_ms, k_bytes = time_gateup_kernel(model.params, dims.trunk.num_hidden_layers)
    peak, peak_kind = measured_peak_hbm()
    k_gbs = k_bytes / (k_ms * 1e-3) / 1e9
    bpf = bytes_per_frame(weights_bytes, wl["n_text"], wl["n_ref"], frames)
    frame_ms = dec_total_s * 1e3 / (args.steps * frames)
    f_gbs = bpf / (frame_ms * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        class A:  # bounded sample: 1 warm-up-free step
            pass
        a = A()
        a.warmup, a.steps, a.cpu_frames, a.workload = 0, 1, args.cpu_frames, args.workload
        fps, dec_s, pre_s, threads = run_reference(a, wl)
        cpu = {"value": round(fps, 4), "unit": "frames/s", "cores": threads, "kind": "port",
               "sample": f"{args.cpu_frames} decode frames of {args.workload} after its prefill "
                         f"({dec_s:.1f} s decode, {pre_s:.1f} s prefill), oracle/model_np.py"}

    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(statistics.mean(dec_ms), 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {
            "workload": f"{args.workload}: {wl['n_text']} text + {wl['n_ref']} ref frames, {frames} decode frames, "
                        "bs1 CFG 1.5, T 0.9, top-k 50, top-p 0.95",
            "model": "soraku-TTS v2 talker (Qwen3 28L d1024 16/8 heads, FFN 3072) + depth head, random-init seed 42",
            "global_batch": world, "rows_per_gpu": 2, "seq_len": 2 + wl["n_text"] + wl["n_ref"] + frames,
            "parallelism": "replicas" if world > 1 else "single",
            "frames_per_graph": fpg, "pdl": not args.no_pdl, "l2_prefetch": not args.no_prefetch,
            "rtf": round(FRAME_RATE / (value / world), 5), "prefill_ms": round(statistics.mean(pre_ms), 2),
            "frame_ms": round(frame_ms, 4), "l2": "inputs larger than L2: each frame streams ~2.1 GB",
            "wall_s_value_region": round(t_wall, 3),
        },
        "e2e": {"value": round(e2e, 3), "unit": "frames/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "achieved": round(k_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(k_gbs / peak, 4), "traffic": profiled_traffic(),
                     "kernel": "rgemv_kernel (trunk gate/up SwiGLU GEMV, M=2, 25.2 MB weights/launch)",
                     "peak_kind": peak_kind, "launch_ms": round(k_ms, 5), "bytes_per_launch": k_bytes},
        "roofline_frame": {"bound": "hbm", "achieved": round(f_gbs, 1), "peak": peak, "unit": "GB/s",
                           "frac": round(f_gbs / peak, 4), "bytes_per_frame": int(bpf), "peak_kind": peak_kind},
        "gpu_launches": int(eng.launches_per_step() * (frames // fpg) * args.steps),
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ config 4
def config4_requests(n_req: int, text, ref):
    """Seeded ragged requests: (ids [1, 1+t], uncond [1, 1], prompt [r, 16], seed)."""
    out = []
    for i in range(n_req):
        rng = np.random.default_rng(5000 + i)
        t = int(rng.integers(text[0], text[1] + 1))
        r = int(rng.integers(ref[0], ref[1] + 1))
        ids, uncond, prompt = make_inputs(5000 + i, t, r)
        out.append((ids, uncond, prompt, 7000 + i))
    return out


def split_requests(reqs, frames: int, world: int):
    """Static split balanced on the KV positions a request keeps (prompt
    length + frames)."""
    from soraku_tts_b200.batching import split_requests as split

    return split([r[0].shape[1] + r[2].shape[0] + frames for r in reqs], world)


def profile_frame_main(args, wl):
    """A config-4 engine (requests x 2 rows) for ncu captures: NVTX range
    'prefill' around the last request's prefill, range 'decode' around one
    frame after three warm-up frames."""
    import torch

    from soraku_tts_b200.config import ModelDims
    from soraku_tts_b200.graph_frame import NativeEngine
    from soraku_tts_b200.model import SorakuModel

    n = args.requests or wl["requests"]
    frames = 32
    reqs = config4_requests(n, wl["text"], wl["ref"])
    model = SorakuModel.random(ModelDims(), 42, "cuda:0")
    max_prompt = max(r[0].shape[1] + r[2].shape[0] + 2 for r in reqs)
    max_len = ((max_prompt + frames + 2 + 63) // 64) * 64
    eng = NativeEngine(model, max_requests=n, rows_per_request=2, max_len=max_len, max_frames=frames,
                       max_prefill=max_prompt + 2)
    for j, (ids, uncond, prompt, seed) in enumerate(reqs):
        eng.set_sampling(j, cfg=SAMPLING["cfg_scale"], temperature=0.9, temperature_q0=0.9, top_k=50, top_p=0.95,
                         top_k_q0=50, top_p_q0=0.95, seed=seed, min_new_frames=frames, eos_rule=1)
        last = j == n - 1
        if last:
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_push("prefill")
        eng.prefill(j, ids, uncond, prompt)
        if last:
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_pop()
    eng.capture(n, 1)
    for _ in range(3):
        eng.step(True)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("decode")
    eng.step(True)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    print(f"profile frame: {n} requests, {2 * n} rows, {eng.launches_per_step()} kernels per frame", file=sys.stderr)
    eng.close()
    return 0


def config4_main(args, wl):
    """Batched decode (config 4): every rank decodes its share of the 64
    requests as one batch of 2 rows per request; value = all ranks' frames
    over the slowest rank's decode time (fixed total work: strong scaling)."""
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    from soraku_tts_b200.config import ModelDims
    from soraku_tts_b200.graph_frame import NativeEngine
    from soraku_tts_b200.model import SorakuModel

    frames = args.frames or wl["frames"]
    fpg = max(1, min(args.fpg, frames))
    while frames % fpg:  # a whole number of graph replays per utterance
        fpg -= 1
    reqs = config4_requests(wl["requests"], wl["text"], wl["ref"])
    mine = split_requests(reqs, frames, world)[rank]
    n = len(mine)
    dims = ModelDims()
    model = SorakuModel.random(dims, 42, f"cuda:{local}")
    max_prompt = max(r[0].shape[1] + r[2].shape[0] + 2 for r in reqs)
    max_len = ((max_prompt + frames + 2 + 63) // 64) * 64
    pbatch = min(n, 16)  # prompts per prefill pass
    eng = NativeEngine(model, max_requests=n, rows_per_request=2, max_len=max_len, max_frames=frames,
                       max_prefill=max_prompt + 2, use_pdl=not args.no_pdl, l2_prefetch=not args.no_prefetch,
                       prefill_batch=pbatch)
    stream = torch.cuda.current_stream()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def prefill_all(step):
        for j, i in enumerate(mine):
            ids, uncond, prompt, seed = reqs[i]
            eng.set_sampling(j, cfg=SAMPLING["cfg_scale"], temperature=0.9, temperature_q0=0.9, top_k=50,
                             top_p=0.95, top_k_q0=50, top_p_q0=0.95, seed=seed + 1000 * step,
                             min_new_frames=frames, eos_rule=1)
        for j0 in range(0, n, pbatch):  # several prompts per pass over the trunk
            js = list(range(j0, min(n, j0 + pbatch)))
            eng.prefill_many(js, [reqs[mine[j]][0] for j in js], [reqs[mine[j]][1] for j in js],
                             [reqs[mine[j]][2] for j in js])

    prefill_all(0)
    eng.capture(n, fpg)
    for w in range(args.warmup):
        prefill_all(w)
        for _ in range(frames // fpg):
            eng.step(True)
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    clocks.start()
    for s_ in range(args.steps):
        prefill_all(100 + s_)
        ev[s_][0].record(stream)
        for _ in range(frames // fpg):
            eng.step(True)
        ev[s_][1].record(stream)
    barrier()
    clk = clocks.stop()
    dec_ms = [a.elapsed_time(b) for a, b in ev]
    dec_s = max_over_ranks(sum(dec_ms) / 1e3)
    total_frames = wl["requests"] * frames * args.steps
    value = total_frames / dec_s
    # results: every request's codes on rank 0 (outside the timed region)
    from soraku_tts_b200.batching import gather_codes

    local = {}
    for j, i in enumerate(mine):
        c = eng.read_codes(j, 0, frames).cpu().numpy()
        assert c.shape == (frames, 16) and int(c.max()) < 2048 and int(c.min()) >= 0
        local[i] = c
    merged = gather_codes(local)
    if rank == 0:
        assert sorted(merged) == list(range(wl["requests"])), "a request produced no codes"

    # end to end: prefill from host ids, decode, codes back to host
    barrier()
    t0 = time.perf_counter()
    h2d = d2h = 0
    for s_ in range(args.steps):
        prefill_all(200 + s_)
        for _ in range(frames // fpg):
            eng.step(True)
        for j in range(n):
            eng.read_codes(j, 0, frames).cpu()
            d2h += frames * 16 * 8
    for i in mine:
        h2d += reqs[i][0].nbytes + reqs[i][1].nbytes + reqs[i][2].nbytes
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    launches = int(eng.launches_per_step() * (frames // fpg) * args.steps)
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(statistics.mean(dec_ms), 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {
            "workload": f"config4: {wl['requests']} requests (text U{list(wl['text'])}, ref U{list(wl['ref'])}), "
                        f"{frames} frames each, CFG 1.5, T 0.9, top-k 50, top-p 0.95, split by request over the GPUs",
            "model": "soraku-TTS v2 talker (Qwen3 28L d1024 16/8 heads, FFN 3072) + depth head, random-init seed 42",
            "global_batch": wl["requests"], "rows_per_gpu": 2 * n, "parallelism": f"requests split over {world}",
            "frames_per_graph": fpg, "step_ms_per_frame": round(statistics.mean(dec_ms) / frames, 4),
            "l2": "inputs larger than L2",
        },
        "e2e": {"value": round(total_frames / e2e_s, 1), "unit": "frames/s", "h2d_bytes_per_step": h2d // args.steps,
                "d2h_bytes_per_step": d2h // args.steps},
        "gpu_launches": launches,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    wl = WORKLOADS[args.workload]
    if args.workload == "config4" and args.impl != "reference":
        if args.profile_frame:
            return profile_frame_main(args, wl)
        if args.requests:
            wl = dict(wl, requests=args.requests)
        return config4_main(args, wl)
    if args.impl == "reference":
        return reference_main(args, wl)
    if args.kernel_only:
        return kernel_only_main(args)
    return b200_main(args, wl)


if __name__ == "__main__":
    sys.exit(main())
