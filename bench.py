#!/usr/bin/env python
"""Benchmark of soraku-TTS's per-frame decode loop on B200.

Metric: decode frames/s at batch 1 with CFG (cond + uncond rows), RTF, and
the HBM roofline fraction; batched frames/s of 64 requests split over the
GPUs.  Workload of the headline line (config 2): 96 text tokens (+ BOS) and a
144-frame reference block, 600 decoded frames (context 242 -> 842 cond,
146 -> 746 uncond), CFG 1.5, temperature 0.9, top-k 50, top-p 0.95;
random-init weights (seed 42) of the 28-layer talker.  EOS is masked
(min_new_frames = max_new_frames) so every utterance decodes exactly 600
frames.

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
the timing reduction.  The same line carries ``batched``: config 4 (64
ragged requests, 250 frames each, 128 CFG rows in all) split by request over
the N ranks, aggregate frames/s over the slowest rank (strong scaling), with
its HBM fraction.

--workload config4 prints the batched measurement as its own line;
--workload config5 prints the kernel microbench (RMSNorm, QKV GEMV, SwiGLU
GEMV pair, 16-head classifier, CFG + sampling at M = 1, 2, 8, 64 rows, GB/s
against the measured HBM peak).

--impl reference times the reference's native FP32 CPU algorithm (the
oracle port in oracle/model_np.py, pinned to the reference by tests/golden;
the reference is Python and cannot be installed on the GPU box) on bounded
samples of the same workload and context range.
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
    # kernel microbench: ops at these row counts (FP32 weights N(0, 0.02), seed 3)
    "config5": dict(rows=(1, 2, 8, 64)),
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
    ap.add_argument("--cpu-frames", type=int, default=8, help="decoded frames per CPU-baseline window")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--no-prefetch", action="store_true")
    ap.add_argument("--kernel-only", action="store_true", help="time only the dominant kernel (for ncu captures)")
    ap.add_argument("--profile-frame", action="store_true",
                    help="config4 only: prefill every request, then one NVTX range 'prefill' around the last "
                         "request's prefill and one range 'decode' around a single frame (for ncu --nvtx "
                         "captures); prints no JSON line")
    ap.add_argument("--requests", type=int, default=0, help="override the number of requests (config4)")
    ap.add_argument("--no-batched", action="store_true", help="skip the batched (config 4) record of the default line")
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
_ORACLE = None


def _oracle():
    """The oracle port of the reference's native FP32 path with the benchmark
    model's weights (seed 42), built once per process."""
    global _ORACLE
    if _ORACLE is None:
        from oracle.model_np import OracleModel
        from soraku_tts_b200.config import ModelDims
        from soraku_tts_b200.weights import random_state_dict, rope_inv_freq

        dims = ModelDims()
        sd = random_state_dict(dims, 42)
        _ORACLE = OracleModel(sd, dims, rope_inv_freq(dims).numpy())
    return _ORACLE


def _threads() -> int:
    from threadpoolctl import threadpool_info

    return max([p.get("num_threads", 1) for p in threadpool_info()] + [1])


def cpu_windows(n_text: int, n_ref: int, frames: int, per_window: int, seed: int, step: int):
    """Decode frames/s of the oracle port on the host cores over the context
    range an utterance of `frames` frames covers: one window of `per_window`
    decoded frames at the midpoint of each third of the utterance (the prompt
    extended by F/6, F/2 and 5F/6 reference frames, so the window starts at the
    context the GPU arm reaches there), each after a prefill of that length.
    A frame's cost grows linearly with its context, so the mean over the three
    windows is the utterance's mean.  Returns (frames/s, decode s, prefill s)."""
    orc = _oracle()
    dec = pre = 0.0
    n = 0
    for k, frac in enumerate((1 / 6, 1 / 2, 5 / 6)):
        extra = int(round(frames * frac))
        ids, uncond, prompt = make_inputs(seed, n_text, n_ref + extra)
        t = {}
        orc.generate(input_ids=ids[0], prompt_codes=prompt, uncond_input_ids=uncond[0], max_new_frames=per_window,
                     min_new_frames=per_window, seed=1000 * step + k, timings=t, **SAMPLING)
        dec += t["decode_s"]
        pre += t["prefill_s"]
        n += per_window
    return n / dec, dec, pre


def cpu_sample(args, workload: str, step: int):
    """One bounded CPU sample of a workload: (frames/s, decode s, prefill s, description)."""
    wl = WORKLOADS[workload]
    if workload == "config4":
        # three of the ragged requests, one window each at the middle of its 250 frames
        reqs = config4_requests(3, wl["text"], wl["ref"])
        dec = pre = 0.0
        n = 0
        orc = _oracle()
        for i, (ids, uncond, prompt, seed) in enumerate(reqs):
            extra = wl["frames"] // 2
            rng = np.random.default_rng(seed)
            more = rng.integers(0, 2048, size=(extra, 16)).astype(np.int64)
            t = {}
            orc.generate(input_ids=ids[0], prompt_codes=np.concatenate([prompt, more]), uncond_input_ids=uncond[0],
                         max_new_frames=args.cpu_frames, min_new_frames=args.cpu_frames, seed=seed + 1000 * step,
                         timings=t, **SAMPLING)
            dec += t["decode_s"]
            pre += t["prefill_s"]
            n += args.cpu_frames
        desc = (f"{args.cpu_frames} decode frames of each of config4 requests 0-2 (one request at a time, both CFG "
                f"branches) at the middle of their {wl['frames']} frames, after a prefill of that length; "
                "oracle/model_np.py")
        return n / dec, dec, pre, desc
    fps, dec, pre = cpu_windows(wl["n_text"], wl["n_ref"], wl["frames"], args.cpu_frames, 1000, step)
    lc0 = 2 + wl["n_text"] + wl["n_ref"]
    ctx = [lc0 + int(round(wl["frames"] * f)) for f in (1 / 6, 1 / 2, 5 / 6)]
    desc = (f"{args.cpu_frames} decode frames at each of cond contexts {ctx} (the midpoints of the thirds of "
            f"{workload}'s {lc0}->{lc0 + wl['frames']} range) after prefills of those lengths; oracle/model_np.py")
    return fps, dec, pre, desc


def reference_main(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    work = "config2" if args.workload == "config5" else args.workload
    dec_s, pre_s = [], []
    desc = ""
    n_frames = 0
    for step in range(args.warmup + args.steps):
        fps, dec, pre, desc = cpu_sample(args, work, step)
        if step >= args.warmup:
            dec_s.append(dec)
            pre_s.append(pre)
            n_frames += int(round(fps * dec))
    fps = n_frames / sum(dec_s)
    threads = _threads()
    line = {
        "metric": METRIC, "value": round(fps, 4), "unit": "frames/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(statistics.mean(dec_s) * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": work, "prefill_ms": round(statistics.mean(pre_s) * 1e3, 1),
                   "rtf": round(FRAME_RATE / fps, 4),
                   "model": "soraku-TTS v2 talker (Qwen3 28L d1024) + depth head, random-init seed 42"},
        "impl": "reference",
        "cpu_baseline": {"value": round(fps, 4), "unit": "frames/s", "cores": threads, "kind": "port",
                         "sample": desc},
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

    launches = int(eng.launches_per_step() * (frames // fpg) * args.steps)
    # batched requests (config 4) split over the same ranks: the multi-GPU curve
    batched = None
    if not args.no_batched:
        del gen, eng
        torch.cuda.empty_cache()
        wl4 = WORKLOADS["config4"]
        r = run_config4(args, wl4, model, dist, world, rank, args.steps, args.warmup)
        batched = {
            "workload": f"config4: {wl4['requests']} requests (text U{list(wl4['text'])}, ref U{list(wl4['ref'])}), "
                        f"{r['frames']} frames each, CFG 1.5, split by request over the GPUs",
            "value": round(r["value"], 1), "unit": "frames/s", "scaling": "strong", "n_gpus": world,
            "rows_per_gpu": r["rows"], "ms_per_frame_step": round(r["step_ms"], 4),
            "ms_per_step": round(statistics.mean(r["dec_ms"]), 3),
            "e2e": {"value": round(r["e2e"], 1), "unit": "frames/s", "h2d_bytes_per_step": r["h2d"],
                    "d2h_bytes_per_step": r["d2h"]},
            "roofline": r["roofline"], "gpu_launches": r["launches"],
        }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        fps, dec_s, pre_s, desc = cpu_sample(args, args.workload, 0)
        cpu = {"value": round(fps, 4), "unit": "frames/s", "cores": _threads(), "kind": "port",
               "sample": f"{desc} ({dec_s:.1f} s decode, {pre_s:.1f} s prefill)"}

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
                     "traffic_source": "prior ncu capture of the same kernel and shape "
                                       "(profiles/gemv_swiglu_m2_trunk_gateup.md), not this run",
                     "kernel": "rgemv_kernel (trunk gate/up SwiGLU GEMV, M=2, 25.2 MB weights/launch)",
                     "peak_kind": peak_kind, "launch_ms": round(k_ms, 5), "bytes_per_launch": k_bytes},
        "roofline_frame": {"bound": "hbm", "achieved": round(f_gbs, 1), "peak": peak, "unit": "GB/s",
                           "frac": round(f_gbs / peak, 4), "bytes_per_frame": int(bpf), "peak_kind": peak_kind},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if batched is not None:
        line["batched"] = batched
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


def config4_kv_bytes(reqs, mine, frames: int) -> float:
    """Mean KV bytes one frame step reads for this rank's requests: every
    cached position of every row, averaged over the utterance."""
    total = 0.0
    for i in mine:
        ids, uncond, prompt, _ = reqs[i]
        for L in (ids.shape[1] + 1 + prompt.shape[0], uncond.shape[1] + 1 + prompt.shape[0]):
            total += L + (frames - 1) / 2
    return KV_BYTES_PER_POS_ROW * total


def run_config4(args, wl, model, dist, world, rank, steps, warmup, clocks=None):
    """Batched decode (config 4) on this rank: its share of the requests
    (split by request, longest first to the least-loaded rank) as one batch of
    2 rows per request.  Returns a dict of the measurements; `value` is all
    ranks' frames over the slowest rank's decode time (strong scaling)."""
    import torch

    from soraku_tts_b200.batching import gather_codes
    from soraku_tts_b200.graph_frame import NativeEngine

    frames = args.frames if (args.frames and args.workload == "config4") else wl["frames"]
    fpg = max(1, min(args.fpg, frames))
    while frames % fpg:  # a whole number of graph replays per utterance
        fpg -= 1
    reqs = config4_requests(wl["requests"], wl["text"], wl["ref"])
    mine = split_requests(reqs, frames, world)[rank]
    n = len(mine)
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
    for w in range(warmup):
        prefill_all(w)
        for _ in range(frames // fpg):
            eng.step(True)
    torch.cuda.synchronize()

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    barrier()
    if clocks is not None:
        clocks.start()
    for s_ in range(steps):
        prefill_all(100 + s_)
        ev[s_][0].record(stream)
        for _ in range(frames // fpg):
            eng.step(True)
        ev[s_][1].record(stream)
    barrier()
    clk = clocks.stop() if clocks is not None else None
    dec_ms = [a.elapsed_time(b) for a, b in ev]
    dec_s = max_over_ranks(sum(dec_ms) / 1e3)
    total_frames = wl["requests"] * frames * steps
    # results: every request's codes on rank 0 (outside the timed region)
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
    for s_ in range(steps):
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
    launches = int(eng.launches_per_step() * (frames // fpg) * steps)
    eng.close()
    weights_bytes = sum(t.numel() * 4 for k, t in model.params.items() if k != "trunk.embed_tokens.weight")
    step_ms = statistics.mean(dec_ms) / frames  # this rank's mean ms per frame step
    bytes_step = weights_bytes + config4_kv_bytes(reqs, mine, frames)
    peak, peak_kind = measured_peak_hbm()
    gbs = bytes_step / (step_ms * 1e-3) / 1e9
    return {
        "value": total_frames / dec_s, "frames": frames, "fpg": fpg, "rows": 2 * n, "requests_here": n,
        "dec_ms": dec_ms, "step_ms": step_ms, "e2e": total_frames / e2e_s, "h2d": h2d // steps,
        "d2h": d2h // steps, "launches": launches, "clocks": clk,
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "bytes_per_step": int(bytes_step), "peak_kind": peak_kind,
                     "note": "rank 0's frame step: every weight once + the KV of its rows"},
    }


def config4_main(args, wl):
    """Batched decode (config 4) as its own line."""
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
    from soraku_tts_b200.model import SorakuModel

    model = SorakuModel.random(ModelDims(), 42, f"cuda:{local}")
    r = run_config4(args, wl, model, dist, world, rank, args.steps, args.warmup, ClockSampler(local))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    frames = r["frames"]
    line = {
        "metric": METRIC, "value": round(r["value"], 1), "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(statistics.mean(r["dec_ms"]), 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {
            "workload": f"config4: {wl['requests']} requests (text U{list(wl['text'])}, ref U{list(wl['ref'])}), "
                        f"{frames} frames each, CFG 1.5, T 0.9, top-k 50, top-p 0.95, split by request over the GPUs",
            "model": "soraku-TTS v2 talker (Qwen3 28L d1024 16/8 heads, FFN 3072) + depth head, random-init seed 42",
            "global_batch": wl["requests"], "rows_per_gpu": r["rows"], "parallelism": f"requests split over {world}",
            "frames_per_graph": r["fpg"], "step_ms_per_frame": round(r["step_ms"], 4),
            "l2": "inputs larger than L2",
        },
        "e2e": {"value": round(r["e2e"], 1), "unit": "frames/s", "h2d_bytes_per_step": r["h2d"],
                "d2h_bytes_per_step": r["d2h"]},
        "roofline": r["roofline"],
        "gpu_launches": r["launches"],
        "clocks": r["clocks"],
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ config 5
def config5_main(args, wl):
    """Kernel microbench: RMSNorm on 1024-vectors, the QKV GEMV 1024 -> 4096,
    the SwiGLU GEMV pair 1024 -> 2 x 3072 -> 1024, the 16-head classifier
    1024 -> 16 x 2048 in one launch (the 16 codebook tables stacked into one
    [32768, 1024] matrix), and the fused CFG + top-k 50 / top-p 0.95 sampler over
    the 16 heads, each at M = 1, 2, 8, 64 rows (M <= 4 runs the ring GEMV,
    larger M the 3xTF32 tensor-core GEMM).  FP32 weights N(0, 0.02), seed 3.
    Several weight copies are rotated so that every launch reads its weights
    from HBM (the copies together hold more than 3x L2); each op's launches are
    recorded once as a CUDA graph and timed over its replays with CUDA events.
    GB/s = (weight + activation bytes) / launch time."""
    import math

    import torch

    from soraku_tts_b200 import kernels as K

    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)

    def rnd(*shape):
        return torch.randn(*shape, device="cuda", generator=g) * 0.02

    D, NQKV, F, V, HEADS = 1024, 4096, 3072, 2048, 16
    l2 = 126e6
    peak, peak_kind = measured_peak_hbm()

    def n_copies(nbytes):
        return max(2, int(math.ceil(3 * l2 / nbytes)))

    def time_calls(calls, reps=10):
        """ms per call of a list of zero-argument callables replayed as one graph."""
        for c in calls:
            c()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for c in calls:
                c()
        graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            graph.replay()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / (reps * len(calls))
        del graph
        return ms

    w_qkv = [rnd(NQKV, D) for _ in range(n_copies(NQKV * D * 4))]
    b_qkv = torch.zeros(NQKV, device="cuda")
    n_sw = n_copies(3 * F * D * 4)
    w_g = [rnd(F, D) for _ in range(n_sw)]
    w_u = [rnd(F, D) for _ in range(n_sw)]
    w_d = [rnd(D, F) for _ in range(n_sw)]
    n_cls = n_copies(HEADS * V * D * 4)
    w_cls = [rnd(HEADS * V, D) for _ in range(n_cls)]
    b_cls = rnd(HEADS * V)
    norm_w = 1.0 + rnd(D)
    ops = {}
    for M in wl["rows"]:
        x = torch.randn(M, D, device="cuda", generator=g)
        res = {}

        def rec(name, ms, nbytes):
            gbs = nbytes / (ms * 1e-3) / 1e9
            res[name] = {"us": round(ms * 1e3, 3), "bytes": int(nbytes), "gbs": round(gbs, 1),
                         "frac": round(gbs / peak, 4)}

        k_norm = K.rmsnorm(M, D, 1e-6)
        rec("rmsnorm", time_calls([lambda: k_norm(x, norm_w)] * 32), 2 * M * D * 4 + D * 4)
        k_qkv = K.classifier_gemv(M, NQKV, D)
        rec("qkv_gemv", time_calls([lambda w=w: k_qkv(x, w, b_qkv) for w in w_qkv]),
            NQKV * D * 4 + NQKV * 4 + M * (D + NQKV) * 4)
        k_su = K.swiglu_gemv(M, F, D)
        k_dn = K.down_residual_gemv(M, D, F)
        act = torch.randn(M, F, device="cuda", generator=g)
        rec("swiglu_gate_up", time_calls([lambda a=a, b=b: k_su(x, a, b) for a, b in zip(w_g, w_u)]),
            2 * F * D * 4 + M * (D + F) * 4)
        rec("down_residual", time_calls([lambda w=w: k_dn(act, w, x) for w in w_d]), F * D * 4 + M * (F + 2 * D) * 4)
        rec("swiglu_pair", time_calls([lambda a=a, b=b, c=c: k_dn(k_su(x, a, b), c, x)
                                       for a, b, c in zip(w_g, w_u, w_d)]),
            3 * F * D * 4 + M * (2 * D + 2 * F + D) * 4)
        k_cls = K.classifier_gemv(M, HEADS * V, D)
        rec("classifier_16heads", time_calls([lambda w=w: k_cls(x, w, b_cls) for w in w_cls]),
            HEADS * V * D * 4 + HEADS * V * 4 + M * (D + HEADS * V) * 4)
        # CFG + sampling of every head: CFG pairs of rows (one row without CFG)
        rpr = 2 if M >= 2 else 1
        n_req = HEADS * (M // rpr)
        vs = V + 3
        logits = torch.randn(n_req * rpr, vs, device="cuda", generator=g) * 2.0
        params = K.pack_sample_params([dict(cfg_scale=1.5 if rpr == 2 else 1.0, temperature=0.9, top_k=50,
                                            top_p=0.95, mask_eos=True, request=i, q=i % HEADS, seed=3, V=vs)
                                       for i in range(n_req)])
        rec("cfg_sample_16heads", time_calls([lambda: K.cfg_sample(logits, params, rows_per_req=rpr, bos_id=V,
                                                                  pad_id=V + 2, eos_id=V + 1)] * 16),
            n_req * rpr * vs * 4)
        ops[f"M={M}"] = res

    # CPU reference of the same ops at M = 2 (numpy FP32 on the host cores)
    cpu = None
    if not args.no_cpu_baseline:
        xs = np.random.default_rng(3).standard_normal((2, D)).astype(np.float32)
        wq = np.random.default_rng(4).standard_normal((NQKV, D)).astype(np.float32) * 0.02
        wc = np.random.default_rng(5).standard_normal((HEADS * V, D)).astype(np.float32) * 0.02
        t0 = time.perf_counter()
        reps = 20
        for _ in range(reps):
            xs @ wc.T
        cls_s = (time.perf_counter() - t0) / reps
        t0 = time.perf_counter()
        for _ in range(reps):
            xs @ wq.T
        qkv_s = (time.perf_counter() - t0) / reps
        cpu = {"value": round(HEADS * V * D * 4 / cls_s / 1e9, 2), "unit": "GB/s", "cores": _threads(),
               "kind": "port",
               "sample": f"numpy FP32 matmul at M=2: 16-head classifier {cls_s * 1e3:.2f} ms, "
                         f"QKV {qkv_s * 1e3:.2f} ms per call ({reps} calls each)"}
    head = ops["M=2"]["classifier_16heads"]
    line = {
        "metric": "config5 kernel microbench: HBM GB/s per op and row count (classifier_16heads at M=2 as value)",
        "value": head["gbs"], "unit": "GB/s", "n_gpus": 1, "steps": 10, "warmup": 1,
        "ms_per_step": round(head["us"] / 1e3, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config5: RMSNorm d=1024, QKV 1024->4096, SwiGLU 1024->2x3072->1024, 16-head "
                               "classifier 1024->16x2048 + CFG/top-k 50/top-p 0.95, M in {1, 2, 8, 64}",
                   "weights": "FP32 N(0, 0.02) seed 3, rotated copies > 3x L2 per op", "peak_kind": peak_kind,
                   "peak_gbs": peak, "l2": "weight copies rotated, together more than 3x L2"},
        "ops": ops,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    wl = WORKLOADS[args.workload]
    if args.workload == "config5" and args.impl != "reference":
        return config5_main(args, wl)
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
