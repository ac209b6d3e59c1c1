#!/usr/bin/env python
"""Codec frames/s of qwen3-tts.cpp's per-frame codec-token loop on B200.

Workload (default): BASELINE.json configs[0] — greedy F16 frame loop, batch 1,
seeded random-init GGUF with the 0.6B layout, ICL prompt with 55 reference
frames (64 talker prefill positions), 32 frames per utterance, repetition
penalty 1.05, EOS suppressed by eos_bias = -1e9.  `--config q8` runs
configs[1] (Q8_0, 128 prefill, 256 frames).

A step = one codec frame: codebook-0 sampling, the 2-token code-predictor
prefill, 14 code-predictor steps with on-device sampling, the next-step
embedding sum and one 28-layer talker step.  The K timed steps are K / F
replays of the config's F-frame utterance (each replay rewinds the device
frame state to frame 0 after the prefill).  Each rank runs its own utterance
on its own GPU (weak scaling, no collective on the data path); the timed
region is bracketed by a barrier + synchronize and the device time is the max
over ranks.  Every frame streams 3.3 GB of weights (> 126 MB L2), so no L2
flush is needed between steps.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "qwen3-tts.cpp_b200")
sys.path.insert(0, ROOT)

METRIC = "codec frames/s"
UNIT = "frames/s"
# Algorithmic bytes per frame per sequence: every weight byte of the talker step and
# of the 15 code-predictor passes once; KV added per frame below.
WEIGHT_BYTES = {"f16": 3_309_305_856, "q8": 1_790_509_056}
KV_TALKER_PER_POS = 114_688      # 28 layers x (K+V) x 8 heads x 128 x 2 B
KV_CP_PER_POS = 20_480           # 5 layers x (K+V) x 8 x 128 x 2 B
CONFIGS = {
    "f16": dict(wtype="f16", n_ref=55, prefill=64, frames=32,
                workload="BASELINE configs[0]: greedy F16 frame loop, batch 1, ICL prefill 64, 32 frames, rep 1.05"),
    "q8": dict(wtype="q8_0", n_ref=119, prefill=128, frames=256,
               workload="BASELINE configs[1]: greedy Q8_0 frame loop, batch 1, ICL prefill 128, 256 frames, rep 1.05"),
    "batch": dict(wtype="f16", n_utts=64, p_lo=32, p_hi=512, frames=1024,
                  workload="BASELINE configs[3]: batched F16 serving, 64 utterances, ICL prefill U[32,512], "
                           "1024 greedy frames each, paged F16 KV, tcgen05 GEMMs"),
    "q8long": dict(wtype="q8_0", utts_per_gpu=32, p_lo=512, p_hi=512, frames=4096, e2e_frames=256,
                   workload="BASELINE configs[4]: long-form Q8_0 serving, 32 utterances per GPU (256 on 8), "
                            "ICL prefill 512, up to 4096 greedy frames each, paged F16 KV; Q8_0 projections as "
                            "kind::i8 tcgen05 GEMMs, F16 heads as kind::f16 tcgen05 GEMMs"),
}


def _pkg():
    spec = importlib.util.spec_from_file_location("qtts_b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["qtts_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def _inputs(seed: int, n_ref: int):
    rng = np.random.default_rng(seed)
    tgt = rng.integers(0, 151643, 24).astype(np.int32)
    ref = rng.integers(0, 151643, 30).astype(np.int32)
    codes = rng.integers(0, 2048, (n_ref, 16)).astype(np.int32)
    spk = rng.standard_normal(1024).astype(np.float32)
    spk /= np.linalg.norm(spk)
    return tgt, ref, codes, spk


def _model(cfg, rank: int, local_rank: int, barrier):
    pkg = _pkg()
    d = os.environ.get("QTTS_MODEL_DIR", os.path.join(ROOT, ".models"))
    path = os.path.join(d, f"synth-full-{cfg['wtype']}-s0.gguf")
    if local_rank == 0 and not os.path.exists(path):
        pkg.synth_gguf.ensure_gguf(d, pkg.synth_gguf.FULL, cfg["wtype"], seed=0)
    barrier()
    return pkg, path


class ClockSampler:
    """Polls SM clock and throttle reasons through NVML from a background thread.

    Started before the warm-up (NVML's first calls are slow); mark() brackets the
    timed region and summary() keeps the samples taken inside it."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, index: int):
        self.samples, self.ok = [], False   # (t, mhz, reasons bitmask)
        self.t0 = self.t1 = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), mhz, r))
            except Exception:
                pass
            time.sleep(0.001)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join()

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def summary(self):
        inside = [(m, r) for t, m, r in self.samples
                  if self.t0 is not None and self.t1 is not None and self.t0 <= t <= self.t1]
        reasons = sorted({name for _, r in inside for bit, name in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median([m for m, _ in inside]) if inside else None,
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(inside)}


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _profile_figure(fname: str, key: str):
    """A figure from a committed ncu summary under profiles/ (`key: value` line)."""
    p = os.path.join(ROOT, "profiles", fname)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def cpu_model() -> str:
    """The host CPU's model name (for the CPU baseline's record)."""
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_frames_per_s(path: str, n_ref_prefill: int, budget_s: float, max_frames: int, warmup: int = 0,
                     windows: int = 1):
    """The CPU oracle port on all host cores: frames after a prefill of the same
    length; `warmup` untimed frames first.  With windows > 1 the timed frames
    are split into that many consecutive windows of equal budget and frame
    count, and the rate is their median."""
    from oracle import Oracle, available_cpus
    cores = available_cpus()
    o = Oracle(path, threads=cores, engine_order=False)
    H = o.cfg["hidden"]
    rng = np.random.default_rng(7)
    rows = (rng.standard_normal((n_ref_prefill, H)) * 0.1).astype(np.float32)
    o.init_kv(n_ref_prefill + warmup + max_frames + 16)
    hid, lg = o.forward_prefill(rows)
    hidden = hid[-1]
    pos, frames, t_used = n_ref_prefill, 0, 0.0
    cb0 = int(np.argmax(lg[:2048]))
    done_warm = 0
    rates, w_frames, w_time = [], 0, 0.0
    w_budget, w_max = budget_s / max(windows, 1), max(1, max_frames // max(windows, 1))
    while frames < max_frames and t_used < budget_s:
        warm = done_warm < warmup
        t0 = time.perf_counter()
        codes, _ = o.predict_codes(hidden, cb0)
        step = o.lookup(0, [cb0])[0]
        for g in range(15):
            step = step + o.lookup(g + 1, [int(codes[g])])[0]
        lg, hidden = o.forward_step(step, pos)
        cb0 = int(np.argmax(lg[:2048]))
        pos += 1
        if warm:
            done_warm += 1
            continue
        dt = time.perf_counter() - t0
        t_used += dt
        frames += 1
        w_frames += 1
        w_time += dt
        if windows > 1 and (w_time >= w_budget or w_frames >= w_max) and len(rates) < windows:
            rates.append(w_frames / w_time)
            w_frames, w_time = 0, 0.0
            if len(rates) == windows:
                break
    if windows > 1 and rates:
        return float(np.median(rates)), cores, frames, t_used
    return frames / t_used, cores, frames, t_used


def frames_config(cfg, args, world, plen, K, F):
    """The `config` of a batch-1 line; the reference arm reports the same dict."""
    return {"workload": cfg["workload"], "batch_per_gpu": 1, "prefill": plen, "frames_per_utterance": F,
            "utterance_replays": (K + F - 1) // F, "frames_timed": K,
            "parallelism": f"independent utterance per GPU x{world}",
            "l2": "inputs larger than L2 (3.3 GB of weights streamed per frame), no flush"}


def run_reference(args, cfg):
    """Reference arm: the CPU port of the path (the reference's ggml build is not
    buildable: its ggml submodule is empty), rank 0 only, all host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    pkg, path = _model(cfg, 0, 0, lambda: None)
    fps, cores, frames, secs = cpu_frames_per_s(path, cfg.get("prefill", 64), budget_s=1e9, max_frames=args.steps,
                                                warmup=max(0, args.warmup))
    line = {"impl": "reference", "metric": METRIC, "value": fps, "unit": UNIT, "n_gpus": args.gpus,
            "steps": frames, "warmup": args.warmup, "ms_per_step": 1000.0 * secs / max(frames, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16" if cfg["wtype"] == "f16" else "q8_0", "data": "synthetic (seeded random-init GGUF, 0.6B layout)",
            "config": frames_config(cfg, args, args.gpus, cfg.get("prefill", 64), frames, cfg.get("frames", 32)),
            "cpu_baseline": {"value": fps, "unit": UNIT, "cores": cores, "kind": "port", "cpu_model": cpu_model(),
                             "sample": f"{frames} frames (talker step + 15 code-predictor passes) after a {cfg.get('prefill', 64)}-row prefill; "
                                       "CPU oracle port (reference ggml build not buildable: ggml submodule absent)"},
            "e2e": {"value": fps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)
    return 0


def run_batch(args, cfg):
    """the 64 utterances are LPT-sharded over the ranks; each rank
    runs its share as one batch (one CUDA-graph frame for all its sequences).
    32 utterances per rank (weak scaling), timed over the first
    frames of their 4096-frame budget."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    pkg, path = _model(cfg, rank, local, barrier)
    from qtts_b200.scheduler import Utterance, lpt_partition
    F = cfg["frames"]
    rng = np.random.default_rng(4242)
    if args.utts_per_gpu > 0:   # weak scaling: a fixed batch per GPU
        cfg = dict(cfg, utts_per_gpu=args.utts_per_gpu)
        cfg.pop("n_utts", None)
    n_utts = cfg["n_utts"] if "n_utts" in cfg else cfg["utts_per_gpu"] * world
    P = rng.integers(cfg["p_lo"], cfg["p_hi"] + 1, n_utts)
    utts = [Utterance(uid=i, prefill=int(P[i]), frames=F) for i in range(n_utts)]
    mine = lpt_partition(utts, world)[rank]
    eng = pkg.Engine(path, local)
    H = eng.cfg["hidden_size"]

    def params(u):
        r = np.random.default_rng(10_000 + u.uid)
        n_ref = u.prefill - 9
        spk = r.standard_normal(H).astype(np.float32)
        spk /= np.linalg.norm(spk)
        return dict(text=r.integers(0, 151643, 24).astype(np.int32), max_len=F, speaker=spk,
                    ref_text=r.integers(0, 151643, 30).astype(np.int32),
                    ref_codes=r.integers(0, 2048, (n_ref, 16)).astype(np.int32),
                    rep_penalty=1.05, temperature=0.0, top_k=0, eos_bias=-1e9)

    plist = [params(u) for u in mine]
    B = len(plist)
    max_pos = max(u.prefill for u in mine) + F + 1
    W = max(args.warmup, 3)
    PF = 2                                   # eagerly profiled frames after the timed region
    SK = max(0, min(args.skip_frames, F - W - PF - 1))   # untimed frames before the timed window
    K = max(1, min(args.steps, F - W - PF - SK))
    bt = pkg.engine.Batch(eng, max_batch=B, max_positions=max_pos, max_frames=F)
    bt.begin(plist)
    bt.run(W + SK)
    t0 = bt.timing()["frames_ms"]
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize()
        clk.mark_start()
        got = bt.run(K)
        barrier()
        torch.cuda.synchronize()
        clk.mark_end()
    tm = bt.timing()
    ms = tm["frames_ms"] - t0
    prof = bt.profile(PF)
    t = torch.tensor([ms, float(got)], dtype=torch.float64, device="cuda")
    if world > 1:
        mx = t[:1].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t[1:].clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        ms_max, frames_all = float(mx.item()), float(sm.item())
    else:
        ms_max, frames_all = ms, float(got)

    # e2e through the public API: prompts from host memory, per-sequence prefill,
    # the frames (all F, or the config's bounded e2e run), codes back to the host
    FE = min(F, cfg.get("e2e_frames", F))
    barrier()
    torch.cuda.synchronize()
    te0 = time.perf_counter()
    bt.begin(plist)
    bt.run(FE)
    codes = bt.codes()
    te = time.perf_counter() - te0
    assert all(c.shape[0] == FE for c in codes)
    et = torch.tensor([te, float(B * FE)], dtype=torch.float64, device="cuda")
    if world > 1:
        e1 = et[:1].clone()
        dist.all_reduce(e1, op=dist.ReduceOp.MAX)
        e2 = et[1:].clone()
        dist.all_reduce(e2, op=dist.ReduceOp.SUM)
        te_max, e2e_frames = float(e1.item()), float(e2.item())
    else:
        te_max, e2e_frames = te, float(B * FE)
    h2d = sum(4 * (p["text"].size + p["ref_text"].size + p["ref_codes"].size + H) for p in plist)
    d2h = 4 * B * F * 16   # the codes buffer read back holds max_frames rows per sequence
    bt.close()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    peak, peak_kind = _peaks()
    frame_ms = ms_max / K
    kv_mean = float(np.mean([u.prefill for u in mine])) + W + SK + K / 2.0
    wkey = "f16" if cfg["wtype"] == "f16" else "q8"
    frame_bytes = WEIGHT_BYTES[wkey] + B * (KV_TALKER_PER_POS * kv_mean + KV_CP_PER_POS * 135)
    achieved = frame_bytes / (frame_ms / 1e3) / 1e9
    # ncu DRAM / algorithmic bytes of the batched projections (kind::f16 / kind::i8 tcgen05 GEMMs)
    ratio = _profile_figure("k_gemm_tc_batch16.md" if wkey == "f16" else "k_gemm_q8_batch32.md",
                            "dram_bytes_per_algorithmic_byte")
    traffic = ratio * frame_bytes if ratio else None
    flops = 2.0 * (WEIGHT_BYTES["f16"] / 2.0) * B
    weak = "utts_per_gpu" in cfg
    line = {
        "metric": METRIC, "value": frames_all / (ms_max / 1e3), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": frame_ms, "higher_is_better": True, "scaling": "weak" if weak else "strong",
        "vs_baseline": None, "dtype": "f16" if wkey == "f16" else "q8_0",
        "data": f"synthetic (seeded random-init GGUF with the 0.6B layout; random prompts, "
                f"P ~ U[{cfg['p_lo']},{cfg['p_hi']}])",
        "config": {"workload": cfg["workload"], "utterances": n_utts, "batch_per_gpu": B,
                   "frames_per_utterance": F, "frames_timed_per_sequence": K,
                   "frames_before_timing": W + SK,
                   "parallelism": f"LPT utterance sharding over {world} GPU(s), one batch per GPU",
                   "l2": "inputs larger than L2 (3.3 GB of weights + KV streamed per frame), no flush"},
        "roofline": {"bound": "hbm", "kernel": "batched frame (CUDA graph: tcgen05 GEMMs + paged attention)" if wkey == "f16"
                     else "batched frame (CUDA graph: kind::i8 tcgen05 GEMMs, kind::f16 heads, paged attention)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "frame_algorithmic_bytes": frame_bytes, "launches_per_frame": tm["launches_per_frame"],
                     "tensor_tflops": flops / (frame_ms / 1e3) / 1e12},
        "e2e": {"value": e2e_frames / te_max, "unit": UNIT, "h2d_bytes_per_step": h2d / (B * F),
                "d2h_bytes_per_step": d2h / (B * F),
                "includes": f"qtts_batch_begin (prompt upload + per-sequence prefill) + {FE} frames + codes download"},
        "kernel_classes": prof,
        "gpu_launches": tm["launches_per_frame"] * K,
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        fps, cores, frames, secs = cpu_frames_per_s(path, 64, args.cpu_budget_s, 1024, warmup=2, windows=3)
        line["cpu_baseline"] = {"value": fps, "unit": UNIT, "cores": cores, "kind": "port", "cpu_model": cpu_model(),
                                "sample": f"{frames} frames of one sequence after a 64-row prefill in {secs:.1f} s, "
                                          "median rate of 3 consecutive windows (CPU restatement, not reference "
                                          "build: the in-repo oracle port, OpenMP over all host threads; the CPU "
                                          "path serves one sequence at a time)"}
    emit(line)
    return 0


def run_ncu_workload(args):
    """A small fixed workload for ncu captures (no timing, no JSON line):
    `frames`: the config's ICL prefill and --frames frames through the frame
    loop (QTTS_FRAME_MODE=fused selects the clustered frame path); `batch`: --batch
    utterances with --prompt-position ICL prompts (Q8_0 model for --config q8 / q8long),
    --frames batched frames, then two eagerly profiled frames.  A few GB on the device at most."""
    pkg = _pkg()
    d = os.environ.get("QTTS_MODEL_DIR", os.path.join(ROOT, ".models"))
    cfg_m = pkg.synth_gguf.TINY if args.tiny else pkg.synth_gguf.FULL
    if args.ncu_workload == "frames":
        wtype = "f16" if args.config == "f16" else "q8_0"
        path = pkg.synth_gguf.ensure_gguf(d, cfg_m, wtype, seed=0)
        eng = pkg.Engine(path, 0)
        rng = np.random.default_rng(1000)
        n_ref = CONFIGS[args.config].get("n_ref", 55)
        tgt = rng.integers(0, 151643, 24).astype(np.int32)
        ref = rng.integers(0, 151643, 30).astype(np.int32)
        codes = rng.integers(0, 2048, (n_ref, 16)).astype(np.int32)
        spk = rng.standard_normal(cfg_m.hidden).astype(np.float32)
        eng.generate_begin(tgt, args.frames, speaker=spk, ref_text=ref, ref_codes=codes, rep_penalty=1.05,
                           temperature=0.0, top_k=0, eos_bias=-1e9)
        got = eng.run_frames(args.frames)
        print(f"frames={got} {eng.timing()}", file=sys.stderr)
        eng.close()
        return 0
    path = pkg.synth_gguf.ensure_gguf(d, cfg_m, "q8_0" if CONFIGS[args.config]["wtype"] == "q8_0" else "f16", seed=0)
    eng = pkg.Engine(path, 0)
    H = eng.cfg["hidden_size"]
    frames = args.frames + 2
    utts = []
    P = max(16, args.prompt)   # talker prefill positions per utterance (ICL: 9 + reference frames)
    for i in range(args.batch):
        r = np.random.default_rng(2000 + i)
        utts.append(dict(text=r.integers(0, 151643, 24).astype(np.int32), max_len=frames,
                         speaker=r.standard_normal(H).astype(np.float32),
                         ref_text=r.integers(0, 151643, 30).astype(np.int32),
                         ref_codes=r.integers(0, 2048, (P - 9, 16)).astype(np.int32),
                         rep_penalty=1.05, eos_bias=-1e9))
    bt = pkg.engine.Batch(eng, max_batch=args.batch, max_positions=P + frames + 1, max_frames=frames)
    bt.begin(utts)
    got = bt.run(args.frames)
    prof = bt.profile(2)
    print(f"batch={args.batch} sequence-frames={got} {bt.timing()}", file=sys.stderr)
    for k, v in prof.items():
        print(f"{k:12s} {v['launches_per_frame']:5d} launches/frame  {v['ms_per_frame']:8.3f} ms/frame (eager)",
              file=sys.stderr)
    bt.close()
    eng.close()
    return 0


_RESULT_OUT = None


def emit(line: dict):
    """The one JSON result line, on the process's original standard output."""
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    # Everything else a run prints (NCCL banners, library warnings) goes to
    # stderr, so standard output carries exactly the result line.
    global _RESULT_OUT
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="f16")
    ap.add_argument("--profile-frames", type=int, default=4)
    ap.add_argument("--cpu-budget-s", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu-workload", choices=["frames", "batch"], default=None,
                    help="run a small fixed workload for ncu captures instead of the benchmark")
    ap.add_argument("--frames", type=int, default=2, help="--ncu-workload: frames to run")
    ap.add_argument("--batch", type=int, default=16, help="--ncu-workload batch: utterances")
    ap.add_argument("--tiny", action="store_true", help="--ncu-workload: the 2-layer test model")
    ap.add_argument("--prompt", type=int, default=64, help="--ncu-workload batch: prefill positions per utterance")
    ap.add_argument("--utts-per-gpu", type=int, default=0,
                    help="batch configs: utterances per GPU (weak scaling) instead of the config's total")
    ap.add_argument("--skip-frames", type=int, default=0,
                    help="batch configs: untimed frames after the warm-up, so the timed window sits deeper in "
                         "the utterance (longer KV contexts)")
    args = ap.parse_args()
    if args.ncu_workload:
        return run_ncu_workload(args)
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        return run_reference(args, cfg)
    if args.config in ("batch", "q8long"):
        return run_batch(args, cfg)
    args.warmup = max(args.warmup, 3)

    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    pkg, path = _model(cfg, rank, local, barrier)
    eng = pkg.Engine(path, local)
    tgt, ref, codes, spk = _inputs(1000 + rank, cfg["n_ref"])
    gen = dict(speaker=spk, ref_text=ref, ref_codes=codes, rep_penalty=1.05, temperature=0.0, top_k=0, eos_bias=-1e9)
    K, W = args.steps, args.warmup

    # ---- device-resident timing: inputs in HBM.  The utterance of the config
    # (F frames after the prefill) is replayed K / F times: each replay rewinds
    # the device frame state to frame 0 (no new prefill) and runs F frames as F
    # launches of the frame CUDA graph.
    F = cfg["frames"]
    reps = max(1, (K + F - 1) // F)
    runs = [min(F, K - i * F) for i in range(reps)]   # whole replays, then the remainder of a partial one
    with ClockSampler(local) as clk:
        plen = eng.generate_begin(tgt, F, **gen)
        assert plen == cfg["prefill"], plen
        eng.run_frames(W)
        eng.generate_rewind()
        eng.run_frames(F)
        t0 = eng.timing()["frames_ms"]
        barrier()
        torch.cuda.synchronize()
        clk.mark_start()
        got = 0
        for n in runs:
            eng.generate_rewind()
            got += eng.run_frames(n)
        barrier()
        torch.cuda.synchronize()
        clk.mark_end()
    ms = eng.timing()["frames_ms"] - t0
    assert got == K, got
    ms_t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    launches_per_frame = eng.timing()["kernel_launches"]

    # ---- per-kernel roofline: eager replay with events around each launch
    eng.generate_begin(tgt, W + args.profile_frames, **gen)
    eng.run_frames(W)
    prof = eng.profile_frames(args.profile_frames)

    # ---- end to end through the C ABI with host buffers: each step of an
    # utterance includes its share of the prompt upload, the prefill, the frames
    # and the codes download (qtts_generate with host arrays), reps utterances.
    eng.generate(tgt, 2, **gen)            # untimed warm call
    barrier()
    torch.cuda.synchronize()
    t_e0 = time.perf_counter()
    for n in runs:
        out = eng.generate(tgt, n, **gen)
        assert out["n_frames"] == n
    t_e = time.perf_counter() - t_e0
    et = torch.tensor([t_e], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    t_e = float(et.item())
    H = eng.cfg["hidden_size"]
    n_text_rows = 3 + 3 + (len(ref) - 8) + (len(tgt) - 8) + 1
    # embedding rows read back for the host assembly: 6 special rows + one summed
    # codec row per reference frame (the reference codes go up once, counted above)
    n_lookup_rows = 3 + 2 + 1 + cfg["n_ref"]
    h2d_utt = (4 * (len(tgt) + len(ref) + codes.size) + 4 * H * (plen + 1) + 4 * n_text_rows + 4 * 6)
    d2h_all = sum(4 * H * (n_text_rows + n_lookup_rows) + 4 * 16 * n + 4 * H + 1024 * ((n + 15) // 16) for n in runs)

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0

    peak, peak_kind = _peaks()
    g = prof["gemv"]
    gemv_gbs = (g["bytes"] / g["launches"]) / (g["ms"] / g["launches"] / 1e3) / 1e9 if g["launches"] else None
    frame_ms = ms_max / K
    kv_pos_mean = plen + F / 2.0
    frame_bytes = WEIGHT_BYTES[args.config] + KV_TALKER_PER_POS * kv_pos_mean + KV_CP_PER_POS * 135
    prof_total = sum(prof[c]["ms"] for c in ("gemv", "attention", "sample", "other"))
    # the timed path: the frame CUDA graph; its launches overlap under programmatic dependent
    # launch, so the unit is the frame (algorithmic bytes of a frame / device time per frame)
    mode = eng.frame_mode()
    if mode == "fused":
        kernel = (f"frame CUDA graph, fused path ({launches_per_frame} launches per frame: k_ff_attn, k_ff_ffn, "
                  "k_ff_head; programmatic dependent launch)")
        ratio = _profile_figure(f"k_ff_{args.config}.md", "dram_bytes_per_algorithmic_byte")
    else:
        kernel = f"frame CUDA graph ({launches_per_frame} launches per frame, programmatic dependent launch)"
        # ncu: DRAM bytes per algorithmic byte over captured frame GEMVs (the graph's bytes are GEMV weights)
        ratio = _profile_figure(f"k_gemv_{args.config}.md", "dram_bytes_per_algorithmic_byte")
    bytes_per_launch = frame_bytes
    achieved = frame_bytes / (frame_ms / 1e3) / 1e9
    traffic = ratio * frame_bytes if ratio else None
    launches_per_frame_k = float(launches_per_frame)
    line = {
        "metric": METRIC, "value": world * K / (ms_max / 1e3), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": frame_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16" if args.config == "f16" else "q8_0",
        "data": "synthetic (seeded random-init GGUF with the 0.6B layout; random prompt ids and reference codes)",
        "config": frames_config(cfg, args, world, plen, K, F),
        "roofline": {"bound": "hbm", "kernel": kernel,
                     "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": (achieved / peak) if achieved else None, "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else peak_kind,
                     "bytes_per_launch": bytes_per_launch,
                     "launches_per_frame": launches_per_frame_k,
                     "frame_algorithmic_bytes": frame_bytes,
                     "frame_algorithmic_gbs": frame_bytes / (frame_ms / 1e3) / 1e9,
                     "frame_path": mode,
                     "eager_gemv_gbs_serialised": gemv_gbs,
                     "eager_gemv_share_serialised": g["ms"] / prof_total if prof_total else None},
        "kernel_classes": {c: {"launches_per_frame": prof[c]["launches"] / max(prof["frames"], 1),
                               "ms_per_frame": prof[c]["ms"] / max(prof["frames"], 1)}
                           for c in ("gemv", "attention", "sample", "other")},
        "e2e": {"value": world * K / t_e, "unit": UNIT, "h2d_bytes_per_step": h2d_utt * reps / K,
                "d2h_bytes_per_step": d2h_all / K,
                "includes": f"{reps} x qtts_generate ({'+'.join(str(n) for n in runs)} frames): prompt upload, "
                            "prefill, frames, codes download"},
        "gpu_launches": launches_per_frame * K,
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        fps, cores, frames, secs = cpu_frames_per_s(path, plen, args.cpu_budget_s, 1024, warmup=2, windows=3)
        line["cpu_baseline"] = {"value": fps, "unit": UNIT, "cores": cores, "kind": "port", "cpu_model": cpu_model(),
                                "sample": f"{frames} frames after a {plen}-row prefill in {secs:.1f} s, median "
                                          "rate of 3 consecutive windows (CPU restatement, not reference build: the "
                                          "in-repo oracle port, OpenMP over all host threads)"}
    emit(line)
    return 0


if __name__ == "__main__":
    sys.exit(main())
