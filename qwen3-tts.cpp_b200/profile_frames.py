"""Small fixed workload for ncu captures: load a seeded GGUF, run the ICL
prefill of BASELINE config 1 (64 positions) and N frames through the frame
loop, and exit.  Frame mode comes from QTTS_FRAME_MODE (graph | persistent).

    python qwen3-tts.cpp_b200/profile_frames.py [--frames N] [--config f16|q8] [--tiny]
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--frames", type=int, default=2)
    ap.add_argument("--config", choices=["f16", "q8"], default="f16")
    ap.add_argument("--tiny", action="store_true")
    a = ap.parse_args()
    spec = importlib.util.spec_from_file_location("qtts_b200", os.path.join(HERE, "__init__.py"),
                                                  submodule_search_locations=[HERE])
    pkg = importlib.util.module_from_spec(spec)
    sys.modules["qtts_b200"] = pkg
    spec.loader.exec_module(pkg)
    cfg = pkg.synth_gguf.TINY if a.tiny else pkg.synth_gguf.FULL
    wtype = "f16" if a.config == "f16" else "q8_0"
    path = pkg.synth_gguf.ensure_gguf(os.environ.get("QTTS_MODEL_DIR", os.path.join(ROOT, ".models")), cfg, wtype,
                                      seed=0)
    eng = pkg.Engine(path, 0)
    rng = np.random.default_rng(1000)
    n_ref = 55 if a.config == "f16" else 119
    tgt = rng.integers(0, 151643, 24).astype(np.int32)
    ref = rng.integers(0, 151643, 30).astype(np.int32)
    codes = rng.integers(0, 2048, (n_ref, 16)).astype(np.int32)
    spk = rng.standard_normal(cfg.hidden).astype(np.float32)
    eng.generate_begin(tgt, a.frames, speaker=spk, ref_text=ref, ref_codes=codes, rep_penalty=1.05,
                       temperature=0.0, top_k=0, eos_bias=-1e9)
    got = eng.run_frames(a.frames)
    print(f"frames={got} {eng.timing()}")
    if os.environ.get("QTTS_PK_TRACE"):
        types, tr = eng.op_trace()
        names = {1: "gemv", 2: "attn", 3: "sample", 4: "input", 5: "frame_end"}
        n = len(types)
        t = tr[: n * got].astype(np.int64)
        nxt = np.append(t[1:, 0], t[-1, 4])
        issue = t[:, 1] - t[:, 0]
        ready = np.where(t[:, 2] > 0, t[:, 2] - t[:, 0], 0)
        work0 = t[:, 3] - t[:, 0]
        straggle = t[:, 4] - t[:, 3]
        barrier = nxt - t[:, 4]
        for ty in sorted(set(types.tolist())):
            idx = np.nonzero(np.tile(types, got) == ty)[0]
            print(f"op {names.get(ty, ty):9s} n={len(idx)//max(got,1):4d}/frame  issue {issue[idx].mean()/1e3:5.2f}"
                  f"  last-weights {ready[idx].mean()/1e3:5.2f}  cta0-done {work0[idx].mean()/1e3:5.2f}"
                  f"  last-done +{straggle[idx].mean()/1e3:5.2f}  barrier+next {barrier[idx].mean()/1e3:5.2f} us")
        print(f"frame span {(t[-1, 4] - t[0, 0]) / 1e3 / max(got, 1):.1f} us")
    eng.close()


if __name__ == "__main__":
    main()
