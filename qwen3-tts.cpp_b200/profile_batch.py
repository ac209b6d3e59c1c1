"""Small fixed workload of the batched frame loop for ncu captures: load the
seeded 0.6B F16 GGUF, arm a batch of B utterances with short ICL prompts
(64 prefill positions each), run N batched frames, print the per-class profile
of two more frames, and exit.  A few GB on the device at most (B = 16: a
0.5 GB page pool next to the 1.8 GB of weights and their tiled copies).

    python qwen3-tts.cpp_b200/profile_batch.py [--batch B] [--frames N]
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
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--frames", type=int, default=2)
    a = ap.parse_args()
    spec = importlib.util.spec_from_file_location("qtts_b200", os.path.join(HERE, "__init__.py"),
                                                  submodule_search_locations=[HERE])
    pkg = importlib.util.module_from_spec(spec)
    sys.modules["qtts_b200"] = pkg
    spec.loader.exec_module(pkg)
    path = pkg.synth_gguf.ensure_gguf(os.environ.get("QTTS_MODEL_DIR", os.path.join(ROOT, ".models")),
                                      pkg.synth_gguf.FULL, "f16", seed=0)
    eng = pkg.Engine(path, 0)
    H = eng.cfg["hidden_size"]
    frames = a.frames + 2
    utts = []
    for i in range(a.batch):
        r = np.random.default_rng(2000 + i)
        utts.append(dict(text=r.integers(0, 151643, 24).astype(np.int32), max_len=frames,
                         speaker=r.standard_normal(H).astype(np.float32),
                         ref_text=r.integers(0, 151643, 30).astype(np.int32),
                         ref_codes=r.integers(0, 2048, (55, 16)).astype(np.int32),
                         rep_penalty=1.05, eos_bias=-1e9))
    bt = pkg.engine.Batch(eng, max_batch=a.batch, max_positions=64 + frames + 1, max_frames=frames)
    bt.begin(utts)
    got = bt.run(a.frames)
    prof = bt.profile(2)
    print(f"batch={a.batch} sequence-frames={got} {bt.timing()}")
    for k, v in prof.items():
        print(f"{k:12s} {v['launches_per_frame']:5d} launches/frame  {v['ms_per_frame']:8.3f} ms/frame (eager, events)")
    bt.close()
    eng.close()


if __name__ == "__main__":
    main()
