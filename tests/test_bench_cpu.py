"""bench.py's host-side contract, on CPU: the committed ncu figures it reads
exist, standard output carries exactly one JSON result line, every config
names what its runner needs, and the CPU baseline honours its warm-up and
budget."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


@pytest.mark.parametrize("fname,key", [
    ("k_gemv_f16.md", "dram_bytes_per_algorithmic_byte"),
    ("k_gemv_q8.md", "dram_bytes_per_algorithmic_byte"),
    ("k_gemm_tc_batch16.md", "dram_bytes_per_algorithmic_byte"),
])
def test_profile_figures_read_by_bench_exist(fname, key):
    v = bench._profile_figure(fname, key)
    assert v is not None and v > 0, (fname, key)


def test_stdout_carries_only_the_result_line():
    code = ("import sys; sys.path.insert(0, %r); import bench, os\n"
            "sys.stdout.flush(); bench._RESULT_OUT = os.fdopen(os.dup(1), 'w'); os.dup2(2, 1)\n"
            "print('incidental output'); os.write(1, b'NCCL banner\\n')\n"
            "bench.emit({'metric': 'codec frames/s', 'value': 1.0})\n") % ROOT
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    assert len(lines) == 1 and json.loads(lines[0])["value"] == 1.0
    assert "incidental output" in r.stderr and "NCCL banner" in r.stderr


@pytest.mark.parametrize("name", sorted(bench.CONFIGS))
def test_configs_name_what_their_runner_needs(name):
    cfg = bench.CONFIGS[name]
    assert cfg["wtype"] in ("f16", "q8_0") and cfg["workload"].startswith("BASELINE configs[")
    if "p_lo" in cfg:   # batched runner
        assert ("n_utts" in cfg) != ("utts_per_gpu" in cfg)
        assert 9 < cfg["p_lo"] <= cfg["p_hi"] and cfg["frames"] > 0
    else:               # batch-1 runner
        assert cfg["prefill"] == 9 + cfg["n_ref"] and cfg["frames"] > 0


def test_cpu_baseline_warmup_and_budget(tiny_f16):
    fps, cores, frames, secs = bench.cpu_frames_per_s(tiny_f16, 13, budget_s=1e9, max_frames=5, warmup=2)
    assert frames == 5 and fps > 0 and cores >= 1 and secs > 0
    fps2, _, frames2, secs2 = bench.cpu_frames_per_s(tiny_f16, 13, budget_s=0.2, max_frames=100000)
    assert 1 <= frames2 < 100000 and secs2 >= 0.2 and fps2 > 0
    assert bench.cpu_model()
    fps3, _, frames3, _ = bench.cpu_frames_per_s(tiny_f16, 13, budget_s=1e9, max_frames=9, warmup=1, windows=3)
    assert frames3 == 9 and fps3 > 0   # three windows of three frames, median rate
