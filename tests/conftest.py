"""Shared fixtures: the engine package (loaded by path; its directory name is not
a Python identifier), the CPU oracle, and seeded synthetic GGUF models."""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "qwen3-tts.cpp_b200")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_pkg():
    if "qtts_b200" in sys.modules:
        return sys.modules["qtts_b200"]
    spec = importlib.util.spec_from_file_location("qtts_b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["qtts_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (run with -m gpu)")


@pytest.fixture(scope="session")
def qtts():
    return load_pkg()


@pytest.fixture(scope="session")
def model_dir():
    """Seeded GGUFs are cached here (kept out of the repository and of the GPU snapshot); bench.py uses the same files."""
    d = os.environ.get("QTTS_MODEL_DIR", os.path.join(ROOT, ".models"))
    os.makedirs(d, exist_ok=True)
    return d


@pytest.fixture(scope="session")
def tiny_f16(qtts, model_dir):
    return qtts.synth_gguf.ensure_gguf(model_dir, qtts.synth_gguf.TINY, "f16", seed=1)


@pytest.fixture(scope="session")
def tiny_q8(qtts, model_dir):
    return qtts.synth_gguf.ensure_gguf(model_dir, qtts.synth_gguf.TINY, "q8_0", seed=2)


@pytest.fixture(scope="session")
def full_f16(qtts, model_dir):
    return qtts.synth_gguf.ensure_gguf(model_dir, qtts.synth_gguf.FULL, "f16", seed=0)


@pytest.fixture(scope="session")
def full_q8(qtts, model_dir):
    return qtts.synth_gguf.ensure_gguf(model_dir, qtts.synth_gguf.FULL, "q8_0", seed=0)


def text_ids(rng, n):
    """Synthetic text-token ids (ordinary vocabulary, below the special ids)."""
    return rng.integers(0, 151643, n).astype(np.int32)


def icl_inputs(rng, n_ref_frames, n_target_text=24, n_ref_text=30):
    """ICL prompt: role prefix (3) + text + 5-token tail, reference codes."""
    tgt = text_ids(rng, n_target_text)
    ref = text_ids(rng, n_ref_text)
    codes = rng.integers(0, 2048, (n_ref_frames, 16)).astype(np.int32)
    spk = rng.standard_normal(1024).astype(np.float32)
    return tgt, ref, codes, spk
