"""CPU tests of the host-side pieces: the seeded GGUF layout, the C ABI surface
(library loads and exports every symbol the headers declare; no compute)."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import numpy as np

import gguf
from conftest import ROOT


def test_synth_gguf_layout_matches_reference_loader(qtts, tiny_q8):
    # tensor set / shapes / types as create_tensors expects
    # (src/tts_transformer.cpp:379-668) and the converter's Q8_0 policy (:249-292)
    r = gguf.GGUFReader(tiny_q8)
    cfg = qtts.synth_gguf.TINY
    specs = dict(qtts.synth_gguf.tensor_specs(cfg))
    seen = {t.name: t for t in r.tensors}
    assert set(seen) == set(specs)
    for name, shape in specs.items():
        t = seen[name]
        assert tuple(int(v) for v in t.shape) == tuple(reversed(shape)), name
        if len(shape) == 1:
            assert t.tensor_type == gguf.GGMLQuantizationType.F32
        elif "_embd" in name or "lm_head" in name or "codec_head" in name:
            assert t.tensor_type == gguf.GGMLQuantizationType.F16, name
        else:
            assert t.tensor_type == gguf.GGMLQuantizationType.Q8_0, name
    # metadata keys the reference loader reads (aliases of parse_config)
    for key in ["qwen3-tts.block_count", "qwen3-tts.embedding_length", "qwen3-tts.attention.head_count",
                "qwen3-tts.attention.head_count_kv", "qwen3-tts.code_predictor.layer_count",
                "qwen3-tts.code_predictor.rope.freq_base", "qwen3-tts.codec.eos_id"]:
        assert key in r.fields, key


def _declared(header):
    txt = open(os.path.join(ROOT, "include", header)).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(qtts_[a-z0-9_]+)\s*\(", txt)) - {"qtts_frame_callback"})


def test_library_exports_every_declared_symbol(qtts):
    path = qtts.build.build()
    lib = ctypes.CDLL(path)       # loads without a GPU
    for sym in _declared("qwen3tts_b200.h"):
        assert hasattr(lib, sym), sym
    nm = subprocess.run(["nm", "-DC", "--defined-only", path], capture_output=True, text=True).stdout
    for member in ["TTSTransformer::load_model", "TTSTransformer::generate(", "TTSTransformer::generate_icl",
                   "TTSTransformer::forward_prefill", "TTSTransformer::forward_step",
                   "TTSTransformer::predict_codes_autoregressive", "TTSTransformer::predict_codes(",
                   "TTSTransformer::init_kv_cache", "TTSTransformer::get_hidden_states",
                   "qwen3_tts::free_transformer_model", "qwen3_tts::free_tts_kv_cache"]:
        assert member in nm, member


def test_create_reports_errors_without_gpu_or_file(qtts):
    lib = qtts.lib()
    assert not lib.qtts_create(b"/nonexistent/model.gguf", 0)
    assert lib.qtts_create_error()


def test_drop_in_header_compiles():
    # the reference's own call pattern (tests/test_transformer.cpp) against our header
    src = r'''
#include "tts_transformer.h"
#include <vector>
int use(qwen3_tts::TTSTransformer & t) {
    std::vector<float> out, logits; std::vector<int32_t> codes;
    int32_t toks[10] = {0};
    t.init_kv_cache(4096); t.clear_kv_cache();
    t.forward_prefill(nullptr, 10, 0, out, &logits);
    t.generate(toks, 10, nullptr, 64, codes, 2050, 1.05f, 0.0f, 0);
    t.generate_icl(toks, 10, toks, 10, toks, 1, nullptr, 8, codes);
    return t.get_config().n_codebooks + (int) t.get_error().size();
}
'''
    p = os.path.join(ROOT, ".pytest_cache", "dropin_check.cpp")
    os.makedirs(os.path.dirname(p), exist_ok=True)
    open(p, "w").write(src)
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", os.path.join(ROOT, "include"), p],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
