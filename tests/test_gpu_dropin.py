"""The C++ drop-in boundary on the GPU: a C++ program compiled against
include/tts_transformer.h and linked to libqwen3tts_b200.so drives
qwen3_tts::TTSTransformer the way the reference's transformer test does
(tests/test_transformer.cpp:169-355 of the reference) and through the rest of
its public members; every result is checked against the CPU oracle.

The reference's goldens (reference/det_*.bin) are absent, so the checks are
against the oracle: codes token-for-token (near-ties excepted), logits and
hidden rows within the F16 tolerance, and the 'ATTD' attention dump
(src/tts_transformer.cpp:2978-3005) parsed and compared row for row with the
oracle's post-softmax rows of the same layer.
"""
from __future__ import annotations

import os
import struct
import subprocess
import sys

import numpy as np
import pytest

from conftest import PKG_DIR, ROOT, text_ids
from oracle import Oracle

pytestmark = pytest.mark.gpu
TIE_TOL = 1e-3


def _build_driver(tmp):
    exe = os.path.join(tmp, "dropin_driver")
    cmd = ["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "dropin_driver.cpp"), "-L", PKG_DIR, "-lqwen3tts_b200",
           f"-Wl,-rpath,{PKG_DIR}", "-o", exe]
    subprocess.run(cmd, check=True)
    return exe


def _parse_attd(path):
    """'ATTD' file: u32 magic 0x41545444, i32 version, layer, n_head, n_rows, then
    per row i32 n_kv and n_head * n_kv F32 ([head][key])."""
    b = open(path, "rb").read()
    magic, version, layer, n_head, n_rows = struct.unpack_from("<Iiiii", b, 0)
    assert magic == 0x41545444 and version == 1
    off, rows = 20, []
    for _ in range(n_rows):
        (n_kv,) = struct.unpack_from("<i", b, off)
        off += 4
        rows.append(np.frombuffer(b, np.float32, n_head * n_kv, off).reshape(n_head, n_kv))
        off += 4 * n_head * n_kv
    assert off == len(b)
    return layer, n_head, rows


def test_dropin_class_against_oracle(qtts, tiny_f16, tmp_path):
    qtts.build.build()
    exe = _build_driver(str(tmp_path))
    rng = np.random.default_rng(301)
    H = 256
    text = text_ids(rng, 20)
    ref_text = text_ids(rng, 14)
    ref_codes = rng.integers(0, 2048, (6, 16)).astype(np.int32)
    spk = rng.standard_normal(H).astype(np.float32)
    prefill = (rng.standard_normal((10, H)) * 0.1).astype(np.float32)
    d = str(tmp_path)
    text.tofile(os.path.join(d, "text.i32"))
    ref_text.tofile(os.path.join(d, "ref_text.i32"))
    ref_codes.tofile(os.path.join(d, "ref_codes.i32"))
    spk.tofile(os.path.join(d, "speaker.f32"))
    prefill.tofile(os.path.join(d, "prefill.f32"))
    env = dict(os.environ, QWEN3_TTS_DEVICE="0", QWEN3_TTS_TIMING="1")
    out = subprocess.run([exe, tiny_f16, d], capture_output=True, text=True, env=env, timeout=600)
    print(out.stdout, out.stderr[-2000:], file=sys.stderr)
    assert out.returncode == 0 and "DONE" in out.stdout, out.stdout
    lines = dict(ln.split(" ", 1) for ln in out.stdout.splitlines() if " " in ln)
    rd = lambda n, dt: np.fromfile(os.path.join(d, n), dt)

    o = Oracle(tiny_f16)
    # forward_prefill: hidden rows and logits
    o.init_kv(4096)
    hid_o, lg_o = o.forward_prefill(prefill)
    hid = rd("prefill_hidden.f32", np.float32).reshape(10, H)
    assert np.abs(hid - hid_o).max() < 2e-2 * max(1.0, np.abs(hid_o).max())
    assert np.abs(rd("prefill_logits.f32", np.float32) - lg_o).max() < 2e-2
    assert np.array_equal(rd("prefill_last_hidden.f32", np.float32), hid[-1])

    # generate (language 2050, penalty 1.05, greedy) and the attention dump of layer 1
    codes = rd("gen_codes.i32", np.int32).reshape(-1, 16)
    assert codes.shape == (8, 16)
    kw = dict(speaker=spk, language_id=2050, rep_penalty=1.05, temperature=0.0, top_k=0, eos_bias=-1e9)
    r, rows_o = o.generate_with_attn_dump(1, 256, 16, text=text, max_len=8, follow=codes, tie_tol=TIE_TOL, **kw)
    assert r["n_mismatch"] == 0 and r["n_frames"] == 8
    layer, n_head, rows = _parse_attd(os.path.join(d, "attn.bin"))
    assert layer == 1 and n_head == 4
    assert int(lines["attn_rows"]) == len(rows) == 7 == len(rows_o)
    for f, row in enumerate(rows):
        assert row.shape == (4, r["prefill_len"] + f + 1)
        assert np.allclose(row.sum(axis=1), 1.0, atol=1e-5)
        assert np.abs(row - rows_o[f, :, : row.shape[1]]).max() < 1e-3, f

    # generate_icl aborted by the callback after frame 3: four frames kept
    icl = rd("icl_codes.i32", np.int32).reshape(-1, 16)
    assert icl.shape == (4, 16) and int(lines["icl_callback_frames"]) == 4
    ki = dict(speaker=spk, ref_text=ref_text, ref_codes=ref_codes, language_id=2050, rep_penalty=1.05,
              temperature=0.0, top_k=0, eos_bias=-1e9)
    ri = o.generate(text, 4, follow=icl, tie_tol=TIE_TOL, **ki)
    assert ri["n_mismatch"] == 0 and ri["n_frames"] == 4

    # forward_text: projected text rows + speaker embedding through the talker prefill
    o.init_kv(4096)
    rows_t = o.project_text(text[:6]) + spk
    th_o, _ = o.forward_prefill(rows_t.astype(np.float32))
    th = rd("text_hidden.f32", np.float32).reshape(6, H)
    assert np.abs(th - th_o).max() < 2e-2 * max(1.0, np.abs(th_o).max())
    # forward_codec: codec_bos embedding as one talker step at position 6
    cl_o, ch_o = o.forward_step(o.lookup(0, [2149])[0], 6)
    assert np.abs(rd("codec_logits.f32", np.float32) - cl_o).max() < 2e-2
    ch = rd("codec_hidden.f32", np.float32)
    assert np.abs(ch - ch_o).max() < 2e-2 * max(1.0, np.abs(ch_o).max())
    # predict_codes_autoregressive from that hidden state with codebook-0 token 7
    ar = rd("cp_ar_codes.i32", np.int32)
    ar_o, _ = o.predict_codes(ch, 7, temperature=0.0, top_k=0)
    assert ar.shape == (15,)
    assert np.array_equal(ar, ar_o)

    # legacy predict_codes: float64 restatement of build_code_pred_graph
    from ref_numpy import legacy_predict_codes
    prev = np.array([(17 * g + 3) % 2048 for g in range(15)], np.int32)
    ref = legacy_predict_codes(tiny_f16, ch, prev)
    got = rd("cp_legacy_logits.f32", np.float32).reshape(15, 2048)
    assert np.abs(got - ref).max() < 2e-2 * max(1.0, np.abs(ref).max())

    # the QWEN3_TTS_TIMING report after each generate (src/tts_transformer.cpp:3311-3353 layout)
    assert out.stderr.count("=== Detailed Generation Timing (") == 2     # generate and generate_icl
    assert "=== Detailed Generation Timing (8 frames) ===" in out.stderr
    assert "Code predictor (total / per-frame):" in out.stderr and "Total generate:" in out.stderr

    # error convention: bool + get_error()
    assert lines["short_text_rejected"].startswith("1") and "at least 4" in lines["short_text_rejected"]
    assert lines["unloaded_forward_rejected"] == "1"
