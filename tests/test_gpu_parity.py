"""GPU parity: the B200 engine (through its C ABI) against the CPU oracle.

Contract: greedy codec tokens identical to the
reference path except at recorded near-ties (top-2 logit gap < 1e-3); logits
within max-abs 2e-2 (F16) / 5e-2 (Q8_0); per-block Q8_0 int8 dots bit-exact.
Tie handling: the oracle replays the engine's codes and counts a divergence as
a mismatch unless the oracle's own top-2 gap there is below TIE_TOL.

The oracle runs its reductions in the engine's order with the same exp, so the
single-sequence engine is held to more than the contract: its frame-loop
logits equal the oracle's bit for bit (_check_follow).  Prompts here go
through the GEMV prefill (QTTS_PREFILL=gemv), whose order the oracle restates;
the tolerances remain the bar for paths with other orders (the tensor-core
prefill, tests/test_gpu_prefill_tc.py; the tensor-core batched path;
forward_prefill's hidden rows).
"""
from __future__ import annotations

import numpy as np
import pytest

import gguf
from conftest import icl_inputs, text_ids
from oracle import Oracle, quantize_q8_0, uniform01

pytestmark = pytest.mark.gpu

TIE_TOL = 1e-3
LOGIT_TOL = {"f16": 2e-2, "q8": 5e-2}


@pytest.fixture(autouse=True)
def _gemv_prefill(monkeypatch):
    monkeypatch.setenv("QTTS_PREFILL", "gemv")


@pytest.fixture(scope="module")
def eng_tiny(qtts, tiny_f16):
    return qtts.Engine(tiny_f16, 0)


@pytest.fixture(scope="module")
def eng_tiny_q8(qtts, tiny_q8):
    return qtts.Engine(tiny_q8, 0)


# ---------------------------------------------------------------- kernels
@pytest.mark.parametrize("rows,cols,nv", [(4096, 1024, 1), (1024, 3072, 1), (3072, 1024, 2), (333, 256, 8), (64, 2048, 3)])
def test_gemv_f16_matches_fp64(qtts, rows, cols, nv):
    from qtts_b200.engine import op_gemv
    rng = np.random.default_rng(rows + cols)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16)
    x = rng.standard_normal((nv, cols)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, cols).astype(np.float32)
    for norm, act32 in [(None, False), (g, False), (None, True)]:
        y = op_gemv(w, 1, rows, cols, x, norm_gain=norm, act_f32=act32)
        xs = x.astype(np.float64)
        if norm is not None:
            ms = (x.astype(np.float64) ** 2).mean(axis=1, keepdims=True).astype(np.float32)
            xs = (x * (np.float32(1) / np.sqrt(ms + np.float32(1e-6))) * norm).astype(np.float64)
        if not act32:
            xs = xs.astype(np.float32).astype(np.float16).astype(np.float64)
        ref = xs @ w.astype(np.float64).T
        assert np.abs(y - ref).max() < 2e-5 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("rows,cols,nv", [(4096, 1024, 1), (1024, 3072, 2), (100, 512, 8)])
def test_gemv_q8_block_dots_bit_exact(qtts, rows, cols, nv):
    from qtts_b200.engine import op_gemv
    rng = np.random.default_rng(rows * 7 + cols)
    wf = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    wq = gguf.quants.quantize(wf, gguf.GGMLQuantizationType.Q8_0)       # reference converter's quantiser
    x = rng.standard_normal((nv, cols)).astype(np.float32) * rng.uniform(0.01, 5.0, (nv, 1)).astype(np.float32)
    y, bd = op_gemv(wq, 8, rows, cols, x, want_block_dots=True)
    nb = cols // 32
    qw = wq.reshape(rows, nb, 34)[:, :, 2:].copy().view(np.int8).astype(np.int64)
    dw = wq.reshape(rows, nb, 34)[:, :, :2].copy().view(np.float16).astype(np.float64)[:, :, 0]
    for v in range(nv):
        qa, da = quantize_q8_0(x[v])          # quantize_row_q8_0_ref semantics
        qa = qa.reshape(nb, 32).astype(np.int64)
        exact = np.einsum("rbj,bj->rb", qw, qa)
        assert np.array_equal(bd[v], exact), "per-block int8 dots must be bit-exact"
        ref = (exact * dw * da.view(np.float16).astype(np.float64)[None, :]).sum(axis=1)
        assert np.abs(y[v] - ref).max() < 1e-5 * max(1.0, np.abs(ref).max())


def test_sampler_rules_match_oracle(qtts):
    from qtts_b200.engine import op_sample
    L = Oracle.lib()
    import ctypes as C
    rng = np.random.default_rng(9)
    # argmax: first index wins; suppression [V-1024, V) except EOS; presence penalty; EOS bias ramp
    lg = rng.standard_normal(3072).astype(np.float32)
    lg[100] = lg[200] = 9.0
    assert op_sample(lg, 0, suppress_start=2048) == 100
    lg2 = lg.copy(); lg2[2500] = 50.0
    assert op_sample(lg2, 0, suppress_start=2048) == 100          # suppressed
    pres = np.zeros(3072, np.int32); pres[100] = 1
    assert op_sample(lg, 0, rep_penalty=1.05, presence=pres, suppress_start=2048) == 200
    assert op_sample(lg, 0, eos_bias=20.0, suppress_start=2048) == 2150
    assert op_sample(lg, 0, eos_bias=0.0, target_frames=1, frame=300, suppress_start=2048) in (100, 2150)
    # sampled: same draw as the oracle's inverse-CDF rule
    for trial in range(40):
        lg = rng.standard_normal(2048).astype(np.float32) * 2
        if trial % 5 == 0:
            lg[::7] = 1.5                                            # many ties at the top-k threshold
        k = [0, 50, 7, 1][trial % 4]
        got = op_sample(lg, 3, temperature=0.9, top_k=k, seed=11, frame=trial)
        u = uniform01(11, trial, 3)
        want = L.orc_sample(lg.copy().ctypes.data_as(C.POINTER(C.c_float)), 2048, 0.9, k, u)
        assert got == want, (trial, got, want)


# ---------------------------------------------------------------- forward passes
@pytest.mark.parametrize("which", ["f16", "q8"])
def test_prefill_and_step_logits(which, request):
    path = request.getfixturevalue("tiny_f16" if which == "f16" else "tiny_q8")
    eng = request.getfixturevalue("eng_tiny" if which == "f16" else "eng_tiny_q8")
    o = Oracle(path, threads=4)
    rng = np.random.default_rng(12)
    rows = (rng.standard_normal((13, 256)) * 0.1).astype(np.float32)
    eng.init_kv_cache(64)
    o.init_kv(64)
    # F16: only reduction order differs (tight bound).  Q8_0: a 1-ulp difference in
    # an activation can move one int8 quant of its block, so the bound is the
    # north-star Q8_0 logit tolerance.
    tol = 1e-3 if which == "f16" else LOGIT_TOL["q8"]
    he, le = eng.forward_prefill(rows, 0)
    ho, lo = o.forward_prefill(rows, 0)
    assert np.abs(le - lo).max() < tol and np.abs(he - ho).max() < tol
    step = (rng.standard_normal(256) * 0.1).astype(np.float32)
    le2, he2 = eng.forward_step(step, 13)
    lo2, ho2 = o.forward_step(step, 13)
    assert np.abs(le2 - lo2).max() < tol and np.abs(he2 - ho2).max() < tol
    ce = eng.predict_codes_autoregressive(he2, 77, 0.0, 0)
    co, cpl = o.predict_codes(ho2, 77)
    first = np.nonzero(ce != co)[0]
    if first.size:
        g = first[0]
        assert cpl[g][co[g]] - cpl[g][ce[g]] < TIE_TOL


def _check_follow(o, eng_out, tag, tie_tol=TIE_TOL, **kw):
    r = o.generate(follow=eng_out["codes"], want_logits=True, tie_tol=tie_tol, **kw)
    n = eng_out["n_frames"]
    diag = dict(tag=tag, n_mismatch=r["n_mismatch"], n_ties=r["n_ties"], max_tie_gap=r["max_tie_gap"],
                max_mismatch_gap=r["max_mismatch_gap"], first_mismatch=r["first_mismatch"],
                min_decision_gap=r["min_decision_gap"])
    if "talker_logits" in eng_out and n:
        diag["talker_logit_maxabs"] = float(np.abs(eng_out["talker_logits"][:n] - r["talker_logits"][:n]).max())
        diag["cp_logit_maxabs"] = float(np.abs(eng_out["cp_logits"][:n] - r["cp_logits"][:n]).max())
    print("parity:", diag)
    assert r["n_mismatch"] == 0, diag
    assert r["n_frames"] == n, (tag, r["n_frames"], n)
    if "talker_logit_maxabs" in diag:
        # the oracle runs every reduction in the engine's order with the same exp:
        # the engine's logits are bit-identical to the oracle's
        assert diag["talker_logit_maxabs"] == 0.0 and diag["cp_logit_maxabs"] == 0.0, diag
    return r


@pytest.mark.parametrize("which", ["f16", "q8"])
def test_generate_greedy_token_parity(which, request):
    path = request.getfixturevalue("tiny_f16" if which == "f16" else "tiny_q8")
    eng = request.getfixturevalue("eng_tiny" if which == "f16" else "eng_tiny_q8")
    o = Oracle(path, threads=4)
    rng = np.random.default_rng(21)
    text = text_ids(rng, 24)
    spk = np.zeros(256, np.float32)
    kw = dict(speaker=spk, rep_penalty=1.05, temperature=0.0, top_k=0, eos_bias=-1e9)
    e = eng.generate(text, 24, want_logits=True, **kw)
    assert e["n_frames"] == 24
    r = _check_follow(o, e, which, text=text, max_len=24, **kw)
    n = e["n_frames"]
    assert np.abs(e["talker_logits"][:n] - r["talker_logits"][:n]).max() < LOGIT_TOL[which]
    assert np.abs(e["cp_logits"][:n] - r["cp_logits"][:n]).max() < LOGIT_TOL[which]


def test_generate_icl_and_instruct(eng_tiny, tiny_f16):
    o = Oracle(tiny_f16, threads=4)
    rng = np.random.default_rng(22)
    tgt, ref, codes, _ = icl_inputs(rng, 20, n_target_text=40)
    spk = rng.standard_normal(256).astype(np.float32)
    kw = dict(speaker=spk, ref_text=ref, ref_codes=codes, eos_bias=-1e9)
    e = eng_tiny.generate(tgt, 12, **kw)
    _check_follow(o, e, "icl", text=tgt, max_len=12, **kw)
    ins = text_ids(rng, 7)
    kw2 = dict(speaker=None, instruct=ins, language_id=-1, eos_bias=-1e9)
    e2 = eng_tiny.generate(tgt, 6, **kw2)
    _check_follow(o, e2, "instruct", text=tgt, max_len=6, **kw2)


def test_generate_sampled_reproducible(eng_tiny, tiny_f16):
    o = Oracle(tiny_f16, threads=4)
    rng = np.random.default_rng(23)
    text = text_ids(rng, 30)
    kw = dict(speaker=np.zeros(256, np.float32), temperature=0.9, top_k=50, rep_penalty=1.05, seed=1234, eos_bias=-1e9)
    a = eng_tiny.generate(text, 16, **kw)
    b = eng_tiny.generate(text, 16, **kw)
    assert np.array_equal(a["codes"], b["codes"])
    _check_follow(o, a, "sampled", text=text, max_len=16, **kw)


def test_stop_conditions(eng_tiny, tiny_f16):
    o = Oracle(tiny_f16, threads=4)
    rng = np.random.default_rng(24)
    text = text_ids(rng, 20)
    # EOS forced on the first frame
    assert eng_tiny.generate(text, 8, eos_bias=1e9)["n_frames"] == 0
    # callback abort keeps the frames up to and including the aborting one
    seen = []
    e = eng_tiny.generate(text, 30, eos_bias=-1e9, on_frame=lambda codes, f: (seen.append(f), f < 4)[1])
    assert e["n_frames"] == 5 and seen == [0, 1, 2, 3, 4]
    # repetition-loop detection on: engine and oracle agree on every code and on
    # where the run stops (the oracle replays the engine's codes; any divergence
    # or a different stopping frame fails)
    e2 = eng_tiny.generate(text, 40, eos_bias=-1e9, rep_penalty=1.0, rep_loop_detect=True)
    r2 = o.generate(text, 40, eos_bias=-1e9, rep_penalty=1.0, rep_loop_detect=True, follow=e2["codes"])
    assert r2["n_mismatch"] == 0
    assert r2["n_frames"] == e2["n_frames"]
    assert np.array_equal(r2["codes"][: e2["n_frames"]], e2["codes"])


# ---------------------------------------------------------------- full-size (0.6B layout)
def test_full_f16_config1_shape(qtts, full_f16):
    """BASELINE config 1 shape: ICL, 55 reference frames -> 64 prefill, greedy."""
    eng = qtts.Engine(full_f16, 0)
    o = Oracle(full_f16)
    rng = np.random.default_rng(101)
    tgt, ref, codes, spk = icl_inputs(rng, 55)
    kw = dict(speaker=spk, ref_text=ref, ref_codes=codes, rep_penalty=1.05, temperature=0.0, top_k=0, eos_bias=-1e9)
    e = eng.generate(tgt, 32, want_logits=True, **kw)
    r = _check_follow(o, e, "full-f16", text=tgt, max_len=32, **kw)
    assert r["prefill_len"] == 64 and e["n_frames"] == 32
    n = e["n_frames"]
    assert np.abs(e["talker_logits"][:n] - r["talker_logits"][:n]).max() < LOGIT_TOL["f16"]
    eng.close()


def test_full_q8_config2_shape(qtts, full_q8):
    """Q8_0, 119 reference frames -> 128 prefill, 256 greedy frames."""
    eng = qtts.Engine(full_q8, 0)
    o = Oracle(full_q8)
    rng = np.random.default_rng(102)
    tgt, ref, codes, spk = icl_inputs(rng, 119)
    kw = dict(speaker=spk, ref_text=ref, ref_codes=codes, rep_penalty=1.05, temperature=0.0, top_k=0, eos_bias=-1e9)
    e = eng.generate(tgt, 256, want_logits=True, **kw)
    r = _check_follow(o, e, "full-q8", text=tgt, max_len=256, **kw)
    assert r["prefill_len"] == 128 and e["n_frames"] == 256
    n = e["n_frames"]
    assert np.abs(e["talker_logits"][:n] - r["talker_logits"][:n]).max() < LOGIT_TOL["q8"]
    eng.close()


def test_full_f16_config3_sampled(qtts, full_f16):
    """plain-mode voice clone with 200 text tokens (prefill 10
    + 192 trailing rows), a unit-norm Gaussian x-vector, temperature 0.9, top-k 50,
    repetition penalty 1.05, fixed Philox seed, 512 frames.  Every sampled code
    (8,192 decisions) is checked against the oracle's draw with the same uniform,
    then a greedy rerun of the same prompt."""
    eng = qtts.Engine(full_f16, 0)
    o = Oracle(full_f16)
    rng = np.random.default_rng(103)
    text = text_ids(rng, 200)
    spk = rng.standard_normal(1024).astype(np.float32)
    spk /= np.linalg.norm(spk)
    kw = dict(speaker=spk, temperature=0.9, top_k=50, rep_penalty=1.05, seed=2024, eos_bias=-1e9)
    e = eng.generate(text, 512, want_logits=True, **kw)
    r = _check_follow(o, e, "full-f16-sampled", text=text, max_len=512, **kw)
    assert r["prefill_len"] == 10 and e["n_frames"] == 512
    kg = dict(kw, temperature=0.0, top_k=0)
    g = eng.generate(text, 32, want_logits=True, **kg)
    _check_follow(o, g, "full-f16-greedy", text=text, max_len=32, **kg)
    eng.close()


def test_both_frame_paths_match_the_oracle(qtts, tiny_f16, tiny_q8, monkeypatch):
    """The fused frame path (two clustered kernels per layer) and the
    kernel-per-op CUDA graph each equal the oracle in their own reduction order:
    greedy codes and every logit, bit for bit (the two paths differ from each
    other only in how the O-projection and ffn_down are summed)."""
    rng = np.random.default_rng(25)
    text = text_ids(rng, 26)
    kw = dict(speaker=np.zeros(256, np.float32), eos_bias=-1e9, rep_penalty=1.05)
    for path in (tiny_f16, tiny_q8):
        for mode in ("graph", "fused"):
            monkeypatch.setenv("QTTS_FRAME_MODE", mode)
            eng = qtts.Engine(path, 0)
            assert eng.frame_mode() == mode
            e = eng.generate(text, 20, want_logits=True, **kw)
            eng.close()
            _check_follow(Oracle(path, threads=4, frame_split=mode == "fused"), e, f"{mode}", text=text, max_len=20,
                          **kw)


@pytest.mark.gpu
def test_rewind_replays_the_utterance(qtts, tiny_f16, monkeypatch):
    """qtts_generate_rewind restores the post-prefill frame state: a replay of the
    same utterance (greedy, repetition penalty on) yields the same codes, in both
    frame modes."""
    rng = np.random.default_rng(31)
    text = text_ids(rng, 20)
    for mode in ("fused", "graph"):
        monkeypatch.setenv("QTTS_FRAME_MODE", mode)
        eng = qtts.Engine(tiny_f16, 0)
        eng.generate_begin(text, 12, speaker=np.zeros(256, np.float32), eos_bias=-1e9, rep_penalty=1.05)
        a = np.zeros((12, 16), np.int32)
        assert eng.run_frames(12, a) == 12
        for _ in range(2):
            eng.generate_rewind()
            b = np.zeros((12, 16), np.int32)
            assert eng.run_frames(12, b) == 12
            assert np.array_equal(a, b)
        eng.close()


def test_stage_timing(qtts, tiny_f16):
    """QWEN3_TTS_TIMING's stages (src/tts_transformer.h:20-54): with stage timing
    on, every stage of a generate call has a positive time, the stages fit in the
    call, and the codes are the frame graph's."""
    rng = np.random.default_rng(32)
    text = text_ids(rng, 20)
    kw = dict(speaker=np.zeros(256, np.float32), eos_bias=-1e9, rep_penalty=1.05)
    eng = qtts.Engine(tiny_f16, 0)
    ref = eng.generate(text, 6, **kw)
    eng.set_stage_timing(True)
    out = eng.generate(text, 6, **kw)
    t = eng.stage_timing()
    eng.set_stage_timing(False)
    eng.close()
    assert np.array_equal(out["codes"], ref["codes"])
    assert t["frames"] == 6
    for k in ("prefill_build_ms", "prefill_forward_ms", "talker_ms", "code_pred_ms", "sample_embed_ms", "total_ms"):
        assert t[k] > 0.0, (k, t)
    assert t["prefill_forward_ms"] + t["talker_ms"] + t["code_pred_ms"] + t["sample_embed_ms"] <= t["total_ms"], t
