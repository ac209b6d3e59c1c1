"""CPU tests: pin the oracle (the engine's checker) against independent sources.

* Q8_0 quantiser: bit-exact vs gguf-py 0.19.0 (the package the reference's
  converter imports, scripts/convert_tts_to_gguf.py:35), which states it is
  bit-exact with ggml-quants.c's reference quantiser.
* GGUF reader: the oracle's embedding rows vs gguf-py's GGUFReader.
* Graph maths: oracle logits vs an independent NumPy statement (ref_numpy.py).
* Prefill layout: the 10 plain-mode positions documented by the reference's
  reference/det_prefill_token_types.json, restated in PREFILL_LAYOUT below.
* Sampling rules of src/tts_transformer.cpp:2583-2593, 2750-2788, 3108-3184.
"""
from __future__ import annotations

import numpy as np
import pytest

import gguf
from conftest import icl_inputs, text_ids
from oracle import Oracle, philox, quantize_q8_0, rope_cache, uniform01
from ref_numpy import NpModel


def test_q8_0_quantiser_matches_gguf_py():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(32 * 257) * rng.uniform(0.001, 3.0, 32 * 257)).astype(np.float32)
    x[:32] = 0.0                      # all-zero block: d = 0, q = 0
    x[32:64] = 0.5                    # equal values (x * id exactly 127)
    x[64:96] = np.linspace(-1, 1, 32)  # halves to round away from zero
    q, d = quantize_q8_0(x)
    ref = gguf.quants.quantize(x.reshape(1, -1), gguf.GGMLQuantizationType.Q8_0).reshape(-1, 34)
    assert np.array_equal(d, ref[:, :2].copy().view(np.uint16)[:, 0])
    assert np.array_equal(q.reshape(-1, 32), ref[:, 2:].copy().view(np.int8))


def test_gguf_reader_rows_match_gguf_py(tiny_f16):
    o = Oracle(tiny_f16, threads=4)
    r = gguf.GGUFReader(tiny_f16)
    byname = {t.name: t for t in r.tensors}
    ids = np.array([0, 5, 2148, 2149, 3071], np.int32)
    ref = np.array(byname["talker.codec_embd.weight"].data).astype(np.float32)[ids]
    assert np.array_equal(o.lookup(0, ids), ref)
    ids2 = np.array([1, 2047], np.int32)
    ref2 = np.array(byname["code_pred.codec_embd.14.weight"].data).astype(np.float32)[ids2]
    assert np.array_equal(o.lookup(15, ids2), ref2)
    assert o.cfg["hidden"] == 256 and o.cfg["n_layers"] == 2 and o.cfg["cp_theta"] == 1e6


@pytest.mark.parametrize("which", ["tiny_f16", "tiny_q8"])
def test_oracle_matches_numpy_statement(which, request):
    path = request.getfixturevalue(which)
    o, npm = Oracle(path, threads=4), NpModel(path)
    rng = np.random.default_rng(3)
    rows = (rng.standard_normal((6, 256)) * 0.1).astype(np.float32)
    hid_o, lg_o = o.forward_prefill(rows)
    hid_n, lg_n = npm.talker(rows, 0)
    tol = 2e-3 if which == "tiny_q8" else 1e-3
    assert np.abs(lg_o - lg_n).max() < tol * max(1.0, np.abs(lg_n).max())
    assert np.abs(hid_o - hid_n).max() < tol * 10
    step = (rng.standard_normal(256) * 0.1).astype(np.float32)
    lg2_o, hid2_o = o.forward_step(step, 6)
    hid2_n, lg2_n = npm.talker(step[None], 6)
    assert np.abs(lg2_o - lg2_n).max() < tol * max(1.0, np.abs(lg2_n).max())
    codes_o, cpl_o = o.predict_codes(hid2_o, 17)
    codes_n, cpl_n = npm.code_predictor(hid2_o, 17)
    assert np.abs(cpl_o[0] - cpl_n[0]).max() < tol * max(1.0, np.abs(cpl_n[0]).max())
    # token agreement except at near-ties
    for g in range(15):
        if codes_o[g] != codes_n[g]:
            gap = cpl_o[g][codes_o[g]] - cpl_o[g][codes_n[g]]
            assert gap < 1e-3
            break


def test_rope_cache_is_ggml_recurrence():
    cs = rope_cache(37, 128, 1e6)
    s = np.float32(1e6) ** np.float32(-2.0 / 128)
    th = np.float32(37.0)
    for i in range(64):
        assert cs[2 * i] == pytest.approx(np.cos(np.float64(th)), abs=2e-6)
        assert cs[2 * i + 1] == pytest.approx(np.sin(np.float64(th)), abs=2e-6)
        th = np.float32(th * s)


def _philox_py(c, k):
    c = list(c); k0, k1 = k
    M = 0xFFFFFFFF
    for _ in range(10):
        p0 = 0xD2511F53 * c[0]
        p1 = 0xCD9E8D57 * c[2]
        c = [(p1 >> 32) ^ c[1] ^ k0, p1 & M, (p0 >> 32) ^ c[3] ^ k1, p0 & M]
        k0 = (k0 + 0x9E3779B9) & M
        k1 = (k1 + 0xBB67AE85) & M
    return c


def test_philox_matches_python_statement():
    for ctr, key in [([0, 0, 0, 0], [0, 0]), ([1, 2, 3, 4], [5, 6]), ([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2)]:
        assert philox(ctr, key) == _philox_py(ctr, key)
    u = [uniform01(7, f, cb) for f in range(200) for cb in range(16)]
    assert 0.0 <= min(u) and max(u) < 1.0 and abs(np.mean(u) - 0.5) < 0.02


# reference/det_prefill_token_types.json (plain mode, language 2050, speaker):
# position -> (text-projection part, codec-embedding part)
PREFILL_LAYOUT = [
    ("text0", None), ("text1", None), ("text2", None),
    ("pad", 2154), ("pad", 2156), ("pad", 2050), ("pad", 2157),
    ("pad", "speaker"), ("bos", 2148), ("text3", 2149),
]


def test_prefill_layout_matches_reference_token_types(tiny_f16):
    o = Oracle(tiny_f16, threads=4)
    rng = np.random.default_rng(4)
    text = text_ids(rng, 14)
    spk = rng.standard_normal(256).astype(np.float32)
    r = o.generate(text, 1, speaker=spk, want_prefill=True, eos_bias=-1e9)
    pf = r["prefill"]
    assert r["prefill_len"] == 10
    sp = o.project_text([151672, 151673, 151671])
    parts = {"bos": sp[0], "pad": sp[2]}
    tp = o.project_text(text[:4])
    for i in range(3):
        parts[f"text{i}"] = tp[i]
    parts["text3"] = tp[3]
    for pos, (tpart, cpart) in enumerate(PREFILL_LAYOUT):
        want = parts[tpart].copy()
        if cpart == "speaker":
            want = want + spk
        elif cpart is not None:
            want = want + o.lookup(0, [cpart])[0]
        np.testing.assert_allclose(pf[pos], want, rtol=0, atol=1e-6)


def test_icl_prefill_length(tiny_f16):
    o = Oracle(tiny_f16, threads=4)
    rng = np.random.default_rng(5)
    tgt, ref, codes, _ = icl_inputs(rng, 55)
    spk = rng.standard_normal(256).astype(np.float32)
    r = o.generate(tgt, 2, speaker=spk, ref_text=ref, ref_codes=codes, eos_bias=-1e9)
    assert r["prefill_len"] == 9 + 55        # src/tts_transformer.cpp:1290, 1396


def test_sampling_rules():
    from oracle import Oracle as _O
    L = _O.lib()
    import ctypes as C
    # argmax: first index wins on ties
    lg = np.array([0.5, 2.0, 2.0, 1.0], np.float32)
    assert L.orc_sample(lg.ctypes.data_as(C.POINTER(C.c_float)), 4, 0.0, 0, 0.0) == 1
    # top-k keeps ties at the threshold: k=2 over [3, 1, 3, 3] keeps all the 3s
    for u, want in [(0.0, 0), (0.34, 2), (0.99, 3)]:
        lg = np.array([3.0, 1.0, 3.0, 3.0], np.float32)
        assert L.orc_sample(lg.ctypes.data_as(C.POINTER(C.c_float)), 4, 1.0, 2, u) == want


def test_oracle_follow_self_and_eos(tiny_f16):
    o = Oracle(tiny_f16, threads=4)
    rng = np.random.default_rng(6)
    text = text_ids(rng, 20)
    a = o.generate(text, 6, eos_bias=-1e9)
    b = o.generate(text, 6, eos_bias=-1e9, follow=a["codes"])
    assert b["n_mismatch"] == 0 and np.array_equal(a["codes"], b["codes"])
    e = o.generate(text, 6, eos_bias=1e9)          # EOS forced at the first frame
    assert e["n_frames"] == 0
    t = o.generate(text, 40, eos_bias=0.0, target_frames=2)
    assert t["n_frames"] <= 40


def test_oracle_expf_within_2_ulp():
    """The exp shared by engine and oracle (Cody-Waite + degree-7 Taylor) is
    within 2 ulp of e^x over the range the softmax and SiLU use, and saturates
    to 0 / inf outside the float range."""
    from oracle import expf
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.uniform(-87.0, 88.0, 20000), rng.uniform(-1.0, 1.0, 20000),
                        np.array([0.0, -0.0, 1.0, -1.0, 88.5, -87.3, -100.0])]).astype(np.float32)
    y = expf(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    ulp = np.spacing(ref.astype(np.float32)).astype(np.float64)
    assert np.all(np.abs(y - ref) <= 2 * ulp), float(np.max(np.abs(y - ref) / ulp))
    assert expf(np.array([200.0]))[0] == np.inf and expf(np.array([-200.0]))[0] == 0.0


def test_engine_order_matches_plain_order(tiny_f16):
    """The oracle's engine-order reductions and its plain orders are the same
    arithmetic up to summation order: step logits agree to float rounding."""
    from oracle import Oracle
    rng = np.random.default_rng(8)
    outs = []
    for eng in (True, False):
        o = Oracle(tiny_f16, threads=4, engine_order=eng)
        H = o.cfg["hidden"]
        rows = (rng.standard_normal((12, H)) * 0.1).astype(np.float32) if not outs else rows
        o.init_kv(64)
        _, lg = o.forward_prefill(rows)
        outs.append(lg)
        o.close()
    Oracle(tiny_f16, threads=4, engine_order=True).close()
    assert np.abs(outs[0] - outs[1]).max() < 1e-3
