"""Tensor-core prefill (tcgen05 GEMMs over up to 128 prompt rows per chunk, the
default for prompts of more than 8 rows: kind::f16 for F16 weights, kind::i8
for Q8_0) against the CPU oracle.

The GEMMs accumulate in the MMA's order, not the oracle's, so this path is held
to the north-star contract rather than to bit equality: prefill hidden rows and
logits within max-abs 2e-2 (F16), then greedy codes identical to the oracle's
except at recorded near-ties (top-2 gap < 1e-3), frame logits within 2e-2.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import icl_inputs, text_ids
from oracle import Oracle

pytestmark = pytest.mark.gpu

TIE_TOL = 1e-3
LOGIT_TOL = 2e-2


def _follow(o, e, **kw):
    r = o.generate(follow=e["codes"], want_logits=True, tie_tol=TIE_TOL, **kw)
    n = e["n_frames"]
    assert r["n_mismatch"] == 0, (r["n_mismatch"], r["max_mismatch_gap"], r["first_mismatch"])
    assert r["n_frames"] == n
    assert np.abs(e["talker_logits"][:n] - r["talker_logits"][:n]).max() < LOGIT_TOL
    assert np.abs(e["cp_logits"][:n] - r["cp_logits"][:n]).max() < LOGIT_TOL
    return r


@pytest.mark.parametrize("n_rows,n_past", [(13, 0), (150, 0), (40, 17)])
def test_prefill_rows_match_oracle(qtts, tiny_f16, monkeypatch, n_rows, n_past):
    """forward_prefill hidden rows and logits; 150 rows span two chunks; n_past > 0
    attends over rows already in the cache."""
    rng = np.random.default_rng(300 + n_rows)
    first = (rng.standard_normal((n_past, 256)) * 0.1).astype(np.float32) if n_past else None
    rows = (rng.standard_normal((n_rows, 256)) * 0.1).astype(np.float32)
    outs = {}
    for mode in ("tc", "gemv"):
        monkeypatch.setenv("QTTS_PREFILL", mode)
        eng = qtts.Engine(tiny_f16, 0)
        eng.init_kv_cache(256)
        if first is not None:
            eng.forward_prefill(first, 0)
        outs[mode] = eng.forward_prefill(rows, n_past)
        eng.close()
    o = Oracle(tiny_f16, threads=4)
    o.init_kv(256)
    if first is not None:
        o.forward_prefill(first, 0)
    ho, lo = o.forward_prefill(rows, n_past)
    he, le = outs["tc"]
    assert np.abs(he - ho).max() < LOGIT_TOL and np.abs(le - lo).max() < LOGIT_TOL
    # the two engine paths differ only in summation order
    hg, lg = outs["gemv"]
    assert np.abs(he - hg).max() < LOGIT_TOL and np.abs(le - lg).max() < LOGIT_TOL


def test_generate_icl_tc_prefill(qtts, tiny_f16, monkeypatch):
    monkeypatch.delenv("QTTS_PREFILL", raising=False)   # default: tensor cores for > 8 rows
    eng = qtts.Engine(tiny_f16, 0)
    o = Oracle(tiny_f16, threads=4)
    rng = np.random.default_rng(310)
    tgt, ref, codes, spk = icl_inputs(rng, 40, n_target_text=40)
    kw = dict(speaker=spk, ref_text=ref, ref_codes=codes, rep_penalty=1.05, eos_bias=-1e9)
    e = eng.generate(tgt, 12, want_logits=True, **kw)
    r = _follow(o, e, text=tgt, max_len=12, **kw)
    assert r["prefill_len"] == 49
    eng.close()


def test_generate_plain_tc_prefill(qtts, tiny_f16, monkeypatch):
    monkeypatch.setenv("QTTS_PREFILL", "tc")   # forced even for a 10-row prompt
    eng = qtts.Engine(tiny_f16, 0)
    o = Oracle(tiny_f16, threads=4)
    rng = np.random.default_rng(311)
    text = text_ids(rng, 30)
    kw = dict(speaker=np.zeros(256, np.float32), rep_penalty=1.05, eos_bias=-1e9)
    e = eng.generate(text, 10, want_logits=True, **kw)
    _follow(o, e, text=text, max_len=10, **kw)
    eng.close()


@pytest.mark.parametrize("n_rows", [20, 150])
def test_q8_tc_prefill_rows_match_oracle(qtts, tiny_q8, monkeypatch, n_rows):
    """Q8_0 prompts through the kind::i8 tensor-core GEMMs (quantised
    activations, exact int32 block dots, block sums in order): hidden rows and
    logits within the Q8_0 bound 5e-2 of the oracle and of the GEMV prefill."""
    rng = np.random.default_rng(312 + n_rows)
    rows = (rng.standard_normal((n_rows, 256)) * 0.1).astype(np.float32)
    outs = {}
    for mode in ("tc", "gemv"):
        monkeypatch.setenv("QTTS_PREFILL", mode)
        eng = qtts.Engine(tiny_q8, 0)
        eng.init_kv_cache(256)
        outs[mode] = eng.forward_prefill(rows, 0)
        eng.close()
    o = Oracle(tiny_q8, threads=4)
    o.init_kv(256)
    ho, lo = o.forward_prefill(rows, 0)
    he, le = outs["tc"]
    hg, lg = outs["gemv"]
    assert np.abs(he - ho).max() < 5e-2 and np.abs(le - lo).max() < 5e-2
    assert np.abs(he - hg).max() < 5e-2 and np.abs(le - lg).max() < 5e-2
    assert not np.array_equal(le, lg)   # the tensor-core path ran (its sums differ in the last bits)


def test_full_f16_config1_tc_prefill(qtts, full_f16, monkeypatch):
    """BASELINE config 1 shape through the default (tensor-core) prefill."""
    monkeypatch.delenv("QTTS_PREFILL", raising=False)
    eng = qtts.Engine(full_f16, 0)
    o = Oracle(full_f16)
    rng = np.random.default_rng(101)
    tgt, ref, codes, spk = icl_inputs(rng, 55)
    kw = dict(speaker=spk, ref_text=ref, ref_codes=codes, rep_penalty=1.05, temperature=0.0, top_k=0, eos_bias=-1e9)
    e = eng.generate(tgt, 12, want_logits=True, **kw)
    r = _follow(o, e, text=tgt, max_len=12, **kw)
    assert r["prefill_len"] == 64
    eng.close()
