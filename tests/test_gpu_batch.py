"""Batched frame loop (tcgen05 GEMMs, paged KV, per-sequence state) against the
CPU oracle: every sequence of the batch, with its own prompt and prompt length,
follows the oracle's greedy decisions (divergence allowed only at recorded
near-ties, as for the single-sequence engine)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import text_ids
from oracle import Oracle

pytestmark = pytest.mark.gpu
TIE_TOL = 1e-3


def _utterances(rng, n, frames, hidden):
    out = []
    for i in range(n):
        u = dict(text=text_ids(rng, 14 + 5 * i), max_len=frames, eos_bias=-1e9, rep_penalty=1.05)
        if i % 2:
            u["speaker"] = rng.standard_normal(hidden).astype(np.float32)
        out.append(u)
    return out


@pytest.mark.parametrize("which,n", [("f16", 1), ("f16", 5), ("q8", 1), ("q8", 5)])
def test_batch_matches_oracle(qtts, request, which, n):
    """F16: kind::f16 tcgen05 GEMMs.  Q8_0: the projections as kind::i8 tcgen05
    GEMMs (exact int32 block dots), the F16 heads as kind::f16 GEMMs."""
    path = request.getfixturevalue("tiny_f16" if which == "f16" else "tiny_q8")
    rng = np.random.default_rng(40 + n)
    eng = qtts.Engine(path, 0)
    H = eng.cfg["hidden_size"]
    frames = 10
    utts = _utterances(rng, n, frames, H)
    b = qtts.engine.Batch(eng, max_batch=8, max_positions=256, max_frames=frames)
    b.begin(utts)
    assert b.run(frames) == n * frames
    codes = b.codes()
    o = Oracle(path)
    for i, u in enumerate(utts):
        assert codes[i].shape == (frames, 16)
        kw = {k: v for k, v in u.items() if k not in ("text", "max_len")}
        if which == "f16":
            r = o.generate(u["text"], frames, follow=codes[i], tie_tol=TIE_TOL, **kw)
            assert r["n_mismatch"] == 0, (i, r["n_mismatch"], r["max_mismatch_gap"], r["first_mismatch"])
        else:
            # Q8_0: the activation quantiser turns last-bit differences of the sums
            # (tensor-core order vs the oracle's) into whole int8 levels, so the bar
            # is the full-size tests' near-tie rule: every divergent decision within
            # the Q8_0 margin, and rare
            r = o.generate(u["text"], frames, follow=codes[i], tie_tol=1e9, **kw)
            assert r["max_tie_gap"] <= BATCH_MARGIN["q8"], (i, r["max_tie_gap"], r["n_ties"])
            assert r["n_ties"] <= BATCH_FRAC["q8"] * 16 * frames, (i, r["n_ties"])
        assert r["n_frames"] == frames
    b.close()
    eng.close()


def test_batch_sequence_independence(qtts, tiny_f16):
    """A sequence's codes do not depend on the other sequences of the batch."""
    rng = np.random.default_rng(77)
    eng = qtts.Engine(tiny_f16, 0)
    utts = _utterances(rng, 4, 8, eng.cfg["hidden_size"])
    b = qtts.engine.Batch(eng, max_batch=4, max_positions=256, max_frames=8)
    b.begin(utts)
    b.run(8)
    together = b.codes()
    b.begin(utts[2:3])
    b.run(8)
    alone = b.codes()
    assert np.array_equal(together[2], alone[0])
    b.close()
    eng.close()


def test_codes_device_handoff(qtts, tiny_f16):
    """The device code buffers (single sequence and batch) hold the codes the
    host copies return: a GPU consumer can read them without a host round trip."""
    import torch

    class _Dev:   # a raw device int32 buffer seen through __cuda_array_interface__
        def __init__(self, ptr, shape):
            self.__cuda_array_interface__ = {"shape": shape, "typestr": "<i4", "data": (ptr, False), "version": 2}

    rng = np.random.default_rng(90)
    eng = qtts.Engine(tiny_f16, 0)
    text = text_ids(rng, 20)
    out = eng.generate(text, 7, eos_bias=-1e9)
    ptr, n = eng.codes_device()
    assert n == 7 and ptr != 0
    dev = torch.as_tensor(_Dev(ptr, (n, 16)), device="cuda").cpu().numpy()
    assert np.array_equal(dev, out["codes"])
    utts = _utterances(rng, 3, 5, eng.cfg["hidden_size"])
    b = qtts.engine.Batch(eng, max_batch=4, max_positions=256, max_frames=5)
    b.begin(utts)
    b.run(5)
    host = b.codes()
    bptr, nf = b.codes_device()
    allc = torch.as_tensor(_Dev(bptr, (3, 5, 16)), device="cuda").cpu().numpy()
    for i in range(3):
        assert nf[i] == 5 and np.array_equal(allc[i, :nf[i]], host[i])
    b.close()
    eng.close()


def test_batch_stops_each_sequence_at_its_max_len(qtts, tiny_f16):
    """EOS suppressed, per-sequence max_len 3 / 7 / 5, run() asked for more
    frames than any budget: each sequence stops at its own max_len on the device
    (its position never passes prompt + max_len) and its codes follow the oracle."""
    rng = np.random.default_rng(91)
    eng = qtts.Engine(tiny_f16, 0)
    H = eng.cfg["hidden_size"]
    utts = _utterances(rng, 3, 8, H)
    for u, m in zip(utts, (3, 7, 5)):
        u["max_len"] = m
    b = qtts.engine.Batch(eng, max_batch=4, max_positions=128, max_frames=8)
    b.begin(utts)
    assert b.run(50) == 3 + 7 + 5
    assert b.run(10) == 0
    codes = b.codes()
    o = Oracle(tiny_f16)
    for i, u in enumerate(utts):
        assert codes[i].shape == (u["max_len"], 16)
        kw = {k: v for k, v in u.items() if k not in ("text", "max_len")}
        r = o.generate(u["text"], u["max_len"], follow=codes[i], tie_tol=TIE_TOL, **kw)
        assert r["n_mismatch"] == 0 and r["n_frames"] == u["max_len"]
    b.close()
    eng.close()


def _icl_utterance(seed, prefill, frames, hidden):
    """An ICL utterance whose talker prefill is `prefill` positions (9 + reference frames)."""
    r = np.random.default_rng(seed)
    spk = r.standard_normal(hidden).astype(np.float32)
    spk /= np.linalg.norm(spk)
    return dict(text=text_ids(r, 24), max_len=frames, speaker=spk, ref_text=text_ids(r, 30),
                ref_codes=r.integers(0, 2048, (prefill - 9, 16)).astype(np.int32),
                rep_penalty=1.05, temperature=0.0, top_k=0, eos_bias=-1e9)


# The batched path accumulates its projections in the tcgen05 MMA order and its
# attention in page order, so against either oracle order it diverges only at
# decisions a logit difference within the north_star tolerance (2e-2 F16, 5e-2
# Q8_0) can flip: oracle margin <= 2 x tolerance, and rarely (Q8_0: the
# activation quantiser turns order differences into whole int8 levels).
BATCH_MARGIN = {"f16": 4e-2, "q8": 1e-1}
BATCH_FRAC = {"f16": 0.01, "q8": 0.10}


def _follow(path, utts, codes, frames, idx, engine_order, which):
    """Oracle replay of sequences `idx` of a batch, every divergence recorded."""
    o = Oracle(path, engine_order=engine_order)
    for i in idx:
        u = utts[i]
        assert codes[i].shape == (frames, 16), (i, codes[i].shape)
        kw = {k: v for k, v in u.items() if k not in ("text", "max_len")}
        r = o.generate(u["text"], frames, follow=codes[i], tie_tol=1e9, **kw)
        diag = dict(divergent=r["n_ties"], decisions=16 * frames, max_margin=r["max_tie_gap"], first=r["first_mismatch"])
        print("batch parity:", which, i, diag)
        assert r["n_frames"] == frames
        assert r["max_tie_gap"] <= BATCH_MARGIN[which], (i, diag)
        assert r["n_ties"] <= BATCH_FRAC[which] * 16 * frames, (i, diag)


def test_full_batch64_config4_shape(qtts, full_f16):
    """configs[3] shape on the 0.6B F16 model: 64 utterances, ICL prompts of
    U[32, 512] positions, 64 greedy frames each through the tcgen05 batch path
    (MMA N = 64, the split-K cluster sizes the projections use, up to 9 KV pages
    per sequence).  Eight sequences, the shortest and longest prompts among
    them, are replayed by the CPU oracle (ggml order: its prefill is the fast
    one); every sequence must produce all 64 frames."""
    eng = qtts.Engine(full_f16, 0)
    H = eng.cfg["hidden_size"]
    rng = np.random.default_rng(4242)
    P = rng.integers(32, 513, 64)
    frames = 64
    utts = [_icl_utterance(5000 + i, int(P[i]), frames, H) for i in range(64)]
    b = qtts.engine.Batch(eng, max_batch=64, max_positions=int(P.max()) + frames + 1, max_frames=frames)
    b.begin(utts)
    assert b.run(frames) == 64 * frames
    codes = b.codes()
    b.close()
    eng.close()
    order = np.argsort(P)
    idx = sorted({int(order[0]), int(order[-1])} | {int(order[k]) for k in (9, 18, 27, 36, 45, 54)})
    _follow(full_f16, utts, codes, frames, idx, engine_order=False, which="f16")


def test_full_q8_batch32_config5_shape(qtts, full_q8):
    """configs[4] shape on the 0.6B Q8_0 model: 32 utterances with 512-position
    prompts (8 KV pages each), 24 greedy frames (into the ninth page), four
    sequences replayed by the CPU oracle; then one sequence run to 1,032
    positions (17 pages) and replayed in full."""
    eng = qtts.Engine(full_q8, 0)
    H = eng.cfg["hidden_size"]
    frames = 24
    utts = [_icl_utterance(7000 + i, 512, frames, H) for i in range(32)]
    b = qtts.engine.Batch(eng, max_batch=32, max_positions=512 + frames + 1, max_frames=frames)
    b.begin(utts)
    assert b.run(frames) == 32 * frames
    codes = b.codes()
    b.close()
    _follow(full_q8, utts, codes, frames, [0, 10, 21, 31], engine_order=True, which="q8")
    long_frames = 520
    lu = [_icl_utterance(7999, 512, long_frames, H)]
    b = qtts.engine.Batch(eng, max_batch=1, max_positions=512 + long_frames + 1, max_frames=long_frames)
    b.begin(lu)
    assert b.run(long_frames) == long_frames
    lc = b.codes()
    b.close()
    eng.close()
    _follow(full_q8, lu, lc, long_frames, [0], engine_order=True, which="q8")


@pytest.mark.parametrize("split", [3, 16])
def test_split_kv_attention_matches_oracle(qtts, tiny_f16, monkeypatch, split):
    """Talker attention split over KV page ranges (QTTS_ATTN_SPLIT; flash-decoding
    partials merged in range order): prompts of 40-170 positions give 1-3 pages
    per sequence, so ranges are full, partial and empty; every sequence follows
    the oracle under the batched path's near-tie rule."""
    monkeypatch.setenv("QTTS_ATTN_SPLIT", str(split))
    eng = qtts.Engine(tiny_f16, 0)
    H = eng.cfg["hidden_size"]
    frames = 20
    utts = [_icl_utterance(9100 + i, p, frames, H) for i, p in enumerate((150, 40, 100))]
    b = qtts.engine.Batch(eng, max_batch=4, max_positions=256, max_frames=frames)
    b.begin(utts)
    assert b.run(frames) == 3 * frames
    codes = b.codes()
    b.close()
    eng.close()
    _follow(tiny_f16, utts, codes, frames, [0, 1, 2], engine_order=True, which="f16")
