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
    """F16: tcgen05 GEMMs.  Q8_0: the projections run as 8-row GEMV chunks (the
    batch-1 kernel's int8 block dots), the F16 heads as tcgen05 GEMMs."""
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
        r = o.generate(u["text"], frames, follow=codes[i], tie_tol=TIE_TOL, **kw)
        assert r["n_mismatch"] == 0, (i, r["n_mismatch"], r["max_mismatch_gap"], r["first_mismatch"])
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
