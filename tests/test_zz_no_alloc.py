"""The allocation-free sampler entry point (qtts_op_sample_noalloc) against the
regular one (qtts_op_sample), through the C ABI.

Some callers cannot allocate device memory per call (a real-time streaming
loop, where cudaMalloc/cudaFree synchronise the device and stall audio, or a
host that owns all device memory through its own pool); this entry point keeps
the sampler's state in a fixed device array instead.  The test gives it device
buffers it allocated itself (the test is the caller), runs two calls in a row
on different inputs — the second must not see the first call's state — and
compares each token with the regular entry point's.  It sits in its own file,
collected last, and works alone or after the other tests.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc(lib, torch, logits, cb, presence=None, **kw):
    dev_logits = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).cuda()
    dev_pres = None if presence is None else torch.from_numpy(np.ascontiguousarray(presence, np.int32)).cuda()
    dev_tok = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    rc = lib.qtts_op_sample_noalloc(
        0, dev_logits.data_ptr(), logits.size, cb, kw.get("temperature", 0.0), kw.get("top_k", 0),
        kw.get("rep_penalty", 1.0), None if dev_pres is None else dev_pres.data_ptr(), kw.get("eos_bias", 0.0),
        kw.get("target_frames", 0), kw.get("frame", 0), 2150, kw.get("suppress_start", logits.size),
        kw.get("seed", 0), dev_tok.data_ptr(), None)
    assert rc == 1
    torch.cuda.synchronize()
    return int(dev_tok.item())


def test_noalloc_sampler_matches_regular_entry_point(qtts):
    import torch
    from qtts_b200.engine import lib, op_sample
    L = lib()
    rng = np.random.default_rng(31)
    # call 1: codebook 0 with a presence set and the penalty that demotes its best token
    lg1 = rng.standard_normal(3072).astype(np.float32)
    lg1[40] = 8.0
    lg1[41] = 7.99
    pres = np.zeros(3072, np.int32)
    pres[40] = 1
    kw1 = dict(rep_penalty=1.05, suppress_start=2048)
    want1 = op_sample(lg1, 0, presence=pres, **kw1)
    got1 = _noalloc(L, torch, lg1, 0, presence=pres, **kw1)
    assert got1 == want1 == 41
    # call 2, right after: same logits, no presence set -> token 40 again (state was cleared)
    want2 = op_sample(lg1, 0, **kw1)
    got2 = _noalloc(L, torch, lg1, 0, **kw1)
    assert got2 == want2 == 40
    # sampled code-predictor decisions with top-k, twice in a row
    for trial in range(2):
        lg = (rng.standard_normal(2048) * 2).astype(np.float32)
        kw = dict(temperature=0.9, top_k=50, seed=77, frame=trial)
        assert _noalloc(L, torch, lg, 5, **kw) == op_sample(lg, 5, **kw)


def test_noalloc_sampler_rejects_vocab_beyond_scratch(qtts):
    import torch
    from qtts_b200.engine import lib
    L = lib()
    big = torch.zeros(5000, dtype=torch.float32, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = L.qtts_op_sample_noalloc(0, big.data_ptr(), 5000, 1, 0.0, 0, 1.0, None, 0.0, 0, 0, 2150, 5000, 0,
                                  tok.data_ptr(), None)
    assert rc == -2
