"""tcgen05 tensor-core GEMM (batched / prefill path) against a float64 NumPy
statement of the same arithmetic: activations normalised (RMSNorm, F32 as the
kernel) and rounded to F16, or split into F16 hi + lo (the F32-activation
ffn_down), products of F16 operands accumulated in F32.  Tolerance: F32
accumulation over K terms, 1e-5 x sum |w x| + 1e-6 (the F16 roundings are done
identically on both sides)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng(qtts):
    import qtts_b200.engine as E
    return E


def _act(x, gain, eps, split):
    x = x.astype(np.float32)
    if gain is not None:
        ss = np.sum((x * x).astype(np.float64), axis=1)
        mean = (ss / x.shape[1]).astype(np.float32)
        scale = (np.float32(1.0) / np.sqrt(mean + np.float32(eps))).astype(np.float32)
        x = ((x * scale[:, None]).astype(np.float32) * gain.astype(np.float32)).astype(np.float32)
    hi = x.astype(np.float16).astype(np.float64)
    if not split:
        return hi
    lo = (x - hi.astype(np.float32)).astype(np.float16).astype(np.float64)
    return hi + lo


def _check(y, ref, bound):
    err = np.abs(y.astype(np.float64) - ref)
    tol = 1e-5 * bound + 1e-6
    assert np.all(err <= tol), (float(err.max()), float((err / tol).max()))


@pytest.mark.parametrize("rows,cols,m", [(128, 64, 1), (256, 1024, 16), (4096, 1024, 64), (1024, 2048, 100),
                                         (3072, 1024, 256), (2048, 1024, 7)])
def test_gemm_tc_store(eng, rows, cols, m):
    rng = np.random.default_rng(rows + cols + m)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    g = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    y = eng.op_gemm_tc(w, x, norm_gain=g)
    a = _act(x, g, 1e-6, False)
    w64 = w.astype(np.float64)
    _check(y, a @ w64.T, np.abs(a) @ np.abs(w64).T)


def test_gemm_tc_split_resid(eng):
    rng = np.random.default_rng(5)
    rows, cols, m = 1024, 3072, 64
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16)
    x = (rng.standard_normal((m, cols)) * 0.3).astype(np.float32)
    r = rng.standard_normal((m, rows)).astype(np.float32)
    y = eng.op_gemm_tc(w, x, act=eng.TC_ACT_SPLIT, epi=eng.TC_EPI_RESID, resid=r)
    a = _act(x, None, 0, True)
    w64 = w.astype(np.float64)
    _check(y, a @ w64.T + r, np.abs(a) @ np.abs(w64).T + np.abs(r))
    # the split keeps ~22 bits of the F32 activation: close to the exact F32 product
    exact = x.astype(np.float64) @ w64.T + r
    assert np.abs(y - exact).max() < 1e-4


def test_gemm_tc_swiglu(eng):
    rng = np.random.default_rng(9)
    rows, cols, m = 3072, 1024, 48
    wg = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16)
    wu = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float16)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    g = np.ones(cols, np.float32)
    y = eng.op_gemm_tc(wg, x, w_up=wu, norm_gain=g, epi=eng.TC_EPI_SWIGLU)
    a = _act(x, g, 1e-6, False)
    gate = a @ wg.astype(np.float64).T
    up = a @ wu.astype(np.float64).T
    ref = gate / (1.0 + np.exp(-gate)) * up
    assert np.abs(y - ref).max() < 1e-4 * (1 + np.abs(ref).max())
