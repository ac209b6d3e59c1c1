"""Q8_0 GEMM on the tcgen05 tensor cores (kind::i8, the batched and prefill
paths of Q8_0 models) against a NumPy statement of its arithmetic: weights
quantised by gguf-py (the reference converter's quantiser), activations by the
oracle's quantize_row_q8_0 restatement, per-block int32 dots computed exactly in
int64, then y = sum over blocks in order of float32(isum) * (float32(d_w) *
float32(d_a)) in float32, the k-split partials (block ranges of 128-column
k-tiles per cluster rank) added in rank order.  Store and residual outputs are
compared bit for bit; SwiGLU within 1e-6 relative (exp in the kernel's SiLU)."""
from __future__ import annotations

import numpy as np
import pytest

import gguf
from oracle import quantize_q8_0

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng(qtts):
    import qtts_b200.engine as E
    return E


def _quant_w(rng, rows, cols):
    wf = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    wq = gguf.quants.quantize(wf, gguf.GGMLQuantizationType.Q8_0)
    nb = cols // 32
    blk = wq.reshape(rows, nb, 34)
    q = blk[:, :, 2:].copy().view(np.int8).astype(np.int64)
    d = blk[:, :, :2].copy().view(np.float16).astype(np.float32)[:, :, 0]
    return wq, q, d


def _act(x, gain, eps):
    x = x.astype(np.float32)
    if gain is None:
        return x
    ss = np.sum((x * x).astype(np.float64), axis=1)
    mean = (ss / x.shape[1]).astype(np.float32)
    scale = (np.float32(1.0) / np.sqrt(mean + np.float32(eps))).astype(np.float32)
    return ((x * scale[:, None]).astype(np.float32) * gain.astype(np.float32)).astype(np.float32)


def _ref(q, d, a, S):
    """[m][rows] in the kernel's order: per rank, blocks in order; ranks in order."""
    rows, nb = d.shape
    m = a.shape[0]
    qa = np.zeros((m, nb, 32), np.int64)
    da = np.zeros((m, nb), np.float32)
    for v in range(m):
        qq, dd = quantize_q8_0(a[v])
        qa[v] = qq.reshape(nb, 32)
        da[v] = dd.view(np.float16).astype(np.float32)
    isum = np.einsum("rbk,mbk->mrb", q, qa)                      # exact int64
    nk = nb // 4
    total = np.zeros((m, rows), np.float32)
    for rank in range(S):
        k0, k1 = rank * nk // S, (rank + 1) * nk // S
        acc = np.zeros((m, rows), np.float32)
        for b in range(4 * k0, 4 * k1):
            sc = (d[None, :, b] * da[:, None, b]).astype(np.float32)
            acc = (acc + (isum[:, :, b].astype(np.float32) * sc).astype(np.float32)).astype(np.float32)
        total = (total + acc).astype(np.float32)
    return total


@pytest.mark.parametrize("rows,cols,m,ksplit", [(256, 1024, 32, 1), (4096, 1024, 32, 0), (1024, 3072, 64, 0),
                                                (1024, 2048, 100, 2), (128, 256, 1, 1), (1024, 1024, 16, 8)])
def test_gemm_q8_store_bit_exact(eng, rows, cols, m, ksplit):
    rng = np.random.default_rng(rows + cols + m + ksplit)
    wq, q, d = _quant_w(rng, rows, cols)
    x = rng.standard_normal((m, cols)).astype(np.float32) * rng.uniform(0.05, 4.0, (m, 1)).astype(np.float32)
    y, S = eng.op_gemm_q8(wq, cols, x, ksplit=ksplit)
    assert ksplit == 0 or S == ksplit
    ref = _ref(q, d, x, S)
    assert np.array_equal(y, ref), float(np.abs(y - ref).max())
    # and the GEMM means what it should: float64 of the dequantised operands
    w64 = (q * d[:, :, None].astype(np.float64)).reshape(rows, cols)
    assert np.abs(y - x.astype(np.float64) @ w64.T).max() < 0.05 * (np.abs(ref).max() + 1e-3)


def test_gemm_q8_rmsnorm(eng):
    """The RMSNorm prologue of the activation quantiser: its double sum runs in
    the kernel's thread order, so a last-bit difference of the scale may move an
    int8 level; within 1e-2 of the largest output."""
    rng = np.random.default_rng(5)
    rows, cols, m = 1024, 1024, 32
    wq, q, d = _quant_w(rng, rows, cols)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    g = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    y, S = eng.op_gemm_q8(wq, cols, x, norm_gain=g)
    ref = _ref(q, d, _act(x, g, 1e-6), S)
    assert np.abs(y - ref).max() <= 1e-2 * np.abs(ref).max(), float(np.abs(y - ref).max())


def test_gemm_q8_residual_bit_exact(eng):
    rng = np.random.default_rng(7)
    rows, cols, m = 1024, 3072, 32
    wq, q, d = _quant_w(rng, rows, cols)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    r = rng.standard_normal((m, rows)).astype(np.float32)
    y, S = eng.op_gemm_q8(wq, cols, x, epi=eng.TC_EPI_RESID, resid=r)
    ref = (_ref(q, d, x, S) + r).astype(np.float32)
    assert np.array_equal(y, ref), float(np.abs(y - ref).max())


@pytest.mark.parametrize("ksplit", [1, 0])
def test_gemm_q8_swiglu(eng, ksplit):
    rng = np.random.default_rng(11 + ksplit)
    rows, cols, m = 512, 1024, 48
    wg, qg, dg = _quant_w(rng, rows, cols)
    wu, qu, du = _quant_w(rng, rows, cols)
    x = rng.standard_normal((m, cols)).astype(np.float32)
    y, S = eng.op_gemm_q8(wg, cols, x, w_up=wu, epi=eng.TC_EPI_SWIGLU, ksplit=ksplit)
    a = x
    # the pair tile holds 64 gate rows and the same 64 up rows, so both see the same k-split
    gt = _ref(qg, dg, a, S).astype(np.float64)
    up = _ref(qu, du, a, S).astype(np.float64)
    ref = gt / (1.0 + np.exp(-gt)) * up
    assert np.allclose(y, ref, rtol=1e-6, atol=1e-7), float(np.abs(y - ref).max())
