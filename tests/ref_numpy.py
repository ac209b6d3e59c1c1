"""Independent NumPy statement of the TTSTransformer graphs (test helper).

Written from src/tts_transformer.cpp directly (not from the C++ oracle), with
weights read by gguf-py's GGUFReader and Q8_0 activations quantised by
gguf-py's quantiser, and float64 accumulation.  It pins the oracle's graph
structure (norms, NEOX RoPE, GQA attention with the causal mask, SwiGLU,
residuals, the F32-cast ffn_down, the code predictor's F32 prefill attention)
for small models; the oracle in turn checks the GPU engine.
"""
from __future__ import annotations

import numpy as np

import gguf

F16, F32, Q8 = gguf.GGMLQuantizationType.F16, gguf.GGMLQuantizationType.F32, gguf.GGMLQuantizationType.Q8_0


def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


class NpModel:
    def __init__(self, path: str):
        r = gguf.GGUFReader(path)
        self.t = {}
        for t in r.tensors:
            self.t[t.name] = (t.tensor_type, np.array(t.data))

        def u(key, d):
            f = r.fields.get(key)
            return d if f is None else f.parts[-1][0].item()

        self.H = u("qwen3-tts.embedding_length", 1024)
        self.L = u("qwen3-tts.block_count", 28)
        self.NH = u("qwen3-tts.attention.head_count", 16)
        self.NKV = u("qwen3-tts.attention.head_count_kv", 8)
        self.D = u("qwen3-tts.attention.key_length", 128)
        self.eps = np.float32(u("qwen3-tts.attention.layer_norm_rms_epsilon", 1e-6))
        self.theta = np.float32(u("qwen3-tts.rope.freq_base", 1e6))
        self.cp_theta = np.float32(u("qwen3-tts.code_predictor.rope.freq_base", float(self.theta)))
        self.cp_layers = u("qwen3-tts.code_predictor.layer_count", 5)
        self.caches = {}

    # --- ops -------------------------------------------------------------
    def vec(self, name):
        return self.t[name][1].astype(np.float32)

    def mul_mat(self, name, x, f32_cast=False):
        ty, w = self.t[name]
        x = np.asarray(x, np.float32)
        if ty == F16:
            xa = x if f32_cast else _f16(x)
            return (xa.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)
        assert ty == Q8
        rows = w.shape[0]
        nb = w.shape[1] // 34
        blk = w.reshape(rows, nb, 34)
        dw = blk[:, :, :2].copy().view(np.float16).astype(np.float64)[:, :, 0]
        qw = blk[:, :, 2:].copy().view(np.int8).astype(np.int64)
        out = np.zeros((x.shape[0], rows), np.float64)
        for v in range(x.shape[0]):
            qa = gguf.quants.quantize(x[v:v + 1], Q8).reshape(nb, 34)
            da = qa[:, :2].copy().view(np.float16).astype(np.float64)[:, 0]
            qav = qa[:, 2:].copy().view(np.int8).astype(np.int64)
            isum = np.einsum("rbj,bj->rb", qw, qav)
            out[v] = (isum * (dw * da[None, :])).sum(axis=1)
        return out.astype(np.float32)

    def rms(self, x, gain):
        x = np.asarray(x, np.float32)
        ss = (x * x).astype(np.float64).sum(axis=-1, keepdims=True)
        mean = (ss / x.shape[-1]).astype(np.float32)
        scale = np.float32(1.0) / np.sqrt(mean + self.eps)
        y = x * scale
        return y if gain is None else y * gain

    def rope(self, x, pos, base):
        D = x.shape[-1]
        s = np.float32(base) ** np.float32(-2.0 / D)
        th = np.float32(pos)
        cs = np.zeros((D // 2, 2), np.float32)
        for i in range(D // 2):
            cs[i] = (np.cos(th), np.sin(th))
            th = np.float32(th * s)
        x0, x1 = x[..., :D // 2], x[..., D // 2:]
        return np.concatenate([x0 * cs[:, 0] - x1 * cs[:, 1], x0 * cs[:, 1] + x1 * cs[:, 0]], axis=-1)

    # --- decoder stack ------------------------------------------------------
    def stack(self, pfx, n_layers, X, n_past, cache_key, theta, f16_kv=True):
        H, NH, NKV, D = self.H, self.NH, self.NKV, self.D
        M = X.shape[0]
        cache = self.caches.setdefault(cache_key, {})
        for il in range(n_layers):
            p = f"{pfx}{il}."
            xn = self.rms(X, self.vec(p + "attn_norm.weight"))
            q = self.mul_mat(p + "attn_q.weight", xn).reshape(M, NH, D)
            k = self.mul_mat(p + "attn_k.weight", xn).reshape(M, NKV, D)
            v = self.mul_mat(p + "attn_v.weight", xn).reshape(M, NKV, D)
            q = self.rms(q, self.vec(p + "attn_q_norm.weight"))
            k = self.rms(k, self.vec(p + "attn_k_norm.weight"))
            q = np.stack([self.rope(q[i], n_past + i, theta) for i in range(M)])
            k = np.stack([self.rope(k[i], n_past + i, theta) for i in range(M)])
            K, V = cache.setdefault(il, ({}, {}))
            for i in range(M):
                K[n_past + i] = k[i].astype(np.float16)
                V[n_past + i] = v[i].astype(np.float16)
            att = np.zeros((M, NH, D), np.float32)
            scale = np.float32(1.0) / np.sqrt(np.float32(D))
            for i in range(M):
                for h in range(NH):
                    g = h // (NH // NKV)
                    if f16_kv:
                        keys = np.stack([K[j][g] for j in range(n_past + i + 1)]).astype(np.float64)
                        vals = np.stack([V[j][g] for j in range(n_past + i + 1)]).astype(np.float64)
                        qh = _f16(q[i, h]).astype(np.float64)
                    else:   # code-predictor 2-token prefill: F32 Kcur/Vcur of this call
                        keys = k[:i + 1, g].astype(np.float64)
                        vals = v[:i + 1, g].astype(np.float64)
                        qh = q[i, h].astype(np.float64)
                    s = (keys @ qh).astype(np.float32) * scale
                    e = np.exp(s - s.max())
                    pr = (e / e.astype(np.float64).sum()).astype(np.float32)
                    if f16_kv:
                        pr = _f16(pr)
                    att[i, h] = (pr.astype(np.float64) @ vals).astype(np.float32)
            X = self.mul_mat(p + "attn_output.weight", att.reshape(M, NH * D)) + X
            xn = self.rms(X, self.vec(p + "ffn_norm.weight"))
            gt = self.mul_mat(p + "ffn_gate.weight", xn)
            up = self.mul_mat(p + "ffn_up.weight", xn)
            hh = (gt / (np.float32(1) + np.exp(-gt))) * up
            X = self.mul_mat(p + "ffn_down.weight", hh, f32_cast=True) + X
        return X

    def talker(self, rows, n_past):
        if n_past == 0:
            self.caches.pop("talker", None)
        X = self.stack("talker.blk.", self.L, np.asarray(rows, np.float32), n_past, "talker", self.theta)
        hid = self.rms(X, self.vec("talker.output_norm.weight"))
        return hid, self.mul_mat("talker.codec_head.weight", hid[-1:])[0]

    def code_predictor(self, hidden, cb0):
        """Greedy predict_codes_autoregressive: returns (codes[15], logits[15][V])."""
        self.caches.pop("cp", None)
        emb = self.t["talker.codec_embd.weight"][1].astype(np.float32)
        X = np.stack([hidden, emb[cb0]])
        codes, logits = [], []
        for g in range(15):
            if g == 0:
                Y = self.stack("code_pred.blk.", self.cp_layers, X, 0, "cp", self.cp_theta, f16_kv=False)
            else:
                e = self.t[f"code_pred.codec_embd.{g - 1}.weight"][1].astype(np.float32)
                Y = self.stack("code_pred.blk.", self.cp_layers, e[codes[-1]][None], g + 1, "cp", self.cp_theta)
            hn = self.rms(Y[-1:], self.vec("code_pred.output_norm.weight"))
            lg = self.mul_mat(f"code_pred.lm_head.{g}.weight", hn)[0]
            logits.append(lg)
            codes.append(int(np.argmax(lg)))
        return np.array(codes), np.stack(logits)


def legacy_predict_codes(path: str, hidden, prev_codes) -> np.ndarray:
    """build_code_pred_graph (src/tts_transformer.cpp:1771-1899), the legacy
    non-autoregressive predictor: one row = hidden + the 15 code-predictor
    embeddings of prev_codes, the code-predictor layers with q/k norms and no
    RoPE, self-attention over that single row (softmax of one score is 1, so
    the output is V), no output norm, then every lm_head on the row.  Returns
    logits [15][V]."""
    m = NpModel(path)
    x = np.asarray(hidden, np.float32).copy()
    for cb in range(15):
        x = x + m.t[f"code_pred.codec_embd.{cb}.weight"][1].astype(np.float32)[int(prev_codes[cb])]
    X = x[None]
    NH, NKV, D = m.NH, m.NKV, m.D
    for il in range(m.cp_layers):
        p = f"code_pred.blk.{il}."
        xn = m.rms(X, m.vec(p + "attn_norm.weight"))
        v = m.mul_mat(p + "attn_v.weight", xn).reshape(NKV, D)
        att = np.concatenate([v[h // (NH // NKV)] for h in range(NH)])[None]
        X = m.mul_mat(p + "attn_output.weight", att) + X
        xn = m.rms(X, m.vec(p + "ffn_norm.weight"))
        gt = m.mul_mat(p + "ffn_gate.weight", xn)
        up = m.mul_mat(p + "ffn_up.weight", xn)
        hh = (gt / (np.float32(1) + np.exp(-gt))) * up
        X = m.mul_mat(p + "ffn_down.weight", hh, f32_cast=True) + X
    return np.stack([m.mul_mat(f"code_pred.lm_head.{g}.weight", X)[0] for g in range(15)])
