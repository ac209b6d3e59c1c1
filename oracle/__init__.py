"""CPU oracle for the TTSTransformer decode path (test infrastructure only).

`oracle.Oracle` wraps liboracle.so (built from oracle.cpp by the Makefile
next to this file).  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference legs may import this package; the engine never does.
Parity status: unpinned against ggml (see the header of oracle.cpp).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "liboracle.so")
# OpenMP threads spin only briefly before sleeping between parallel regions: the
# oracle shares the host with the GPU driver thread and other processes.
os.environ.setdefault("GOMP_SPINCOUNT", "20000")


def available_cpus() -> int:
    """CPUs this process may actually use (affinity and cgroup CPU quota)."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    try:
        quota, period = open("/sys/fs/cgroup/cpu.max").read().split()[:2]
        if quota != "max":
            n = min(n, max(1, int(int(quota) / int(period))))
    except (OSError, ValueError):
        pass
    try:
        q = int(open("/sys/fs/cgroup/cpu/cpu.cfs_quota_us").read())
        p = int(open("/sys/fs/cgroup/cpu/cpu.cfs_period_us").read())
        if q > 0:
            n = min(n, max(1, q // p))
    except (OSError, ValueError):
        pass
    return max(1, n)


def build(force: bool = False) -> str:
    src = os.path.join(_HERE, "oracle.cpp")
    if force or not os.path.exists(_LIB) or os.path.getmtime(_LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB


class GenArgs(C.Structure):
    _fields_ = [
        ("text", C.POINTER(C.c_int32)), ("n_text", C.c_int32),
        ("ref_text", C.POINTER(C.c_int32)), ("n_ref_text", C.c_int32),
        ("ref_codes", C.POINTER(C.c_int32)), ("n_ref_frames", C.c_int32),
        ("speaker", C.POINTER(C.c_float)),
        ("max_len", C.c_int32), ("language_id", C.c_int32),
        ("rep_penalty", C.c_float), ("temperature", C.c_float), ("top_k", C.c_int32),
        ("instruct", C.POINTER(C.c_int32)), ("n_instruct", C.c_int32),
        ("eos_bias", C.c_float), ("target_frames", C.c_int32), ("rep_loop_detect", C.c_int32),
        ("seed", C.c_uint64),
        ("follow", C.POINTER(C.c_int32)), ("n_follow", C.c_int32), ("tie_tol", C.c_float),
        ("codes_out", C.POINTER(C.c_int32)), ("codes_cap", C.c_int32),
        ("talker_logits_out", C.POINTER(C.c_float)),
        ("cp_logits_out", C.POINTER(C.c_float)),
        ("prefill_out", C.POINTER(C.c_float)), ("prefill_cap", C.c_int32),
    ]


class GenResult(C.Structure):
    _fields_ = [
        ("n_frames", C.c_int32), ("prefill_len", C.c_int32), ("n_mismatch", C.c_int32),
        ("n_ties", C.c_int32), ("first_mismatch", C.c_int32), ("truncated", C.c_int32),
        ("max_tie_gap", C.c_float), ("min_decision_gap", C.c_float), ("max_mismatch_gap", C.c_float),
    ]


def _p(a, ct):
    return None if a is None else a.ctypes.data_as(C.POINTER(ct))


CONFIG_KEYS = ["text_vocab", "text_dim", "hidden", "n_layers", "n_heads", "n_kv", "ffn", "head_dim",
               "codec_vocab", "n_cb", "cp_layers", "cp_vocab", "cp_hidden", "cp_ffn", "codec_pad",
               "codec_bos", "codec_eos", "tts_bos", "tts_eos", "tts_pad", "think", "nothink",
               "think_bos", "think_eos", "english"]


class Oracle:
    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            L = C.CDLL(build())
            L.orc_load.restype = C.c_void_p
            L.orc_load.argtypes = [C.c_char_p, C.c_char_p, C.c_int]
            L.orc_free.argtypes = [C.c_void_p]
            L.orc_config.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.POINTER(C.c_float)]
            L.orc_init_kv.argtypes = [C.c_void_p, C.c_int]
            L.orc_lookup_rows.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_int32), C.c_int, C.POINTER(C.c_float)]
            L.orc_project_text.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.POINTER(C.c_float)]
            L.orc_forward_prefill.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.c_int, C.c_int,
                                              C.POINTER(C.c_float), C.POINTER(C.c_float)]
            L.orc_forward_step.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.c_int,
                                           C.POINTER(C.c_float), C.POINTER(C.c_float)]
            L.orc_predict_codes_ar.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.c_int, C.c_float, C.c_int,
                                               C.c_uint64, C.c_uint32, C.POINTER(C.c_int32), C.POINTER(C.c_float)]
            L.orc_generate.argtypes = [C.c_void_p, C.POINTER(GenArgs), C.POINTER(GenResult)]
            L.orc_quantize_q8_0.argtypes = [C.POINTER(C.c_float), C.c_int, C.POINTER(C.c_int8), C.POINTER(C.c_uint16)]
            L.orc_rope_cache.argtypes = [C.c_int, C.c_int, C.c_float, C.POINTER(C.c_float)]
            L.orc_uniform01.restype = C.c_double
            L.orc_uniform01.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32]
            L.orc_philox.argtypes = [C.POINTER(C.c_uint32), C.c_uint32, C.c_uint32]
            L.orc_sample.argtypes = [C.POINTER(C.c_float), C.c_int, C.c_float, C.c_int, C.c_double]
            L.orc_forward_talker_rows.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.c_int, C.c_int]
            L.orc_set_threads.argtypes = [C.c_int]
            L.orc_set_attn_dump.restype = None
            L.orc_set_attn_dump.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
            L.orc_attn_rows.restype = C.c_int
            L.orc_attn_rows.argtypes = []
            L.orc_set_engine_order.argtypes = [C.c_int]
            L.orc_set_frame_split.argtypes = [C.c_int]
            L.orc_expf.restype = C.c_float
            L.orc_expf.argtypes = [C.c_float]
            cls._lib = L
        return cls._lib

    def __init__(self, path: str, threads: int | None = None, engine_order: bool = True,
                 frame_split: bool | None = None):
        """engine_order: run every reduction in the engine's order (the parity
        checker's mode; process-wide); False: plain sequential / AVX2 orders,
        used for the CPU baseline timing.  frame_split: in generate()'s frame
        loop, restate the engine's fused frame path (O-projection and ffn_down
        as ordered partial sums, see oracle.cpp); default: on when
        QTTS_FRAME_MODE=fused selects that path in the engine."""
        L = self.lib()
        L.orc_set_threads(int(threads) if threads else available_cpus())
        L.orc_set_engine_order(1 if engine_order else 0)
        if frame_split is None:
            frame_split = os.environ.get("QTTS_FRAME_MODE", "") == "fused"
        L.orc_set_frame_split(1 if frame_split else 0)
        err = C.create_string_buffer(512)
        self.h = L.orc_load(path.encode(), err, 512)
        if not self.h:
            raise RuntimeError("oracle load failed: " + err.value.decode())
        iv = (C.c_int32 * 32)()
        fv = (C.c_float * 4)()
        n = L.orc_config(self.h, iv, fv)
        self.cfg = dict(zip(CONFIG_KEYS, list(iv)[:n]))
        self.cfg.update(eps=fv[0], theta=fv[1], cp_theta=fv[2])

    def generate_with_attn_dump(self, layer: int, stride: int, max_rows: int, **kw):
        """generate(**kw) while recording the post-softmax rows of talker layer
        `layer` at every decode step: returns (generate's result, rows
        [n][n_heads][stride], zero beyond each row's key count)."""
        nh = self.cfg["n_heads"]
        buf = np.zeros((max_rows, nh, stride), np.float32)
        L = self.lib()
        L.orc_set_attn_dump(buf.ctypes.data_as(C.c_void_p), max_rows, stride, layer)
        try:
            r = self.generate(**kw)
            n = L.orc_attn_rows()
        finally:
            L.orc_set_attn_dump(None, 0, 0, -1)
        return r, buf[:n].copy()

    def close(self):
        if self.h:
            self.lib().orc_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- components
    def lookup(self, which: int, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        dim = self.cfg["text_dim"] if which < 0 else self.cfg["hidden"]
        out = np.zeros((len(ids), dim), np.float32)
        assert self.lib().orc_lookup_rows(self.h, which, _p(ids, C.c_int32), len(ids), _p(out, C.c_float)) == 0
        return out

    def project_text(self, toks) -> np.ndarray:
        toks = np.ascontiguousarray(toks, dtype=np.int32)
        out = np.zeros((len(toks), self.cfg["hidden"]), np.float32)
        assert self.lib().orc_project_text(self.h, _p(toks, C.c_int32), len(toks), _p(out, C.c_float)) == 0
        return out

    def init_kv(self, n_ctx: int):
        self.lib().orc_init_kv(self.h, n_ctx)

    def forward_prefill(self, embd: np.ndarray, n_past: int = 0):
        embd = np.ascontiguousarray(embd, dtype=np.float32)
        n = embd.shape[0]
        hid = np.zeros((n, self.cfg["hidden"]), np.float32)
        lg = np.zeros(self.cfg["codec_vocab"], np.float32)
        assert self.lib().orc_forward_prefill(self.h, _p(embd, C.c_float), n, n_past, _p(hid, C.c_float),
                                              _p(lg, C.c_float)) == 0
        return hid, lg

    def forward_step(self, embd: np.ndarray, n_past: int):
        embd = np.ascontiguousarray(embd, dtype=np.float32)
        hid = np.zeros(self.cfg["hidden"], np.float32)
        lg = np.zeros(self.cfg["codec_vocab"], np.float32)
        assert self.lib().orc_forward_step(self.h, _p(embd, C.c_float), n_past, _p(lg, C.c_float),
                                           _p(hid, C.c_float)) == 0
        return lg, hid

    def predict_codes(self, hidden, cb0: int, temperature=0.0, top_k=0, seed=0, frame=0):
        hidden = np.ascontiguousarray(hidden, dtype=np.float32)
        ng = self.cfg["n_cb"] - 1
        codes = np.zeros(ng, np.int32)
        lg = np.zeros((ng, self.cfg["cp_vocab"]), np.float32)
        self.lib().orc_predict_codes_ar(self.h, _p(hidden, C.c_float), int(cb0), float(temperature), int(top_k),
                                        int(seed), int(frame), _p(codes, C.c_int32), _p(lg, C.c_float))
        return codes, lg

    def generate(self, text, max_len, *, speaker=None, ref_text=None, ref_codes=None, language_id=2050,
                 rep_penalty=1.05, temperature=0.0, top_k=0, instruct=None, eos_bias=0.0, target_frames=0,
                 rep_loop_detect=False, seed=0, follow=None, tie_tol=1e-3, want_logits=False,
                 want_prefill=False):
        cfg = self.cfg
        text = np.ascontiguousarray(text, dtype=np.int32)
        keep = [text]
        a = GenArgs()
        a.text, a.n_text = _p(text, C.c_int32), len(text)
        if ref_codes is not None:
            ref_codes = np.ascontiguousarray(ref_codes, dtype=np.int32).reshape(-1, 16)
            ref_text = np.ascontiguousarray(ref_text if ref_text is not None else [], dtype=np.int32)
            keep += [ref_codes, ref_text]
            a.ref_codes, a.n_ref_frames = _p(ref_codes, C.c_int32), ref_codes.shape[0]
            a.ref_text, a.n_ref_text = _p(ref_text, C.c_int32), len(ref_text)
        if speaker is not None:
            speaker = np.ascontiguousarray(speaker, dtype=np.float32)
            keep.append(speaker)
            a.speaker = _p(speaker, C.c_float)
        if instruct is not None:
            instruct = np.ascontiguousarray(instruct, dtype=np.int32)
            keep.append(instruct)
            a.instruct, a.n_instruct = _p(instruct, C.c_int32), len(instruct)
        a.max_len, a.language_id = max_len, language_id
        a.rep_penalty, a.temperature, a.top_k = rep_penalty, temperature, top_k
        a.eos_bias, a.target_frames, a.rep_loop_detect = eos_bias, target_frames, int(rep_loop_detect)
        a.seed = seed
        if follow is not None:
            follow = np.ascontiguousarray(follow, dtype=np.int32).reshape(-1, cfg["n_cb"])
            keep.append(follow)
            a.follow, a.n_follow = _p(follow, C.c_int32), follow.shape[0]
        a.tie_tol = tie_tol
        codes = np.zeros((max_len, cfg["n_cb"]), np.int32)
        a.codes_out, a.codes_cap = _p(codes, C.c_int32), max_len
        tl = cl = pf = None
        if want_logits:
            tl = np.zeros((max_len, cfg["codec_vocab"]), np.float32)
            cl = np.zeros((max_len, cfg["n_cb"] - 1, cfg["cp_vocab"]), np.float32)
            a.talker_logits_out, a.cp_logits_out = _p(tl, C.c_float), _p(cl, C.c_float)
        if want_prefill:
            cap = 4096
            pf = np.zeros((cap, cfg["hidden"]), np.float32)
            a.prefill_out, a.prefill_cap = _p(pf, C.c_float), cap
        r = GenResult()
        rc = self.lib().orc_generate(self.h, C.byref(a), C.byref(r))
        if rc != 0:
            raise RuntimeError(f"oracle generate failed ({rc})")
        n = r.n_frames
        out = dict(codes=codes[:n].copy(), n_frames=n, prefill_len=r.prefill_len, n_mismatch=r.n_mismatch,
                   n_ties=r.n_ties, first_mismatch=r.first_mismatch, truncated=bool(r.truncated),
                   max_tie_gap=r.max_tie_gap, min_decision_gap=r.min_decision_gap,
                   max_mismatch_gap=r.max_mismatch_gap)
        if want_logits:
            out["talker_logits"] = tl[:max(n, 1)]
            out["cp_logits"] = cl[:n]
        if want_prefill:
            out["prefill"] = pf[:r.prefill_len].copy()
        return out


def expf(x) -> np.ndarray:
    """The oracle's exp (Cody-Waite + degree-7 Taylor, as the engine's)."""
    L = Oracle.lib()
    return np.array([L.orc_expf(float(v)) for v in np.ravel(np.asarray(x, np.float32))], np.float32)


def quantize_q8_0(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    q = np.zeros(x.size, np.int8)
    d = np.zeros(x.size // 32, np.uint16)
    Oracle.lib().orc_quantize_q8_0(_p(x, C.c_float), x.size, _p(q, C.c_int8), _p(d, C.c_uint16))
    return q, d


def rope_cache(pos: int, n_dims: int, base: float) -> np.ndarray:
    cs = np.zeros(n_dims, np.float32)
    Oracle.lib().orc_rope_cache(pos, n_dims, base, _p(cs, C.c_float))
    return cs


def uniform01(seed: int, frame: int, cb: int) -> float:
    return Oracle.lib().orc_uniform01(seed, frame, cb)


def philox(counter, key):
    c = (C.c_uint32 * 4)(*counter)
    Oracle.lib().orc_philox(c, key[0], key[1])
    return list(c)
