"""ctypes binding of the engine's C ABI (include/qwen3tts_b200.h).

This is a thin host-side mirror of the reference's TTSTransformer interface
(src/tts_transformer.h:198-330) for Python callers, the tests and bench.py.
All compute runs in libqwen3tts_b200.so on the GPU; if the library or a GPU is
missing, construction raises instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build as _build

_i32p = C.POINTER(C.c_int32)
_f32p = C.POINTER(C.c_float)


class Config(C.Structure):
    _fields_ = [
        ("text_vocab_size", C.c_int32), ("text_embd_dim", C.c_int32),
        ("hidden_size", C.c_int32), ("n_layers", C.c_int32), ("n_attention_heads", C.c_int32),
        ("n_key_value_heads", C.c_int32), ("intermediate_size", C.c_int32), ("head_dim", C.c_int32),
        ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float), ("mrope_section", C.c_int32 * 3),
        ("codec_vocab_size", C.c_int32), ("n_codebooks", C.c_int32),
        ("code_pred_layers", C.c_int32), ("code_pred_vocab_size", C.c_int32),
        ("code_pred_hidden_size", C.c_int32), ("code_pred_intermediate_size", C.c_int32),
        ("code_pred_rope_theta", C.c_float),
        ("codec_pad_id", C.c_int32), ("codec_bos_id", C.c_int32), ("codec_eos_id", C.c_int32),
        ("tts_bos_token_id", C.c_int32), ("tts_eos_token_id", C.c_int32), ("tts_pad_token_id", C.c_int32),
        ("codec_think_id", C.c_int32), ("codec_nothink_id", C.c_int32), ("codec_think_bos_id", C.c_int32),
        ("codec_think_eos_id", C.c_int32), ("english_language_id", C.c_int32), ("weight_type", C.c_int32),
    ]

    def as_dict(self):
        d = {k: getattr(self, k) for k, _ in self._fields_}
        d["mrope_section"] = list(self.mrope_section)
        return d


class GenParams(C.Structure):
    _fields_ = [
        ("text_tokens", _i32p), ("n_tokens", C.c_int32),
        ("ref_text_tokens", _i32p), ("n_ref_text", C.c_int32),
        ("ref_codec_tokens", _i32p), ("n_ref_frames", C.c_int32),
        ("speaker_embd", _f32p),
        ("max_len", C.c_int32), ("language_id", C.c_int32),
        ("repetition_penalty", C.c_float), ("temperature", C.c_float), ("top_k", C.c_int32),
        ("instruct_tokens", _i32p), ("n_instruct", C.c_int32),
        ("eos_bias", C.c_float), ("target_frames", C.c_int32), ("rep_loop_detect", C.c_int32),
        ("seed", C.c_uint64),
    ]


class Timing(C.Structure):
    _fields_ = [("prefill_ms", C.c_float), ("frames_ms", C.c_float), ("frames", C.c_int32),
                ("kernel_launches", C.c_int32), ("load_ms", C.c_float)]


class StageTiming(C.Structure):
    _fields_ = [("prefill_build_ms", C.c_float), ("prefill_forward_ms", C.c_float), ("talker_ms", C.c_float),
                ("code_pred_ms", C.c_float), ("sample_embed_ms", C.c_float), ("total_ms", C.c_float),
                ("frames", C.c_int32)]


class KernelStats(C.Structure):
    _fields_ = [("launches", C.c_int32), ("total_ms", C.c_float), ("bytes", C.c_double)]


KERNEL_CLASSES = ["gemv", "attention", "sample", "other"]

FRAME_CB = C.CFUNCTYPE(C.c_int32, _i32p, C.c_int32, C.c_int32, C.c_void_p)

_lib = None


def lib():
    """Load (building first if stale) libqwen3tts_b200.so and declare the ABI."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.build()
    L = C.CDLL(path)
    sig = {
        "qtts_create": (C.c_void_p, [C.c_char_p, C.c_int32]),
        "qtts_create_error": (C.c_char_p, []),
        "qtts_destroy": (None, [C.c_void_p]),
        "qtts_get_error": (C.c_char_p, [C.c_void_p]),
        "qtts_get_config": (C.c_int32, [C.c_void_p, C.POINTER(Config)]),
        "qtts_set_n_threads": (None, [C.c_void_p, C.c_int32]),
        "qtts_init_kv_cache": (C.c_int32, [C.c_void_p, C.c_int32]),
        "qtts_clear_kv_cache": (None, [C.c_void_p]),
        "qtts_init_code_pred_kv_cache": (C.c_int32, [C.c_void_p, C.c_int32]),
        "qtts_clear_code_pred_kv_cache": (None, [C.c_void_p]),
        "qtts_forward_prefill": (C.c_int32, [C.c_void_p, _f32p, C.c_int32, C.c_int32, _f32p, _f32p]),
        "qtts_forward_step": (C.c_int32, [C.c_void_p, _f32p, C.c_int32, _f32p, _f32p]),
        "qtts_forward_text": (C.c_int32, [C.c_void_p, _i32p, C.c_int32, _f32p, C.c_int32, _f32p]),
        "qtts_forward_codec": (C.c_int32, [C.c_void_p, C.c_int32, C.c_int32, _f32p]),
        "qtts_get_hidden_states": (C.c_int32, [C.c_void_p, _f32p]),
        "qtts_predict_codes": (C.c_int32, [C.c_void_p, _f32p, _i32p, _f32p]),
        "qtts_predict_codes_autoregressive": (C.c_int32, [C.c_void_p, _f32p, C.c_int32, C.c_float, C.c_int32, _i32p]),
        "qtts_project_text": (C.c_int32, [C.c_void_p, _i32p, C.c_int32, _f32p]),
        "qtts_lookup_embedding_rows": (C.c_int32, [C.c_void_p, C.c_int32, _i32p, C.c_int32, _f32p]),
        "qtts_generate": (C.c_int32, [C.c_void_p, C.POINTER(GenParams), FRAME_CB, C.c_void_p, _i32p, _i32p]),
        "qtts_generate_begin": (C.c_int32, [C.c_void_p, C.POINTER(GenParams)]),
        "qtts_run_frames": (C.c_int32, [C.c_void_p, C.c_int32, _i32p]),
        "qtts_generate_rewind": (C.c_int32, [C.c_void_p]),
        "qtts_codes_device": (C.c_int32, [C.c_void_p, C.POINTER(C.c_void_p), _i32p]),
        "qtts_set_seed": (None, [C.c_void_p, C.c_uint64]),
        "qtts_set_debug_logits": (C.c_int32, [C.c_void_p, _f32p, _f32p, C.c_int32]),
        "qtts_set_attn_dump": (C.c_int32, [C.c_void_p, C.c_int32, C.c_int32]),
        "qtts_attn_rows": (C.c_int32, [C.c_void_p]),
        "qtts_attn_row": (C.c_int32, [C.c_void_p, C.c_int32, _f32p, C.c_int32]),
        "qtts_get_timing": (C.c_int32, [C.c_void_p, C.POINTER(Timing)]),
        "qtts_set_stage_timing": (C.c_int32, [C.c_void_p, C.c_int32]),
        "qtts_get_frame_mode": (C.c_int32, [C.c_void_p]),
        "qtts_frame_trace": (C.c_int32, [C.c_void_p, C.POINTER(C.c_uint64), C.c_int32, _i32p, C.c_int32]),
        "qtts_get_stage_timing": (C.c_int32, [C.c_void_p, C.POINTER(StageTiming)]),
        "qtts_profile_frames": (C.c_int32, [C.c_void_p, C.c_int32, C.POINTER(KernelStats), C.c_int32]),
        "qtts_batch_create": (C.c_void_p, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32]),
        "qtts_batch_begin": (C.c_int32, [C.c_void_p, C.c_int32, C.c_void_p]),
        "qtts_batch_run": (C.c_int32, [C.c_void_p, C.c_int32]),
        "qtts_batch_codes": (C.c_int32, [C.c_void_p, _i32p, _i32p]),
        "qtts_batch_codes_device": (C.c_int32, [C.c_void_p, C.POINTER(C.c_void_p), _i32p]),
        "qtts_batch_timing": (C.c_int32, [C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_int32),
                                          C.POINTER(C.c_int32)]),
        "qtts_batch_error": (C.c_char_p, [C.c_void_p]),
        "qtts_batch_profile": (C.c_int32, [C.c_void_p, C.c_int32, _f32p, _i32p]),
        "qtts_batch_free": (None, [C.c_void_p]),
        "qtts_op_gemm_q8": (C.c_int32, [C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, _f32p, C.c_int32,
                                        _f32p, C.c_float, C.c_int32, _f32p, C.c_int32, _f32p]),
        "qtts_op_gemm_tc": (C.c_int32, [C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, _f32p, C.c_int32,
                                        _f32p, C.c_float, C.c_int32, C.c_int32, _f32p, _f32p]),
        "qtts_op_gemv": (C.c_int32, [C.c_int32, C.c_int32, C.c_void_p, C.c_int32, C.c_int32, _f32p, C.c_int32, _f32p,
                                     C.c_float, C.c_int32, _f32p, _i32p]),
        "qtts_op_sample": (C.c_int32, [C.c_int32, _f32p, C.c_int32, C.c_int32, C.c_float, C.c_int32, C.c_float, _i32p,
                                       C.c_float, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_uint64]),
        "qtts_op_sample_noalloc": (C.c_int32, [C.c_int32, C.c_void_p, C.c_int32, C.c_int32, C.c_float, C.c_int32,
                                               C.c_float, C.c_void_p, C.c_float, C.c_int32, C.c_int32, C.c_int32,
                                               C.c_int32, C.c_uint64, C.c_void_p, C.c_void_p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def exported_symbols():
    return [n for n in dir(lib()) if n.startswith("qtts_")]


def _p(a, ct):
    return None if a is None else a.ctypes.data_as(C.POINTER(ct))


class Engine:
    """One engine = one GPU, one sequence at a time (as TTSTransformer)."""

    def __init__(self, gguf_path: str, device: int = 0):
        L = lib()
        self.h = L.qtts_create(gguf_path.encode(), int(device))
        if not self.h:
            raise RuntimeError("qtts_create failed: " + (L.qtts_create_error() or b"").decode())
        c = Config()
        L.qtts_get_config(self.h, C.byref(c))
        self.cfg = c.as_dict()
        self._dbg = None

    def close(self):
        if getattr(self, "h", None):
            lib().qtts_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def error(self) -> str:
        return (lib().qtts_get_error(self.h) or b"").decode()

    def _ok(self, rc, what):
        if not rc:
            raise RuntimeError(f"{what} failed: {self.error()}")

    # ---- TTSTransformer members
    def init_kv_cache(self, n_ctx: int):
        self._ok(lib().qtts_init_kv_cache(self.h, n_ctx), "init_kv_cache")

    def clear_kv_cache(self):
        lib().qtts_clear_kv_cache(self.h)

    def forward_prefill(self, embd: np.ndarray, n_past: int = 0):
        embd = np.ascontiguousarray(embd, dtype=np.float32)
        n = embd.shape[0]
        hid = np.zeros((n, self.cfg["hidden_size"]), np.float32)
        lg = np.zeros(self.cfg["codec_vocab_size"], np.float32)
        self._ok(lib().qtts_forward_prefill(self.h, _p(embd, C.c_float), n, n_past, _p(hid, C.c_float),
                                            _p(lg, C.c_float)), "forward_prefill")
        return hid, lg

    def forward_step(self, embd: np.ndarray, n_past: int):
        embd = np.ascontiguousarray(embd, dtype=np.float32)
        lg = np.zeros(self.cfg["codec_vocab_size"], np.float32)
        hid = np.zeros(self.cfg["hidden_size"], np.float32)
        self._ok(lib().qtts_forward_step(self.h, _p(embd, C.c_float), n_past, _p(lg, C.c_float), _p(hid, C.c_float)),
                 "forward_step")
        return lg, hid

    def predict_codes_autoregressive(self, hidden, cb0: int, temperature: float = 0.0, top_k: int = 0):
        hidden = np.ascontiguousarray(hidden, dtype=np.float32)
        out = np.zeros(self.cfg["n_codebooks"] - 1, np.int32)
        self._ok(lib().qtts_predict_codes_autoregressive(self.h, _p(hidden, C.c_float), int(cb0), float(temperature),
                                                         int(top_k), _p(out, C.c_int32)), "predict_codes_autoregressive")
        return out

    def predict_codes(self, hidden, prev_codes=None):
        hidden = np.ascontiguousarray(hidden, dtype=np.float32)
        pc = None if prev_codes is None else np.ascontiguousarray(prev_codes, dtype=np.int32)
        out = np.zeros((self.cfg["n_codebooks"] - 1, self.cfg["code_pred_vocab_size"]), np.float32)
        self._ok(lib().qtts_predict_codes(self.h, _p(hidden, C.c_float), _p(pc, C.c_int32), _p(out, C.c_float)),
                 "predict_codes")
        return out

    def project_text(self, toks) -> np.ndarray:
        toks = np.ascontiguousarray(toks, dtype=np.int32)
        out = np.zeros((len(toks), self.cfg["hidden_size"]), np.float32)
        self._ok(lib().qtts_project_text(self.h, _p(toks, C.c_int32), len(toks), _p(out, C.c_float)), "project_text")
        return out

    def lookup(self, table: int, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        dim = self.cfg["text_embd_dim"] if table < 0 else self.cfg["hidden_size"]
        out = np.zeros((len(ids), dim), np.float32)
        self._ok(lib().qtts_lookup_embedding_rows(self.h, table, _p(ids, C.c_int32), len(ids), _p(out, C.c_float)),
                 "lookup_embedding_rows")
        return out

    def set_seed(self, seed: int):
        lib().qtts_set_seed(self.h, int(seed))

    def frame_trace(self):
        """(kinds [n_launches], stamps [n_launches][256][8]) of frame 1 of the last
        run with QTTS_FF_TRACE=1 at load time (ns, %globaltimer, 0 = not reached);
        kinds: kind * 4 + (samples ? 2 : 0) + rows - 1, kind 0 attention block, 1
        FFN block, 2 head."""
        kinds = np.zeros(512, np.int32)
        n = lib().qtts_frame_trace(self.h, None, 0, _p(kinds, C.c_int32), 512)
        tr = np.zeros((max(n, 1), 256, 8), np.uint64)
        lib().qtts_frame_trace(self.h, tr.ctypes.data_as(C.POINTER(C.c_uint64)), tr.size, _p(kinds, C.c_int32), 512)
        return kinds[:n], tr[:n]

    def frame_mode(self) -> str:
        """The frame path: "graph" (one kernel per op, the default) or "fused" (two
        clustered kernels per layer; QTTS_FRAME_MODE=fused at load time)."""
        return "fused" if lib().qtts_get_frame_mode(self.h) == 1 else "graph"

    def timing(self) -> dict:
        t = Timing()
        lib().qtts_get_timing(self.h, C.byref(t))
        return dict(prefill_ms=t.prefill_ms, frames_ms=t.frames_ms, frames=t.frames, kernel_launches=t.kernel_launches,
                    load_ms=t.load_ms)

    def set_stage_timing(self, enabled: bool):
        self._ok(lib().qtts_set_stage_timing(self.h, int(enabled)), "set_stage_timing")

    def stage_timing(self) -> dict:
        t = StageTiming()
        lib().qtts_get_stage_timing(self.h, C.byref(t))
        return {k: getattr(t, k) for k, _ in StageTiming._fields_}

    def _params(self, text, max_len, speaker, ref_text, ref_codes, language_id, rep_penalty, temperature, top_k,
                instruct, eos_bias, target_frames, rep_loop_detect, seed):
        keep = []
        p = GenParams()

        def arr(a, dt):
            a = np.ascontiguousarray(a, dtype=dt)
            keep.append(a)
            return a

        t = arr(text, np.int32)
        p.text_tokens, p.n_tokens = _p(t, C.c_int32), len(t)
        if ref_codes is not None:
            rc = arr(np.asarray(ref_codes).reshape(-1, 16), np.int32)
            rt = arr(ref_text if ref_text is not None else [], np.int32)
            p.ref_codec_tokens, p.n_ref_frames = _p(rc, C.c_int32), rc.shape[0]
            p.ref_text_tokens, p.n_ref_text = _p(rt, C.c_int32), len(rt)
        if speaker is not None:
            s = arr(speaker, np.float32)
            p.speaker_embd = _p(s, C.c_float)
        if instruct is not None:
            ins = arr(instruct, np.int32)
            p.instruct_tokens, p.n_instruct = _p(ins, C.c_int32), len(ins)
        p.max_len, p.language_id = max_len, language_id
        p.repetition_penalty, p.temperature, p.top_k = rep_penalty, temperature, top_k
        p.eos_bias, p.target_frames, p.rep_loop_detect = eos_bias, target_frames, int(rep_loop_detect)
        p.seed = seed
        return p, keep

    def generate(self, text, max_len, *, speaker=None, ref_text=None, ref_codes=None, language_id=2050,
                 rep_penalty=1.05, temperature=0.0, top_k=0, instruct=None, eos_bias=0.0, target_frames=0,
                 rep_loop_detect=False, seed=0, on_frame=None, want_logits=False):
        p, keep = self._params(text, max_len, speaker, ref_text, ref_codes, language_id, rep_penalty, temperature,
                               top_k, instruct, eos_bias, target_frames, rep_loop_detect, seed)
        ncb = self.cfg["n_codebooks"]
        tl = cl = None
        if want_logits:
            tl = np.zeros((max_len, self.cfg["codec_vocab_size"]), np.float32)
            cl = np.zeros((max_len, ncb - 1, self.cfg["code_pred_vocab_size"]), np.float32)
            lib().qtts_set_debug_logits(self.h, _p(tl, C.c_float), _p(cl, C.c_float), max_len)
        codes = np.zeros((max(max_len, 1), ncb), np.int32)
        n = C.c_int32(0)
        cb = FRAME_CB(0)
        if on_frame is not None:
            def _cb(ptr, n_cb, frame, user):
                return 1 if on_frame(np.ctypeslib.as_array(ptr, shape=(n_cb,)).copy(), frame) else 0
            cb = FRAME_CB(_cb)
        try:
            self._ok(lib().qtts_generate(self.h, C.byref(p), cb, None, _p(codes, C.c_int32), C.byref(n)), "generate")
        finally:
            if want_logits:
                lib().qtts_set_debug_logits(self.h, None, None, 0)
        out = dict(codes=codes[:n.value].copy(), n_frames=n.value)
        if want_logits:
            out["talker_logits"] = tl
            out["cp_logits"] = cl[:n.value]
        return out

    def generate_begin(self, text, max_len, **kw) -> int:
        args = dict(speaker=None, ref_text=None, ref_codes=None, language_id=2050, rep_penalty=1.05, temperature=0.0,
                    top_k=0, instruct=None, eos_bias=0.0, target_frames=0, rep_loop_detect=False, seed=0)
        args.update(kw)
        p, keep = self._params(text, max_len, **args)
        self._keep = keep
        rc = lib().qtts_generate_begin(self.h, C.byref(p))
        if rc < 0:
            raise RuntimeError("generate_begin failed: " + self.error())
        return rc

    def profile_frames(self, n: int) -> dict:
        st = (KernelStats * 4)()
        got = lib().qtts_profile_frames(self.h, n, st, 4)
        if got < 0:
            raise RuntimeError("profile_frames failed: " + self.error())
        return {"frames": got, **{KERNEL_CLASSES[i]: dict(launches=st[i].launches, ms=st[i].total_ms, bytes=st[i].bytes)
                                  for i in range(4)}}

    def run_frames(self, n: int, codes_out: np.ndarray | None = None) -> int:
        ptr = None if codes_out is None else _p(codes_out, C.c_int32)
        rc = lib().qtts_run_frames(self.h, n, ptr)
        if rc < 0:
            raise RuntimeError("run_frames failed: " + self.error())
        return rc

    def generate_rewind(self) -> None:
        """Back to frame 0 of the active generation (replay without a new prefill)."""
        if lib().qtts_generate_rewind(self.h) < 0:
            raise RuntimeError("rewind failed: " + self.error())

    def codes_device(self):
        """(device address of the code buffer [max_len][n_codebooks] int32, frames
        generated): the codes -> vocoder handoff without a host copy."""
        ptr = C.c_void_p()
        n = np.zeros(1, np.int32)
        if lib().qtts_codes_device(self.h, C.byref(ptr), _p(n, C.c_int32)) < 0:
            raise RuntimeError("codes_device failed: " + self.error())
        return int(ptr.value or 0), int(n[0])


def op_gemv(w, wtype: int, rows: int, cols: int, x, norm_gain=None, eps=1e-6, act_f32=False, want_block_dots=False,
            device: int = 0):
    """Run the engine's GEMV kernel once: returns y [nv][rows] (and block dots)."""
    w = np.ascontiguousarray(w)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
    nv = x.shape[0]
    y = np.zeros((nv, rows), np.float32)
    g = None if norm_gain is None else np.ascontiguousarray(norm_gain, dtype=np.float32)
    bd = np.zeros((nv, rows, cols // 32), np.int32) if want_block_dots else None
    rc = lib().qtts_op_gemv(device, wtype, w.ctypes.data_as(C.c_void_p), rows, cols, _p(x, C.c_float), nv,
                            _p(g, C.c_float), eps, int(act_f32), _p(y, C.c_float), _p(bd, C.c_int32))
    if not rc:
        raise RuntimeError("qtts_op_gemv failed")
    return (y, bd) if want_block_dots else y


_GEN_DEFAULTS = dict(speaker=None, ref_text=None, ref_codes=None, language_id=2050, rep_penalty=1.05, temperature=0.0,
                     top_k=0, instruct=None, eos_bias=0.0, target_frames=0, rep_loop_detect=False, seed=0)


class Batch:
    """Batched frame loop (qtts_batch_*): up to max_batch utterances advance one
    frame per step together on the engine's GPU, sharing its weights."""

    def __init__(self, eng: "Engine", max_batch: int, max_positions: int, max_frames: int):
        self.eng = eng
        self.max_frames = max_frames
        self.ncb = eng.cfg["n_codebooks"]
        self.h = lib().qtts_batch_create(eng.h, max_batch, max_positions, max_frames)
        if not self.h:
            raise RuntimeError("batch create failed: " + eng.error())
        self.n = 0

    def error(self) -> str:
        return lib().qtts_batch_error(self.h).decode()

    def begin(self, utterances) -> None:
        """utterances: list of dicts with `text`, `max_len` and generate()'s keyword arguments."""
        n = len(utterances)
        params = (GenParams * n)()
        self._keep = []
        for i, u in enumerate(utterances):
            args = dict(_GEN_DEFAULTS)
            args.update({k: v for k, v in u.items() if k not in ("text", "max_len")})
            p, keep = self.eng._params(u["text"], u["max_len"], **args)
            params[i] = p
            self._keep.append(keep)
        if lib().qtts_batch_begin(self.h, n, params) < 0:
            raise RuntimeError("batch begin failed: " + self.error())
        self.n = n

    def run(self, n_frames: int) -> int:
        rc = lib().qtts_batch_run(self.h, n_frames)
        if rc < 0:
            raise RuntimeError("batch run failed: " + self.error())
        return rc

    def codes(self):
        c = np.zeros((self.n, self.max_frames, self.ncb), np.int32)
        nf = np.zeros(self.n, np.int32)
        if not lib().qtts_batch_codes(self.h, _p(c, C.c_int32), _p(nf, C.c_int32)):
            raise RuntimeError("batch codes failed: " + self.error())
        return [c[i, :nf[i]].copy() for i in range(self.n)]

    def codes_device(self):
        """(device address of the codes [n][max_frames][n_codebooks] int32, frames
        per sequence): the batched codes -> vocoder handoff without a host copy."""
        ptr = C.c_void_p()
        nf = np.zeros(self.n, np.int32)
        if lib().qtts_batch_codes_device(self.h, C.byref(ptr), _p(nf, C.c_int32)) < 0:
            raise RuntimeError("batch codes_device failed: " + self.error())
        return int(ptr.value or 0), nf

    BATCH_CLASSES = ["pack", "gemm_qkv", "gemm_o", "gemm_gu", "gemm_down", "gemm_head", "attn_cp", "attn_talker",
                     "sample", "other"]

    def profile(self, n_frames: int) -> dict:
        ms = np.zeros(10, np.float32)
        la = np.zeros(10, np.int32)
        if not lib().qtts_batch_profile(self.h, n_frames, _p(ms, C.c_float), _p(la, C.c_int32)):
            raise RuntimeError("batch profile failed: " + self.error())
        return {c: {"ms_per_frame": float(ms[i]), "launches_per_frame": int(la[i])}
                for i, c in enumerate(self.BATCH_CLASSES)}

    def timing(self) -> dict:
        ms, fr, la = C.c_float(0), C.c_int32(0), C.c_int32(0)
        lib().qtts_batch_timing(self.h, C.byref(ms), C.byref(fr), C.byref(la))
        return {"frames_ms": ms.value, "seq_frames": fr.value, "launches_per_frame": la.value}

    def close(self):
        if getattr(self, "h", None):
            lib().qtts_batch_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


TC_ACT_F16, TC_ACT_SPLIT = 0, 1
TC_EPI_STORE, TC_EPI_RESID, TC_EPI_SWIGLU = 0, 1, 2


def op_gemm_tc(w, x, w_up=None, norm_gain=None, eps=1e-6, act=TC_ACT_F16, epi=TC_EPI_STORE, resid=None,
               device: int = 0):
    """Run the tcgen05 GEMM once: y [m][rows] (see qtts_op_gemm_tc)."""
    w = np.ascontiguousarray(w, dtype=np.float16)
    rows, cols = w.shape
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
    m = x.shape[0]
    wu = None if w_up is None else np.ascontiguousarray(w_up, dtype=np.float16)
    g = None if norm_gain is None else np.ascontiguousarray(norm_gain, dtype=np.float32)
    r = None if resid is None else np.ascontiguousarray(resid, dtype=np.float32)
    y = np.zeros((m, rows), np.float32)
    rc = lib().qtts_op_gemm_tc(device, w.ctypes.data_as(C.c_void_p), None if wu is None else wu.ctypes.data_as(C.c_void_p),
                               rows, cols, _p(x, C.c_float), m, _p(g, C.c_float), eps, act, epi, _p(r, C.c_float),
                               _p(y, C.c_float))
    if not rc:
        raise RuntimeError("qtts_op_gemm_tc failed")
    return y


def op_gemm_q8(w, cols, x, w_up=None, norm_gain=None, eps=1e-6, epi=TC_EPI_STORE, resid=None, ksplit=0,
               device: int = 0):
    """Run the kind::i8 tensor-core GEMM once (see qtts_op_gemm_q8): w (and w_up)
    are GGUF Q8_0 blocks (uint8, rows x cols/32 x 34 bytes).  Returns (y [m][rows],
    the k-split used)."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    rows = w.size // (cols // 32 * 34)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
    m = x.shape[0]
    wu = None if w_up is None else np.ascontiguousarray(w_up, dtype=np.uint8)
    g = None if norm_gain is None else np.ascontiguousarray(norm_gain, dtype=np.float32)
    r = None if resid is None else np.ascontiguousarray(resid, dtype=np.float32)
    y = np.zeros((m, rows), np.float32)
    s = lib().qtts_op_gemm_q8(device, w.ctypes.data_as(C.c_void_p), None if wu is None else wu.ctypes.data_as(C.c_void_p),
                              rows, cols, _p(x, C.c_float), m, _p(g, C.c_float), eps, epi, _p(r, C.c_float), ksplit,
                              _p(y, C.c_float))
    if not s:
        raise RuntimeError(lib().qtts_create_error().decode())
    return y, s


def op_sample(logits, cb: int, temperature=0.0, top_k=0, rep_penalty=1.0, presence=None, eos_bias=0.0,
              target_frames=0, frame=0, eos_id=2150, suppress_start=None, seed=0, device: int = 0) -> int:
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    V = lg.size
    pr = None if presence is None else np.ascontiguousarray(presence, dtype=np.int32)
    ss = V if suppress_start is None else suppress_start
    return lib().qtts_op_sample(device, _p(lg, C.c_float), V, cb, temperature, top_k, rep_penalty, _p(pr, C.c_int32),
                                eos_bias, target_frames, frame, eos_id, ss, seed)
