"""B200 engine for qwen3-tts.cpp's per-frame codec-token loop.

The product is libqwen3tts_b200.so (CUDA sm_100a kernels + C++ host code,
C ABI in include/qwen3tts_b200.h, C++ drop-in in include/tts_transformer.h).
This package holds its sources (csrc/), the in-tree build (build.py), a ctypes
binding (engine.py) and the seeded-GGUF writer used for synthetic models
(synth_gguf.py).  The directory name is not a Python identifier; load it with
importlib (see tests/conftest.py).
"""
from . import build, scheduler, synth_gguf  # noqa: F401
from .engine import Engine, exported_symbols, lib  # noqa: F401
