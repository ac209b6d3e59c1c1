"""Seeded random-init GGUF writer for the Qwen3-TTS talker + code predictor.

Writes a GGUF with the tensor names, shapes and metadata keys that the
reference converter emits (scripts/convert_tts_to_gguf.py:45-112 for the
names, :249-292 for the dtype policy, :421-479 for the metadata) and that
the reference loader reads (src/tts_transformer.cpp:228-377 for the keys,
:379-668 for the names and shapes).  The values are synthetic:

* every 2-D matrix and every bias ~ N(0, std) with std = 0.02 by default;
* every RMSNorm gain (``*_norm.weight``) = 1.0;
* 2-D tensors are F16, or Q8_0 for exactly the tensors the reference
  quantizes (``_should_quantize``: layer matrices and the text projection;
  embeddings, norms, biases and heads stay F16), 1-D tensors are F32.

Q8_0 blocks are produced by ``gguf.quants.quantize`` (gguf-py 0.19.0, the
package the reference converter imports), so the bytes are those of the
reference tooling.  The speaker encoder and tokenizer sections are not
written: the decode path never reads them (src/tts_transformer.cpp:408-410).

Usage:  python synth_gguf.py OUT.gguf [--type f16|q8_0] [--seed N] [--tiny]
"""
from __future__ import annotations

import argparse
import dataclasses
import os
import sys

import numpy as np


@dataclasses.dataclass
class SynthConfig:
    hidden: int = 1024
    n_layers: int = 28
    n_heads: int = 16
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 3072
    codec_vocab: int = 3072
    n_codebooks: int = 16
    cp_layers: int = 5
    cp_vocab: int = 2048
    cp_ffn: int = 3072
    text_vocab: int = 151936
    text_embd_dim: int = 2048
    rope_theta: float = 1000000.0
    cp_rope_theta: float = 1000000.0
    eps: float = 1e-6
    std: float = 0.02


# Layout of BASELINE.json configs: the 0.6B talker + code predictor.
FULL = SynthConfig()
# A small model with the same structure (head_dim 128, the special ids, the
# codec/code-predictor vocabularies) for fast CPU tests.
TINY = SynthConfig(hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn=768,
                   cp_layers=2, cp_ffn=512, text_embd_dim=256)


def _should_quantize(name: str) -> bool:
    # scripts/convert_tts_to_gguf.py:249-275
    if "_embd" in name or "codebook" in name:
        return False
    if "_norm" in name:
        return False
    if ".bias" in name:
        return False
    if "lm_head" in name or "codec_head" in name:
        return False
    return True


def tensor_specs(c: SynthConfig):
    """(name, numpy shape (rows, cols) or (n,)) in file order."""
    H, D = c.hidden, c.head_dim
    out = [
        ("talker.text_embd.weight", (c.text_vocab, c.text_embd_dim)),
        ("talker.text_proj.fc1.weight", (c.text_embd_dim, c.text_embd_dim)),
        ("talker.text_proj.fc1.bias", (c.text_embd_dim,)),
        ("talker.text_proj.fc2.weight", (H, c.text_embd_dim)),
        ("talker.text_proj.fc2.bias", (H,)),
        ("talker.codec_embd.weight", (c.codec_vocab, H)),
    ]

    def block(prefix, ffn):
        return [
            (prefix + "attn_norm.weight", (H,)),
            (prefix + "attn_q.weight", (c.n_heads * D, H)),
            (prefix + "attn_k.weight", (c.n_kv_heads * D, H)),
            (prefix + "attn_v.weight", (c.n_kv_heads * D, H)),
            (prefix + "attn_q_norm.weight", (D,)),
            (prefix + "attn_k_norm.weight", (D,)),
            (prefix + "attn_output.weight", (H, c.n_heads * D)),
            (prefix + "ffn_norm.weight", (H,)),
            (prefix + "ffn_gate.weight", (ffn, H)),
            (prefix + "ffn_up.weight", (ffn, H)),
            (prefix + "ffn_down.weight", (H, ffn)),
        ]

    for il in range(c.n_layers):
        out += block(f"talker.blk.{il}.", c.ffn)
    out += [("talker.output_norm.weight", (H,)),
            ("talker.codec_head.weight", (c.codec_vocab, H))]
    for il in range(c.cp_layers):
        out += block(f"code_pred.blk.{il}.", c.cp_ffn)
    out += [("code_pred.output_norm.weight", (H,))]
    for g in range(c.n_codebooks - 1):
        out += [(f"code_pred.codec_embd.{g}.weight", (c.cp_vocab, H))]
    for g in range(c.n_codebooks - 1):
        out += [(f"code_pred.lm_head.{g}.weight", (c.cp_vocab, H))]
    return out


def write_gguf(path: str, c: SynthConfig = FULL, wtype: str = "f16", seed: int = 0) -> str:
    import gguf

    arch = "qwen3-tts"
    w = gguf.GGUFWriter(path=None, arch=arch)
    w.add_name("Qwen3-TTS-12Hz-0.6B-synthetic")
    w.add_type(gguf.GGUFType.MODEL)
    w.add_file_type(gguf.LlamaFileType.MOSTLY_Q8_0 if wtype == "q8_0" else gguf.LlamaFileType.MOSTLY_F16)
    w.add_quantization_version(gguf.GGML_QUANT_VERSION)
    # Keys as the reference converter writes them (convert_tts_to_gguf.py:421-479).
    w.add_block_count(c.n_layers)
    w.add_embedding_length(c.hidden)
    w.add_feed_forward_length(c.ffn)
    w.add_head_count(c.n_heads)
    w.add_head_count_kv(c.n_kv_heads)
    w.add_key_length(c.head_dim)
    w.add_value_length(c.head_dim)
    w.add_rope_freq_base(c.rope_theta)
    w.add_layer_norm_rms_eps(c.eps)
    w.add_vocab_size(c.codec_vocab)
    w.add_uint32(f"{arch}.text_vocab_size", c.text_vocab)
    w.add_uint32(f"{arch}.text_hidden_size", c.text_embd_dim)
    w.add_uint32(f"{arch}.num_code_groups", c.n_codebooks)
    w.add_array(f"{arch}.rope.mrope_section", [24, 20, 20])
    w.add_uint32(f"{arch}.code_predictor.layer_count", c.cp_layers)
    w.add_uint32(f"{arch}.code_predictor.vocab_size", c.cp_vocab)
    w.add_uint32(f"{arch}.code_predictor.embedding_length", c.hidden)
    w.add_uint32(f"{arch}.code_predictor.feed_forward_length", c.cp_ffn)
    # Written explicitly: the header default (1e4) differs from the loader's
    # fallback (the talker theta), src/tts_transformer.h:86 vs .cpp:316-324.
    w.add_float32(f"{arch}.code_predictor.rope.freq_base", c.cp_rope_theta)
    w.add_uint32(f"{arch}.codec.pad_id", 2148)
    w.add_uint32(f"{arch}.codec.bos_id", 2149)
    w.add_uint32(f"{arch}.codec.eos_id", 2150)

    rng = np.random.default_rng(seed)
    for name, shape in tensor_specs(c):
        if name.endswith("_norm.weight"):
            data = np.ones(shape, dtype=np.float32)
        else:
            data = rng.standard_normal(shape, dtype=np.float32)
            data *= np.float32(c.std)
        if len(shape) == 1:
            w.add_tensor(name, data.astype(np.float32), raw_dtype=gguf.GGMLQuantizationType.F32)
        elif wtype == "q8_0" and _should_quantize(name):
            q = gguf.quants.quantize(data, gguf.GGMLQuantizationType.Q8_0)
            w.add_tensor(name, q, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        else:
            w.add_tensor(name, data.astype(np.float16), raw_dtype=gguf.GGMLQuantizationType.F16)
        del data

    tmp = path + ".tmp"
    w.write_header_to_file(path=tmp)
    w.write_kv_data_to_file()
    w.write_tensors_to_file(progress=False)
    w.close()
    os.replace(tmp, path)
    return path


def ensure_gguf(directory: str, c: SynthConfig = FULL, wtype: str = "f16", seed: int = 0,
                tag: str | None = None) -> str:
    """Return the path of a cached seeded GGUF in `directory`, writing it once."""
    os.makedirs(directory, exist_ok=True)
    if tag is None:
        tag = "full" if c == FULL else ("tiny" if c == TINY else "custom")
    path = os.path.join(directory, f"synth-{tag}-{wtype}-s{seed}.gguf")
    if not os.path.exists(path):
        write_gguf(path, c, wtype, seed)
    return path


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("out")
    ap.add_argument("--type", choices=["f16", "q8_0"], default="f16")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--tiny", action="store_true")
    a = ap.parse_args(argv)
    write_gguf(a.out, TINY if a.tiny else FULL, a.type, a.seed)


if __name__ == "__main__":
    sys.exit(main())
