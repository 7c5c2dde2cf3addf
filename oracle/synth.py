"""Seeded synthetic Qwen3-TTS checkpoints (config.json + model.safetensors).

TEST INFRASTRUCTURE. This module writes random-init model directories with the
shapes of the Qwen3-TTS 12 Hz CustomVoice talker + CodePredictor, in the file
layout the reference runtime loads:

* ``config.json`` holds exactly the fields the reference deserialises in
  ``src/model/config.rs:105-150`` (``RawConfig`` / ``RawTalkerConfig`` /
  ``RawTransformerConfig``).
* ``model.safetensors`` holds every tensor the reference reads, under the same
  names: decoder layers (``src/model/decode.rs:2107-2150``), talker head, norm
  and codec embedding (``src/model/talker.rs:96-104``), CodePredictor heads,
  embeddings and optional ``small_to_mtp_projection``
  (``src/model/code_predictor.rs:182-238``), text embedding and text projection
  MLP (``src/model/text.rs:275-301``).

Weights are drawn once from ``numpy.random.default_rng(seed)`` in sorted tensor
name order, N(0, 0.02) for matrices and biases, rounded to bf16
(round-to-nearest-even); RMSNorm gammas are exactly 1.  The same seed gives
the same bytes on every machine, so the GPU box regenerates identical weights
instead of shipping checkpoints.

Nothing in the product path imports this file; tests, ``bench.py`` and
``__graft_entry__.smoke()`` use it to make inputs.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field, asdict
from pathlib import Path

import numpy as np

# Language / speaker codec ids used by the reference's public enums
# (src/model/text.rs:44-56, 108-120); the synthetic config maps the same names.
LANGUAGE_IDS = {
    "chinese": 2055, "english": 2050, "japanese": 2058, "korean": 2064,
    "german": 2053, "french": 2061, "russian": 2069, "portuguese": 2071,
    "spanish": 2054, "italian": 2070,
}
SPEAKER_IDS = {
    "serena": 3066, "vivian": 3065, "uncle_fu": 3010, "ryan": 3061,
    "aiden": 2861, "ono_anna": 2873, "sohee": 2864, "eric": 2875, "dylan": 2878,
}


@dataclass
class Shape:
    """Dimensions of one synthetic checkpoint."""

    name: str
    hidden: int
    intermediate: int
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    cp_hidden: int
    cp_intermediate: int
    cp_layers: int
    cp_vocab: int
    num_code_groups: int
    text_vocab: int
    text_hidden: int
    text_proj_intermediate: int
    rms_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    # special text ids (must be < text_vocab)
    im_start: int = 151644
    assistant: int = 77091
    tts_pad: int = 151671
    tts_bos: int = 151672
    tts_eos: int = 151673
    # special codec ids (in the suppressed band [vocab-1024, vocab))
    codec_pad: int = 2148
    codec_bos: int = 2149
    codec_eos: int = 2150
    codec_think: int = 2154
    codec_think_bos: int = 2156
    codec_think_eos: int = 2157


SHAPES = {
    # BASELINE configs 0/1/3: Qwen3-TTS-0.6B-shaped talker and CodePredictor.
    "0.6b": Shape("0.6b", hidden=1024, intermediate=3072, layers=28, q_heads=16, kv_heads=8,
                  head_dim=128, vocab=3072, cp_hidden=1024, cp_intermediate=3072, cp_layers=5,
                  cp_vocab=2048, num_code_groups=16, text_vocab=151936, text_hidden=2048,
                  text_proj_intermediate=2048),
    # BASELINE configs 2/4: 1.7B-shaped talker; CodePredictor behind a 2048->1024 projection.
    "1.7b": Shape("1.7b", hidden=2048, intermediate=6144, layers=28, q_heads=16, kv_heads=8,
                  head_dim=128, vocab=3072, cp_hidden=1024, cp_intermediate=3072, cp_layers=5,
                  cp_vocab=2048, num_code_groups=16, text_vocab=151936, text_hidden=2048,
                  text_proj_intermediate=2048),
    # Small shapes for CPU-speed parity tests (same code paths, fewer/smaller layers).
    "tiny": Shape("tiny", hidden=256, intermediate=512, layers=2, q_heads=4, kv_heads=2,
                  head_dim=128, vocab=3072, cp_hidden=256, cp_intermediate=512, cp_layers=2,
                  cp_vocab=2048, num_code_groups=16, text_vocab=4096, text_hidden=256,
                  text_proj_intermediate=256, im_start=4000, assistant=4001, tts_pad=4002,
                  tts_bos=4003, tts_eos=4004),
    "tiny_proj": Shape("tiny_proj", hidden=512, intermediate=1024, layers=2, q_heads=4, kv_heads=2,
                       head_dim=128, vocab=3072, cp_hidden=256, cp_intermediate=512, cp_layers=2,
                       cp_vocab=2048, num_code_groups=16, text_vocab=4096, text_hidden=2048,
                       text_proj_intermediate=512, im_start=4000, assistant=4001, tts_pad=4002,
                       tts_bos=4003, tts_eos=4004),
    # One talker layer whose decode-step activations (input row, QKV, attention
    # output, post-attention row and 66,560-wide MLP row) exceed 264 KiB: the
    # allocation-free step must refuse it.
    "tiny_wide": Shape("tiny_wide", hidden=256, intermediate=66560, layers=1, q_heads=4,
                       kv_heads=2, head_dim=128, vocab=3072, cp_hidden=256, cp_intermediate=512,
                       cp_layers=1, cp_vocab=2048, num_code_groups=16, text_vocab=4096,
                       text_hidden=256, text_proj_intermediate=256, im_start=4000,
                       assistant=4001, tts_pad=4002, tts_bos=4003, tts_eos=4004),
}


def config_json(s: Shape) -> dict:
    """config.json fields consumed by the reference (src/model/config.rs:105-150)."""
    cp = {
        "head_dim": s.head_dim, "hidden_size": s.cp_hidden,
        "intermediate_size": s.cp_intermediate, "num_attention_heads": s.q_heads,
        "num_code_groups": s.num_code_groups, "num_hidden_layers": s.cp_layers,
        "num_key_value_heads": s.kv_heads, "rms_norm_eps": s.rms_eps,
        "rope_theta": s.rope_theta, "vocab_size": s.cp_vocab,
    }
    talker = {
        "code_predictor_config": cp,
        "codec_bos_id": s.codec_bos, "codec_eos_token_id": s.codec_eos,
        "codec_language_id": dict(LANGUAGE_IDS), "codec_pad_id": s.codec_pad,
        "codec_think_id": s.codec_think, "codec_think_bos_id": s.codec_think_bos,
        "codec_think_eos_id": s.codec_think_eos, "spk_id": dict(SPEAKER_IDS),
        "head_dim": s.head_dim, "hidden_size": s.hidden,
        "intermediate_size": s.intermediate, "num_attention_heads": s.q_heads,
        "num_code_groups": s.num_code_groups, "num_hidden_layers": s.layers,
        "num_key_value_heads": s.kv_heads, "rms_norm_eps": s.rms_eps,
        "rope_theta": s.rope_theta, "vocab_size": s.vocab,
        "text_hidden_size": s.text_hidden, "text_vocab_size": s.text_vocab,
    }
    return {
        "assistant_token_id": s.assistant, "im_start_token_id": s.im_start,
        "tts_bos_token_id": s.tts_bos, "tts_eos_token_id": s.tts_eos,
        "tts_pad_token_id": s.tts_pad, "talker_config": talker,
        "synthetic": {"shape": s.name},
    }


def tensor_shapes(s: Shape) -> dict[str, tuple[int, ...]]:
    """Every tensor name and [out, in] shape the reference reads."""
    out: dict[str, tuple[int, ...]] = {}

    def layers(prefix: str, n: int, h: int, inter: int) -> None:
        q_out, kv_out = s.q_heads * s.head_dim, s.kv_heads * s.head_dim
        for i in range(n):
            p = f"{prefix}.{i}"
            out[f"{p}.input_layernorm.weight"] = (h,)
            out[f"{p}.self_attn.q_proj.weight"] = (q_out, h)
            out[f"{p}.self_attn.k_proj.weight"] = (kv_out, h)
            out[f"{p}.self_attn.v_proj.weight"] = (kv_out, h)
            out[f"{p}.self_attn.o_proj.weight"] = (h, q_out)
            out[f"{p}.self_attn.q_norm.weight"] = (s.head_dim,)
            out[f"{p}.self_attn.k_norm.weight"] = (s.head_dim,)
            out[f"{p}.post_attention_layernorm.weight"] = (h,)
            out[f"{p}.mlp.gate_proj.weight"] = (inter, h)
            out[f"{p}.mlp.up_proj.weight"] = (inter, h)
            out[f"{p}.mlp.down_proj.weight"] = (h, inter)

    layers("talker.model.layers", s.layers, s.hidden, s.intermediate)
    out["talker.model.norm.weight"] = (s.hidden,)
    out["talker.codec_head.weight"] = (s.vocab, s.hidden)
    out["talker.model.codec_embedding.weight"] = (s.vocab, s.hidden)
    out["talker.model.text_embedding.weight"] = (s.text_vocab, s.text_hidden)
    out["talker.text_projection.linear_fc1.weight"] = (s.text_proj_intermediate, s.text_hidden)
    out["talker.text_projection.linear_fc1.bias"] = (s.text_proj_intermediate,)
    out["talker.text_projection.linear_fc2.weight"] = (s.hidden, s.text_proj_intermediate)
    out["talker.text_projection.linear_fc2.bias"] = (s.hidden,)
    cp = "talker.code_predictor"
    layers(f"{cp}.model.layers", s.cp_layers, s.cp_hidden, s.cp_intermediate)
    out[f"{cp}.model.norm.weight"] = (s.cp_hidden,)
    for g in range(s.num_code_groups - 1):
        out[f"{cp}.lm_head.{g}.weight"] = (s.cp_vocab, s.cp_hidden)
        out[f"{cp}.model.codec_embedding.{g}.weight"] = (s.cp_vocab, s.hidden)
    if s.cp_hidden != s.hidden:
        out[f"{cp}.small_to_mtp_projection.weight"] = (s.cp_hidden, s.hidden)
        out[f"{cp}.small_to_mtp_projection.bias"] = (s.cp_hidden,)
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest, ties to even); returns uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = u + (np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1)))
    return (rounded >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def generate(s: Shape, seed: int = 0) -> dict[str, np.ndarray]:
    """All tensors as bf16 bit patterns (uint16), drawn in sorted-name order."""
    rng = np.random.default_rng(seed)
    tensors: dict[str, np.ndarray] = {}
    for name in sorted(tensor_shapes(s)):
        shape = tensor_shapes(s)[name]
        if name.endswith("norm.weight") or name.endswith("layernorm.weight"):
            tensors[name] = f32_to_bf16_bits(np.ones(shape, dtype=np.float32))
        else:
            vals = rng.standard_normal(size=shape, dtype=np.float32)
            vals *= np.float32(0.02)
            tensors[name] = f32_to_bf16_bits(vals)
    return tensors


def write_safetensors(path: Path, tensors: dict[str, np.ndarray]) -> None:
    """Minimal safetensors writer (8-byte LE header length, JSON header, data)."""
    header: dict = {"__metadata__": {"format": "pt"}}
    offset = 0
    order = sorted(tensors)
    for name in order:
        arr = tensors[name]
        nbytes = arr.size * 2
        header[name] = {"dtype": "BF16", "shape": list(arr.shape),
                        "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
    hjson = json.dumps(header, separators=(",", ":")).encode()
    pad = (8 - len(hjson) % 8) % 8
    hjson += b" " * pad
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hjson)))
        f.write(hjson)
        for name in order:
            f.write(np.ascontiguousarray(tensors[name]).tobytes())


def read_safetensors(path: Path) -> dict[str, np.ndarray]:
    """Reads BF16 / F32 tensors; BF16 is returned as float32 values."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
        base = 8 + n
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        b, e = meta["data_offsets"]
        raw = mm[base + b: base + e]
        if meta["dtype"] == "BF16":
            out[name] = bf16_bits_to_f32(raw.view(np.uint16)).reshape(meta["shape"])
        elif meta["dtype"] == "F32":
            out[name] = np.array(raw.view(np.float32)).reshape(meta["shape"])
        else:
            raise ValueError(f"unsupported dtype {meta['dtype']} for {name}")
    return out


def write_model(out_dir: str | os.PathLike, shape: str = "tiny", seed: int = 0) -> Path:
    """Writes config.json + model.safetensors; skips work when already present."""
    s = SHAPES[shape]
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    stamp = out / ".synth.json"
    want = {"shape": shape, "seed": seed, "version": 1}
    if stamp.exists() and (out / "model.safetensors").exists():
        try:
            if json.loads(stamp.read_text()) == want:
                return out
        except json.JSONDecodeError:
            pass
    (out / "config.json").write_text(json.dumps(config_json(s), indent=1))
    write_safetensors(out / "model.safetensors", generate(s, seed))
    stamp.write_text(json.dumps(want))
    return out


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("out_dir")
    ap.add_argument("--shape", default="tiny", choices=sorted(SHAPES))
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    print(write_model(a.out_dir, a.shape, a.seed))
