"""Writes seeded synthetic checkpoints in the reference's on-disk formats.

TEST INFRASTRUCTURE ONLY (inputs for the product's loader).

* bf16: HF names, every tensor BF16 (what engine/src/lib.rs:164 accepts).
* MXFP4: the layout of python/quantize_mxfp4.py:52-119 -- file metadata
  {"format": "jalapenos-mxfp4-v1"}, 2-D tensors as ``<name>.mxfp4_packed`` /
  ``<name>.mxfp4_scales`` U8 pairs, 1-D norms as raw U16 bf16 bits, and a
  ``quantization_config`` block in config.json.  ``quantize_head=False`` keeps
  the embedding and lm_head as BF16 inside the quantized file, as the
  benchmark configurations ask.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

import oracle as O


def write_safetensors(path: Path, tensors: dict[str, tuple[str, tuple, bytes]],
                      metadata: dict | None = None) -> None:
    """tensors: name -> (dtype, shape, raw little-endian bytes)."""
    header = {}
    offset = 0
    blobs = []
    for name, (dtype, shape, raw) in tensors.items():
        header[name] = {"dtype": dtype, "shape": list(shape),
                        "data_offsets": [offset, offset + len(raw)]}
        offset += len(raw)
        blobs.append(raw)
    if metadata:
        header["__metadata__"] = metadata
    text = json.dumps(header, separators=(",", ":")).encode()
    text += b" " * ((8 - len(text) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for b in blobs:
            f.write(b)


def hf_config(cfg: O.Config, quantized: bool) -> dict:
    c = {
        "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3",
        "hidden_size": cfg.hidden, "intermediate_size": cfg.inter,
        "num_hidden_layers": cfg.layers, "num_attention_heads": cfg.q_heads,
        "num_key_value_heads": cfg.kv_heads, "head_dim": O.HEAD_DIM, "vocab_size": cfg.vocab,
        "max_position_embeddings": cfg.max_positions, "eos_token_id": cfg.eos,
        "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "tie_word_embeddings": cfg.tied,
        "torch_dtype": "bfloat16", "attention_bias": False,
    }
    if quantized:
        c["quantization_config"] = {"quant_method": "mxfp4", "format": "jalapenos-mxfp4-v1",
                                    "block_size": 32, "weights_only": True}
    return c


def write_model(model: O.Model, directory: Path, quantized: bool, shards: int = 2) -> Path:
    """Writes ``model``'s tensors (as the oracle holds them) to `directory`."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    cfg = model.cfg
    entries: list[tuple[str, object]] = [("model.embed_tokens.weight", model.tensors["embed"])]
    if model.tensors.get("lm_head") is not None:
        entries.append(("lm_head.weight", model.tensors["lm_head"]))
    entries.append(("model.norm.weight", model.tensors["norm"]))
    for layer in range(cfg.layers):
        for name in O.LAYER_TENSORS:
            entries.append((f"model.layers.{layer}.{O.HF_NAMES[name]}", model.tensors[f"{layer}.{name}"]))
    per = (len(entries) + shards - 1) // shards
    for s in range(shards):
        out = {}
        for name, t in entries[s * per:(s + 1) * per]:
            if isinstance(t, O.Matrix):
                if t.mxfp4:
                    out[name + ".mxfp4_packed"] = ("U8", (t.rows, t.cols // 2), t.packed.tobytes())
                    out[name + ".mxfp4_scales"] = ("U8", (t.rows, t.cols // 32), t.scales.tobytes())
                else:
                    out[name] = ("BF16", (t.rows, t.cols), t.bf16.astype("<u2").tobytes())
            else:
                dtype = "U16" if quantized else "BF16"
                out[name] = (dtype, tuple(t.shape), np.asarray(t, "<u2").tobytes())
        meta = {"format": "jalapenos-mxfp4-v1"} if quantized else {"format": "pt"}
        write_safetensors(directory / f"model-{s + 1:05d}-of-{shards:05d}.safetensors", out, meta)
    (directory / "config.json").write_text(json.dumps(hf_config(cfg, quantized), indent=2) + "\n")
    return directory
