"""Hugging Face model directories for the checkpoint-ingest tests (test
helper): config.json, safetensors shards and model.safetensors.index.json,
written in the published safetensors layout (u64 little-endian header
length, JSON header of name -> {dtype, shape, data_offsets}, then the data).

The tiny model's tensors are workloads.model_tensors(TINY, seed=0): matrices
are stored as BF16 (their values are bf16 numbers, so the bits are exact),
RMSNorm weights as F32.  With fp8 the projection, FFN and expert matrices
are the block-scaled e4m3 codes of tests/fp8_tiny.py plus their F32
"weight_scale_inv" tensors, as a DeepSeek-V3 checkpoint stores them."""

from __future__ import annotations

import functools
import json
import os
import struct

import numpy as np

from deepseek_cpp_infer_b200.workloads import TINY, model_tensors

MTP_LAYER = TINY["num_hidden_layers"]  # a layer past the model: DeepSeek-V3's multi-token-prediction module


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (round to nearest even)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def write_safetensors(path: str, tensors: list[tuple[str, str, np.ndarray]], metadata: dict | None = None):
    header, blobs, off = {}, [], 0
    for name, dt, a in tensors:
        b = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata is not None:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def hf_config(cfg: dict, fp8: bool = False) -> dict:
    """A model-dict (ModelConfig field names) as config.json."""
    c = {k: v for k, v in cfg.items() if k not in ("scoring_func", "weights_fp8", "q_lora_rank", "norm_topk_prob")}
    c["model_type"] = "deepseek_v3" if cfg.get("scoring_func", 0) == 1 else "deepseek_v2"
    c["scoring_func"] = "sigmoid" if cfg.get("scoring_func", 0) == 1 else "softmax"
    c["topk_method"] = "noaux_tc" if cfg.get("scoring_func", 0) == 1 else "greedy"
    c["q_lora_rank"] = cfg["q_lora_rank"] or None
    c["norm_topk_prob"] = bool(cfg.get("norm_topk_prob", 0))
    c["num_key_value_heads"] = cfg["num_attention_heads"]
    c["moe_layer_freq"] = 1
    if fp8:
        c["quantization_config"] = {"activation_scheme": "dynamic", "fmt": "e4m3", "quant_method": "fp8",
                                    "weight_block_size": [128, 128]}
    return c


def write_model_dir(path: str, config: dict, tensors: list[tuple[str, str, np.ndarray]], n_shards: int = 2):
    """config.json plus the tensors in n_shards contiguous shards and an index
    (n_shards = 0: one model.safetensors without an index)."""
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(config, f, indent=2)
    if n_shards == 0:
        write_safetensors(os.path.join(path, "model.safetensors"), tensors, {"format": "pt"})
        return
    per = -(-len(tensors) // n_shards)
    weight_map, total = {}, 0
    for s in range(n_shards):
        part = tensors[s * per:(s + 1) * per]
        fname = f"model-{s + 1:05d}-of-{n_shards:05d}.safetensors"
        write_safetensors(os.path.join(path, fname), part, {"format": "pt"})
        for name, _, a in part:
            weight_map[name] = fname
            total += a.nbytes
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=2)


@functools.lru_cache(maxsize=2)
def _model_entries(fp8: bool) -> tuple:
    out = []
    for name, a in model_tensors(TINY, seed=0).items():
        if fp8:
            from fp8_tiny import FP8_SUFFIXES, quantise

            if name.startswith("model.layers.") and name.endswith(FP8_SUFFIXES) and "mlp.gate." not in name:
                q, s, _ = quantise(a)
                out += [(name, "F8_E4M3", q), (name + "_scale_inv", "F32", s)]
                continue
        out.append((name, "F32", a) if a.ndim == 1 else (name, "BF16", bf16_bits(a)))
    return tuple(out)


def tiny_tensors(fp8: bool = False, extras: bool = True) -> list[tuple[str, str, np.ndarray]]:
    """The tiny model as (name, safetensors dtype, array), plus (extras) the
    tensors a real checkpoint carries that decoding does not use: a
    multi-token-prediction layer past num_hidden_layers and a rotary
    inv_freq buffer.  The arrays are cached: callers must not modify them."""
    out = list(_model_entries(fp8))
    if extras:
        D, P = TINY["hidden_size"], TINY["qk_rope_head_dim"]
        rng = np.random.default_rng(7)
        out += [
            (f"model.layers.{MTP_LAYER}.enorm.weight", "F32", np.ones(D, np.float32)),
            (f"model.layers.{MTP_LAYER}.eh_proj.weight", "BF16", bf16_bits(rng.standard_normal((D, 2 * D), np.float32))),
            ("model.layers.0.self_attn.rotary_emb.inv_freq", "F32",
             (10000.0 ** (-np.arange(0, P, 2, dtype=np.float32) / P)).astype(np.float32)),
        ]
    return sorted(out, key=lambda t: t[0])


N_EXTRAS = 3
