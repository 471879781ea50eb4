"""Shared builders for the GPU parity tests: one seeded host weight set feeds
both the device model and the CPU oracle."""
import functools

import numpy as np

from llm_inference_edu_b200 import presets, synthetic


def oracle_weights(o, cfg, w, linear_format):
    return o.int8_model_weights(cfg, w, linear_format)


@functools.lru_cache(maxsize=2)
def qwen_host_weights(name, seed, dtype):
    cfg = {"0.5b": presets.qwen_0_5b, "7b": presets.qwen_7b}[name]()
    return synthetic.weights(cfg, seed=seed, dtype=dtype)


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def safetensors_bytes(tensors):
    """A safetensors file: tensors {name: (dtype, shape, raw bytes)}, the
    header's JSON in sorted-name order with back-to-back data offsets,
    padded with spaces to a multiple of 8 bytes (as the format's writer
    does)."""
    import json
    import struct
    header, blobs, at = {}, [], 0
    for name in sorted(tensors):
        dtype, shape, raw = tensors[name]
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [at, at + len(raw)]}
        blobs.append(raw)
        at += len(raw)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    return struct.pack("<Q", len(h)) + h + b"".join(blobs)


def qwen2_tensor_shapes(cfg):
    """The checkpoint names and shapes of a HF config.json dictionary
    (the expected inventory of src/weights.rs:163-185)."""
    h, ff = cfg["hidden_size"], cfg["intermediate_size"]
    kv = cfg["num_key_value_heads"] * (h // cfg["num_attention_heads"])
    out = {"model.embed_tokens.weight": (cfg["vocab_size"], h), "model.norm.weight": (h,)}
    for l in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{l}."
        out.update({p + "input_layernorm.weight": (h,), p + "post_attention_layernorm.weight": (h,),
                    p + "self_attn.q_proj.weight": (h, h), p + "self_attn.q_proj.bias": (h,),
                    p + "self_attn.k_proj.weight": (kv, h), p + "self_attn.k_proj.bias": (kv,),
                    p + "self_attn.v_proj.weight": (kv, h), p + "self_attn.v_proj.bias": (kv,),
                    p + "self_attn.o_proj.weight": (h, h), p + "mlp.gate_proj.weight": (ff, h),
                    p + "mlp.up_proj.weight": (ff, h), p + "mlp.down_proj.weight": (h, ff)})
    return out
