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


# ----------------------------------------------------------- poll bridge ----

def tiny_model_json(weights=None, config=None) -> bytes:
    """The reference's tiny model file format (Decoder::from_json,
    src/model.rs:185; {"config", "weights"}) for the Tiny-R weights."""
    import json
    from llm_inference_edu_b200 import presets
    w = weights or presets.tiny_r_weights()
    c = config or presets.tiny_r(32)
    names = dict(attn_norm="attention_norm", q="query", k="key", v="value", o="attention_output",
                 ffn_norm="ffn_norm", gate="gate", up="up", down="down")
    doc = {
        "config": {"vocab_size": c.vocab_size, "layers": c.layers, "hidden_dim": c.hidden_dim,
                   "query_heads": c.query_heads, "kv_heads": c.kv_heads, "head_dim": c.head_dim,
                   "ff_dim": c.ff_dim, "max_tokens": c.max_tokens, "rope_base": c.rope_base,
                   "norm_epsilon": c.norm_epsilon},
        "weights": {"embedding": [float(x) for x in w["embedding"]],
                    "layers": [{names[k]: [float(x) for x in v] for k, v in l.items()} for l in w["layers"]],
                    "final_norm": [float(x) for x in w["final_norm"]]},
    }
    return json.dumps(doc).encode()


def bridge_event():
    from llm_inference_edu_b200._lib import AieEvent
    return AieEvent(99, 99, 99, 99, 99)


def ev_tuple(e):
    return (e.kind, e.code, e.token, e.processed, e.history)


def bridge_wait(h, seconds=20.0):
    """Polls until the worker's event arrives (src/tests.rs:14-28)."""
    import ctypes as C
    import time
    from llm_inference_edu_b200._lib import lib
    deadline = time.monotonic() + seconds
    while True:
        out = bridge_event()
        st = lib().aie_poll(h, C.byref(out))
        if st == 0:
            return out
        assert st == 1, st  # PENDING
        assert ev_tuple(out) == (99,) * 5
        assert time.monotonic() < deadline, "worker event timeout"
        time.sleep(0.001)


def bridge_open(source: bytes, kind: int = 0, seconds=20.0):
    """aie_open, retrying while a closed worker still releases its model."""
    import ctypes as C
    import time
    from llm_inference_edu_b200._lib import lib
    h = C.c_uint64(0)
    deadline = time.monotonic() + seconds
    while True:
        st = lib().aie_open(kind, source, len(source), C.byref(h))
        if st != 4:  # BUSY
            return st, h.value
        assert time.monotonic() < deadline, "worker never released"
        time.sleep(0.005)


def _bf16_bits(a):
    """FP32 values as BF16 bit patterns (round to nearest even; finite)."""
    import numpy as np
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return a
    f = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((f + 0x7fff + ((f >> 16) & 1)) >> 16).astype(np.uint16)


def small_qwen_checkpoint(seed=5, vocab=256):
    """A small Qwen2 checkpoint: (HF config.json dict, the matching
    ModelConfig, its BF16 weight dictionary, the safetensors bytes)."""
    from llm_inference_edu_b200 import presets, synthetic
    hf = {"architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2", "hidden_act": "silu",
          "vocab_size": vocab, "hidden_size": 64, "intermediate_size": 128, "num_hidden_layers": 2,
          "num_attention_heads": 4, "num_key_value_heads": 2, "max_position_embeddings": 64,
          "rms_norm_eps": 1e-6, "rope_theta": 10000.0, "tie_word_embeddings": True,
          "torch_dtype": "bfloat16", "use_sliding_window": False}
    cfg = presets.ModelConfig(vocab, 2, 64, 4, 2, 16, 128, 64, 10000.0, 1e-6, True, True)
    w = synthetic.weights(cfg, seed=seed, dtype="bf16", bias_std=0.02, norm_std=0.1)
    w = {"embedding": _bf16_bits(w["embedding"]), "final_norm": _bf16_bits(w["final_norm"]),
         "layers": [{k: _bf16_bits(v) for k, v in L.items()} for L in w["layers"]]}
    names = {"attn_norm": "input_layernorm.weight", "ffn_norm": "post_attention_layernorm.weight",
             "q": "self_attn.q_proj.weight", "q_bias": "self_attn.q_proj.bias", "k": "self_attn.k_proj.weight",
             "k_bias": "self_attn.k_proj.bias", "v": "self_attn.v_proj.weight", "v_bias": "self_attn.v_proj.bias",
             "o": "self_attn.o_proj.weight", "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight",
             "down": "mlp.down_proj.weight"}
    shapes = {"q": (64, 64), "k": (32, 64), "v": (32, 64), "o": (64, 64), "gate": (128, 64), "up": (128, 64),
              "down": (64, 128)}
    t = {"model.embed_tokens.weight": ("BF16", (vocab, 64), w["embedding"].astype("<u2").tobytes()),
         "model.norm.weight": ("BF16", (64,), w["final_norm"].astype("<u2").tobytes())}
    for l, L in enumerate(w["layers"]):
        for k, v in L.items():
            t[f"model.layers.{l}.{names[k]}"] = ("BF16", shapes.get(k, (v.size,)), v.astype("<u2").tobytes())
    data = safetensors_bytes(t)
    return hf, cfg, w, data


def chat_tokenizer_files(directory, **over):
    """tokenizer.json, tokenizer_config.json and generation_config.json of a
    chat tokenizer in `directory`: the synthetic golden tokenizer padded to
    151,643 vocabulary entries so that its three special tokens take Qwen's
    ids 151643-151645 (in the Qwen file they are added tokens past the
    vocabulary).  `over` replaces config fields ("cfg" / "gen" dicts)."""
    import json
    import os
    here = os.path.dirname(os.path.abspath(__file__))
    doc = json.loads(open(os.path.join(here, "golden", "tokenizer-synthetic.json"), encoding="utf-8").read())
    vocab = doc["model"]["vocab"]
    order = {"<|endoftext|>": 0, "<|im_start|>": 1, "<|im_end|>": 2}
    for a in doc["added_tokens"]:
        vocab.pop(a["content"], None)
    doc["added_tokens"] = sorted(doc["added_tokens"], key=lambda a: order[a["content"]])
    for k in range(len(vocab), 151643):
        vocab[f"<pad{k}>"] = k
    cfg = {"tokenizer_class": "Qwen2Tokenizer", "add_bos_token": False, "bos_token": None,
           "eos_token": "<|im_end|>"}
    gen = {"eos_token_id": [151645, 151643]}
    cfg.update(over.get("cfg", {}))
    gen.update(over.get("gen", {}))
    for name, obj in (("tokenizer.json", doc), ("tokenizer_config.json", cfg), ("generation_config.json", gen)):
        with open(os.path.join(str(directory), name), "w") as f:
            json.dump(obj, f)
    return directory
