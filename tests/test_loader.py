"""CPU checks of checkpoint loading (qb_qwen_tensor_count,
qb_safetensors_inspect, qb_model_load_safetensors up to its device work),
restating the reference's tests/weights.rs cases on the same tiny config."""
import numpy as np
import pytest

from helpers import qwen2_tensor_shapes, safetensors_bytes


def config(**mods):
    # tests/weights.rs:8-10
    c = {"architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2", "hidden_act": "silu",
         "vocab_size": 4, "hidden_size": 4, "intermediate_size": 6, "num_hidden_layers": 1,
         "num_attention_heads": 2, "num_key_value_heads": 1, "max_position_embeddings": 32,
         "rms_norm_eps": 0.000001, "rope_theta": 1000000, "tie_word_embeddings": True,
         "torch_dtype": "bfloat16", "use_sliding_window": False}
    c.update(mods)
    return c


def contents(c, dtype="BF16"):
    # tests/weights.rs:16-32: every tensor cycles 1, -2, 0.5
    out = {}
    for name, shape in qwen2_tensor_shapes(c).items():
        n = int(np.prod(shape))
        v = np.array([1.0, -2.0, 0.5], np.float32)[np.arange(n) % 3]
        raw = (v.view(np.uint32) >> 16).astype("<u2").tobytes() if dtype == "BF16" else v.astype("<f4").tobytes()
        out[name] = (dtype, shape, raw)
    return out


def kind(fn):
    from llm_inference_edu_b200 import LoadError
    with pytest.raises(LoadError) as e:
        fn()
    return e.value.kind


def test_inventory_of_the_tied_checkpoint():
    # tests/weights.rs:48-62 (the BF16 values themselves are checked on the
    # device, tests/test_gpu_loader.py)
    from llm_inference_edu_b200 import inspect_safetensors, qwen_tensor_count
    c = config()
    assert qwen_tensor_count(c) == 14
    assert inspect_safetensors(safetensors_bytes(contents(c)), c) == 14


def test_missing_extra_wrong_shape_and_wrong_dtype_are_rejected():
    # tests/weights.rs:64-96
    from llm_inference_edu_b200 import inspect_safetensors
    c = config()
    t = contents(c)
    del t["model.norm.weight"]
    assert kind(lambda: inspect_safetensors(safetensors_bytes(t), c)) == "MissingTensor"
    t = contents(c)
    t["lm_head.weight"] = t["model.embed_tokens.weight"]
    assert kind(lambda: inspect_safetensors(safetensors_bytes(t), c)) == "UnexpectedTensor"
    t = contents(c)
    d, _, raw = t["model.layers.0.self_attn.q_proj.weight"]
    t["model.layers.0.self_attn.q_proj.weight"] = (d, (2, 8), raw)
    assert kind(lambda: inspect_safetensors(safetensors_bytes(t), c)) == "InvalidShape"
    assert kind(lambda: inspect_safetensors(safetensors_bytes(contents(c, "F32")), c)) == "InvalidDtype"


def test_parser_bounds_nonfinite_data_and_dimension_overflow_are_rejected():
    # tests/weights.rs:98-150
    from llm_inference_edu_b200 import Decoder, inspect_safetensors, qwen_tensor_count
    c = config()
    f = safetensors_bytes(contents(c))
    assert kind(lambda: inspect_safetensors(f[:-1], c)) == "Format"
    assert kind(lambda: inspect_safetensors(f + b"\0", c)) == "Format"
    t = contents(c)
    d, s, raw = t["model.norm.weight"]
    t["model.norm.weight"] = (d, s, np.array([0x7fc0], "<u2").tobytes() + raw[2:])
    # rejected before any device work, so this needs no GPU
    assert kind(lambda: Decoder.from_safetensors(safetensors_bytes(t), c)) == "NonFinite"
    huge = 2 ** 64 - 1
    assert kind(lambda: qwen_tensor_count(config(vocab_size=huge))) == "DimensionOverflow"
    assert kind(lambda: qwen_tensor_count(config(num_hidden_layers=huge))) == "DimensionOverflow"
    assert kind(lambda: qwen_tensor_count(config(vocab_size=1 << 30))) == "ResourceBudget"
    assert kind(lambda: qwen_tensor_count(config(num_attention_heads=3))) == "UnsupportedConfig"
    assert kind(lambda: qwen_tensor_count(config(tie_word_embeddings=False))) == "UnsupportedConfig"


def test_format_edges():
    # header bounds and offsets of the file format itself
    from llm_inference_edu_b200 import inspect_safetensors
    import struct
    c = config()
    f = safetensors_bytes(contents(c))
    n = struct.unpack("<Q", f[:8])[0]
    assert kind(lambda: inspect_safetensors(f[:7], c)) == "Format"                      # no length
    assert kind(lambda: inspect_safetensors(struct.pack("<Q", len(f)) + f[8:], c)) == "Format"  # past the end
    assert kind(lambda: inspect_safetensors(f[:8] + b" " + f[9:], c)) == "Format"       # must start with '{'
    bad = f[:8] + f[8:8 + n].replace(b'"data_offsets":[0,', b'"data_offsets":[2,', 1) + f[8 + n:]
    assert kind(lambda: inspect_safetensors(bad, c)) == "Format"                        # gap before the first
    meta = safetensors_bytes(contents(c))
    h = meta[8:8 + n].rstrip(b" ")
    h = b'{"__metadata__":{"format":"pt"},' + h[1:]
    h += b" " * (-len(h) % 8)
    assert inspect_safetensors(struct.pack("<Q", len(h)) + h + meta[8 + n:], c) == 14  # metadata skipped
