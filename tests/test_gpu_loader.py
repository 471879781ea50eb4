"""A checkpoint loaded from safetensors (qb_model_load_safetensors) decodes
exactly like the same BF16 weights set tensor by tensor: the BF16 -> FP32
expansion is exact and every tensor lands in its place (tests/weights.rs:48-62
checks the expansion on the host)."""
import numpy as np
import pytest

from helpers import safetensors_bytes

pytestmark = pytest.mark.gpu


def _bf16(a):
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return a
    f = np.ascontiguousarray(a, np.float32).view(np.uint32)
    # round to nearest even (the values here are finite)
    return ((f + 0x7fff + ((f >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("linear_format", ["f32", "int8"])
def test_safetensors_model_decodes_like_the_dictionary_model(linear_format):
    import llm_inference_edu_b200 as qb
    from llm_inference_edu_b200 import presets, synthetic
    hf = {"architectures": ["Qwen2ForCausalLM"], "model_type": "qwen2", "hidden_act": "silu",
          "vocab_size": 256, "hidden_size": 64, "intermediate_size": 128, "num_hidden_layers": 2,
          "num_attention_heads": 4, "num_key_value_heads": 2, "max_position_embeddings": 64,
          "rms_norm_eps": 1e-6, "rope_theta": 10000.0, "tie_word_embeddings": True,
          "torch_dtype": "bfloat16", "use_sliding_window": False}
    cfg = presets.ModelConfig(256, 2, 64, 4, 2, 16, 128, 64, 10000.0, 1e-6, True, True)
    w = synthetic.weights(cfg, seed=5, dtype="bf16", bias_std=0.02, norm_std=0.1)
    w = {"embedding": _bf16(w["embedding"]), "final_norm": _bf16(w["final_norm"]),
         "layers": [{k: _bf16(v) for k, v in L.items()} for L in w["layers"]]}
    names = {"attn_norm": "input_layernorm.weight", "ffn_norm": "post_attention_layernorm.weight",
             "q": "self_attn.q_proj.weight", "q_bias": "self_attn.q_proj.bias", "k": "self_attn.k_proj.weight",
             "k_bias": "self_attn.k_proj.bias", "v": "self_attn.v_proj.weight", "v_bias": "self_attn.v_proj.bias",
             "o": "self_attn.o_proj.weight", "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight",
             "down": "mlp.down_proj.weight"}
    shapes = {"q": (64, 64), "k": (32, 64), "v": (32, 64), "o": (64, 64), "gate": (128, 64), "up": (128, 64),
              "down": (64, 128)}
    t = {"model.embed_tokens.weight": ("BF16", (256, 64), w["embedding"].astype("<u2").tobytes()),
         "model.norm.weight": ("BF16", (64,), w["final_norm"].astype("<u2").tobytes())}
    for l, L in enumerate(w["layers"]):
        for k, v in L.items():
            t[f"model.layers.{l}.{names[k]}"] = ("BF16", shapes.get(k, (v.size,)), v.astype("<u2").tobytes())
    data = safetensors_bytes(t)
    assert qb.inspect_safetensors(data, hf) == 26
    a = qb.Decoder.from_safetensors(data, hf, linear_format=linear_format)
    b = qb.Decoder(cfg, w, linear_format=linear_format)
    assert a.logical_weight_bytes() == b.logical_weight_bytes()
    prompt = synthetic.prompt(256, 12, seed=3)
    sa, sb = qb.CachedSession(a, 32), qb.CachedSession(b, 32)
    la, lb = sa.prefill(prompt), sb.prefill(prompt)
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    tok = int(np.argmax(la))
    for _ in range(6):
        la, lb = sa.step(tok), sb.step(tok)
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
        tok = int(np.argmax(la))
