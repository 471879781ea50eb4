"""A checkpoint loaded from safetensors (qb_model_load_safetensors) decodes
exactly like the same BF16 weights set tensor by tensor: the BF16 -> FP32
expansion is exact and every tensor lands in its place (tests/weights.rs:48-62
checks the expansion on the host)."""
import numpy as np
import pytest

from helpers import small_qwen_checkpoint

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("linear_format", ["f32", "int8"])
def test_safetensors_model_decodes_like_the_dictionary_model(linear_format):
    import llm_inference_edu_b200 as qb
    from llm_inference_edu_b200 import synthetic
    hf, cfg, w, data = small_qwen_checkpoint()
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
