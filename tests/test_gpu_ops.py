"""GPU parity of the standalone operator kernels against the oracle and the
reference's golden vectors (called through the C ABI)."""
import numpy as np
import pytest

from conftest import assert_close, golden

pytestmark = pytest.mark.gpu


def dev(a, dtype=None):
    import torch
    t = torch.as_tensor(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def zeros(n, fill=37.0):
    import torch
    return torch.full((n,), fill, dtype=torch.float32, device="cuda")


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def test_linear_known_answers_and_f64():
    import llm_inference_edu_b200 as qb
    from oracle import oracle
    y = zeros(4)
    qb.linear(dev(np.float32([1, 2, 3, 4, 5, 6])), dev(np.float32([1, 0, -1, 2, 1, 0])), y, 2, 3, 2)
    assert list(host(y)) == [-2, 4, -2, 13]
    for n in [1, 3, 5, 31, 64, 127, 896, 4864]:
        x = (((np.arange(3 * n) * 17 % 101) - 50.0) / 53).astype(np.float32)
        w = (((np.arange(7 * n) * 23 % 97) - 48.0) / 61).astype(np.float32)
        exp = x.reshape(3, n).astype(np.float64) @ w.reshape(7, n).astype(np.float64).T
        for lanes, fn in ((False, qb.linear), (True, qb.linear_lanes4)):
            y = zeros(21)
            fn(dev(x), dev(w), y, 3, n, 7)
            assert_close(host(y), exp.ravel(), name=f"n={n}")
            # the reference's own summation order: bit-identical
            _, ref, _ = oracle.linear(x, w, 3, n, 7, lanes4=lanes)
            assert np.array_equal(host(y).view(np.uint32), ref.view(np.uint32)), (n, lanes)


def test_linear_bit_exact_at_model_shapes():
    # Every standalone linear follows the crate's order (scalar, or the four
    # lanes of dot_lanes4), so outputs are bit-identical to the oracle's
    # restatement at the 0.5B shapes, including tails (in % 4 != 0) and
    # more rows than one CTA holds.
    import llm_inference_edu_b200 as qb
    from oracle import oracle
    rng = np.random.default_rng(11)
    for t, n, o in [(1, 896, 1152), (3, 4864, 130), (2, 1003, 257)]:
        x = rng.standard_normal(t * n).astype(np.float32)
        w = (rng.standard_normal(o * n) * 0.02).astype(np.float32)
        for lanes, fn in ((False, qb.linear), (True, qb.linear_lanes4)):
            y = zeros(t * o)
            fn(dev(x), dev(w), y, t, n, o)
            _, ref, _ = oracle.linear(x, w, t, n, o, lanes4=lanes)
            assert np.array_equal(host(y).view(np.uint32), ref.view(np.uint32)), (t, n, o, lanes)


def test_linear_admission_leaves_output_unchanged():
    import llm_inference_edu_b200 as qb
    for xl, wl, yl in [(5, 6, 4), (7, 6, 4), (6, 5, 4), (6, 7, 4), (6, 6, 3), (6, 6, 5)]:
        y = zeros(yl)
        with pytest.raises(qb.LinearError) as e:
            qb.linear(dev(np.ones(xl, np.float32)), dev(np.ones(wl, np.float32)), y, 2, 3, 2)
        assert e.value.kind == "InvalidLength"
        assert np.all(host(y) == 37.0)


def test_linear_bf16_weights():
    import torch
    import llm_inference_edu_b200 as qb
    from llm_inference_edu_b200 import synthetic
    from oracle import oracle
    w16 = synthetic.normal(0, 9, 300 * 896, 0.02, "bf16")
    x = synthetic.normal(0, 10, 2 * 896, 1.0, "f32")
    y = zeros(600)
    qb.linear(dev(x), dev(w16.view(np.int16)).view(torch.int16), y, 2, 896, 300)
    _, ref, _ = oracle.linear(x, synthetic.as_f32(w16), 2, 896, 300)
    assert np.array_equal(host(y).view(np.uint32), ref.view(np.uint32))


def test_quantize_bit_exact_and_kats():
    import llm_inference_edu_b200 as qb
    from oracle import oracle
    q = qb.GroupwiseInt8.quantize(dev(np.float32([127, 0.5, -0.5, 0, 254, 0, 0, 0, 0, 0])), 2, 5, 4)
    assert list(host(q.values)) == [127, 1, -1, 0, 127, 0, 0, 0, 0, 0]
    assert list(host(q.scales)) == [1, 2, 1, 1]
    mx = np.array([1061777744, 1053389136], dtype=np.uint32).view(np.float32)
    q = qb.GroupwiseInt8.quantize(dev(mx), 1, 2, 2)
    assert host(q.scales).view(np.uint32)[0] == 1003161439 and list(host(q.values)) == [127, 64]
    q = qb.GroupwiseInt8.quantize(dev(np.array([190], np.uint32).view(np.float32)), 1, 1, 32)
    assert host(q.scales).view(np.uint32)[0] == 1 and list(host(q.values)) == [127]
    rng = np.random.default_rng(0)
    for rows, width, group in [(7, 896, 32), (7, 896, 896), (33, 4864, 4864), (5, 127, 3), (3, 1000, 256)]:
        w = (rng.standard_normal(rows * width) * 0.02).astype(np.float32)
        w[::97] *= 50  # outliers
        w[5 * 0:3] = 0
        q = qb.GroupwiseInt8.quantize(dev(w), rows, width, group)
        s, ref = oracle.quantize(w, rows, width, group)
        assert np.array_equal(host(q.values), ref.values.ravel())
        assert np.array_equal(host(q.scales).view(np.uint32), ref.scales.ravel().view(np.uint32))
        x = rng.standard_normal(2 * width).astype(np.float32)
        for lanes, fn in ((False, qb.linear_int8), (True, qb.linear_int8_lanes4)):
            y = zeros(2 * rows)
            fn(dev(x), q, y, 2)
            _, yr = oracle.linear_int8(x, ref, 2, lanes4=lanes)
            # x * (f32(q) * scale) summed in the crate's order: bit-identical
            assert np.array_equal(host(y).view(np.uint32), yr.view(np.uint32)), (rows, width, group, lanes)


def test_quantize_admission_writes_nothing():
    import torch
    import llm_inference_edu_b200 as qb
    for v in [np.nan, np.inf]:
        with pytest.raises(qb.QuantError) as e:
            qb.GroupwiseInt8.quantize(dev(np.float32([1, v])), 1, 2, 32)
        assert e.value.kind == "NonFiniteWeight" and e.value.index == 1
    with pytest.raises(qb.QuantError) as e:
        qb.GroupwiseInt8.quantize(dev(np.array([1], np.uint32).view(np.float32)), 1, 1, 32)
    assert e.value.kind == "UnrepresentableScale"
    with pytest.raises(qb.QuantError) as e:
        qb.GroupwiseInt8.quantize(dev(np.ones(4, np.float32)), 2, 2, 0)
    assert e.value.kind == "InvalidGroupSize"


def test_ops_match_t01():
    import torch
    import llm_inference_edu_b200 as qb
    inp, exp = golden("t01-inputs.json"), golden("t01-expected.json")["outputs"]
    c = inp["embedding"]
    y = zeros(12)
    qb.embedding(c["token_ids"], dev(np.float32(c["table"])), y, c["vocab_size"], c["width"])
    assert_close(host(y), exp["embedding"])
    c = inp["residual_add"]
    y = zeros(6)
    qb.residual_add(dev(np.float32(c["x"])), dev(np.float32(c["residual"])), y)
    assert_close(host(y), exp["residual_add"])
    c = inp["rmsnorm"]
    y = zeros(6)
    qb.rmsnorm(dev(np.float32(c["x"])), dev(np.float32(c["weight"])), y, 2, 3, c["epsilon"])
    assert_close(host(y), exp["rmsnorm"])
    y = zeros(7)
    qb.silu(dev(np.float32(inp["silu"]["x"])), y)
    assert_close(host(y), exp["silu"])
    c = inp["softmax"]
    y = zeros(6)
    qb.softmax(dev(np.float32(c["logits"])), y, 2, 3)
    assert_close(host(y), exp["softmax"])
    c = inp["masked_softmax"]
    y = zeros(12)
    qb.masked_softmax(dev(np.float32(c["logits"])), dev(np.uint8(c["mask"])), y, 3, 4)
    assert_close(host(y), exp["masked_softmax"])


def test_op_admission():
    import llm_inference_edu_b200 as qb
    y = zeros(2)
    with pytest.raises(qb.OpError) as e:
        qb.embedding([0, 5], dev(np.ones(6, np.float32)), zeros(6), 2, 3)
    assert e.value.kind == "InvalidToken"
    with pytest.raises(qb.OpError) as e:
        qb.rmsnorm(dev(np.float32([1, np.nan])), dev(np.ones(2, np.float32)), y, 1, 2, 1e-5)
    assert e.value.kind == "NonFinite"
    assert np.all(host(y) == 37)
    with pytest.raises(qb.OpError) as e:
        qb.masked_softmax(dev(np.float32([1, 2, 3, 4])), dev(np.uint8([1, 1, 0, 0])), zeros(4), 2, 2)
    assert e.value.kind == "AllMasked"


def test_rope_matches_t02_and_oracle_bitwise():
    import llm_inference_edu_b200 as qb
    from oracle import oracle
    inp, exp = golden("t02-inputs.json"), golden("t02-expected.json")["outputs"]
    for c in inp["cases"]:
        y = zeros(len(c["x"]))
        qb.rope(dev(np.float32(c["x"])), y, c["tokens"], c["heads"], c["head_dim"], c["start_position"], c["base"])
        assert_close(host(y), exp[c["name"]])
    x = np.random.default_rng(1).standard_normal(5 * 14 * 64).astype(np.float32)
    y = zeros(x.size)
    qb.rope(dev(x), y, 5, 14, 64, 1000, 1e6)
    _, ref = oracle.rope(x, 5, 14, 64, 1000, 1e6)
    assert np.array_equal(host(y), ref)
