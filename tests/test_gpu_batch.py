"""GPU parity of batched greedy decode (BatchSession over the multi-token
kernels): every row must match the oracle's single-sequence session fed the
same tokens.  Every call goes through the C ABI."""
import numpy as np
import pytest

from conftest import assert_close
from helpers import max_abs, oracle_weights
from llm_inference_edu_b200 import presets, synthetic

pytestmark = pytest.mark.gpu


def _oracle_rows(oracle, om, cap, prompts, steps, kv_bf16=False):
    """Per row: logits after the prompt, the greedy ids of `steps` more steps
    and the logits of the last of them (serial oracle sessions)."""
    out = []
    for p in prompts:
        s = oracle.Session(om, cap, kv_bf16=kv_bf16, budget=0)
        _, lg = s.prefill(list(p))
        first_logits = lg
        ids = [int(np.argmax(lg))]
        for _ in range(steps):
            _, lg = s.step(ids[-1])
            ids.append(int(np.argmax(lg)))
        out.append((first_logits, ids, lg))
    return out


def test_tiny_batch_matches_oracle_rows(oracle):
    import llm_inference_edu_b200 as qb
    w = presets.tiny_r_weights()
    cfg = presets.tiny_r(32)
    m = qb.Decoder(cfg, w)
    om = oracle.Model(cfg, w)
    prompts = np.array([[1, 5, 7, 7], [2, 63, 0, 41], [9, 9, 9, 9]], np.uint32)
    steps = 6
    rows = _oracle_rows(oracle, om, 32, prompts, steps)
    b = qb.BatchSession(m, 3, 32)
    first = b.prefill(prompts)
    assert b.processed() == 4
    for r, (lg0, ids, _) in enumerate(rows):
        assert int(first[r]) == ids[0]
    got0 = b.logits()
    for r, (lg0, _, _) in enumerate(rows):
        assert_close(got0[r], lg0, name=f"prefill row {r}")
    gen = b.decode_greedy(first, steps)
    assert gen.shape == (steps, 3) and b.processed() == 4 + steps
    for r, (_, ids, lgl) in enumerate(rows):
        # step k consumed ids[k] and produced ids[k + 1]
        assert [int(v) for v in gen[:, r]] == ids[1:], r
        assert_close(b.logits()[r], lgl, name=f"last row {r}")
    # Lifecycle and errors (the CachedSession kinds).
    with pytest.raises(qb.CacheError) as e:
        b.prefill(prompts)
    assert e.value.kind == "NotEmpty"
    with pytest.raises(qb.CacheError) as e:
        b.decode_greedy(first, 32)
    assert e.value.kind == "Full" and b.processed() == 4 + steps
    with pytest.raises(qb.CacheError) as e:
        b.decode_greedy(np.array([1, 64, 2], np.uint32), 1)
    assert e.value.kind == "InvalidToken"
    b.reset()
    assert b.processed() == 0 and b.is_valid()
    with pytest.raises(qb.CacheError) as e:
        b.logits()
    assert e.value.kind == "NotStarted"
    with pytest.raises(qb.CacheError) as e:
        b.prefill(np.array([[1, 64], [1, 1], [1, 1]], np.uint32))
    assert e.value.kind == "InvalidToken" and b.processed() == 0
    # After reset the same prompts give the same ids (stale K/V is never read).
    again = b.prefill(prompts)
    assert np.array_equal(again, first)
    with pytest.raises(qb.CacheError) as e:
        qb.BatchSession(m, 0, 8)
    assert e.value.kind == "InvalidCapacity"
    with pytest.raises(qb.CacheError) as e:
        qb.BatchSession(m, 2, 33)
    assert e.value.kind == "InvalidCapacity"


def test_tiny_batch_single_token_prompts(oracle):
    # prompt_len 1: no KV fill launch, only the LM-head row per sequence.
    import llm_inference_edu_b200 as qb
    w = presets.tiny_r_weights()
    cfg = presets.tiny_r(16)
    m = qb.Decoder(cfg, w)
    om = oracle.Model(cfg, w)
    prompts = np.array([[3], [60]], np.uint32)
    rows = _oracle_rows(oracle, om, 16, prompts, 4)
    b = qb.BatchSession(m, 2, 16)
    first = b.prefill(prompts)
    gen = b.decode_greedy(first, 4)
    for r, (_, ids, lgl) in enumerate(rows):
        assert [int(first[r])] + [int(v) for v in gen[:, r]] == ids
        assert_close(b.logits()[r], lgl)


@pytest.mark.parametrize("linear_format,kv,tol", [("int8", "f32", 1e-3), ("int8", "bf16", 2e-2)])
def test_qwen05b_batch_rows_match_oracle(oracle, linear_format, kv, tol):
    # 0.5B shape, three sequences with different 40-token prompts, 12
    # greedy steps: last logits per row within the FP32 (f32 KV) or BF16
    # (bf16 KV) tolerance, greedy ids identical.
    import llm_inference_edu_b200 as qb
    from helpers import qwen_host_weights
    plen, steps, B = 40, 12, 3
    cap = plen + steps + 4
    cfg = presets.qwen_0_5b(cap)
    w = qwen_host_weights("0.5b", 1, "bf16")
    m = qb.Decoder(cfg, w, linear_format=linear_format, table_format="bf16")
    om = oracle.Model(cfg, oracle_weights(oracle, cfg, w, linear_format))
    prompts = np.stack([synthetic.prompt(cfg.vocab_size, plen, seed=10 + r) for r in range(B)]).astype(np.uint32)
    rows = _oracle_rows(oracle, om, cap, prompts, steps, kv_bf16=(kv == "bf16"))
    b = qb.BatchSession(m, B, cap, kv_dtype=kv)
    first = b.prefill(prompts)
    worst = max(max_abs(b.logits()[r], rows[r][0]) for r in range(B))
    gen = b.decode_greedy(first, steps)
    last = b.logits()
    for r, (_, ids, lgl) in enumerate(rows):
        assert [int(first[r])] + [int(v) for v in gen[:, r]] == ids, r
        worst = max(worst, max_abs(last[r], lgl))
    assert worst <= tol, worst


def test_qwen05b_batch64_matches_sessions():
    # The batched workload (64 sequences) against 64 single-sequence device
    # sessions on the same prompts: identical greedy ids.
    import llm_inference_edu_b200 as qb
    from helpers import qwen_host_weights
    plen, steps, B = 16, 24, 64
    cap = plen + steps + 1
    cfg = presets.qwen_0_5b(cap)
    w = qwen_host_weights("0.5b", 2, "bf16")
    m = qb.Decoder(cfg, w, linear_format="int8", table_format="bf16")
    prompts = np.stack([synthetic.prompt(cfg.vocab_size, plen, seed=100 + r) for r in range(B)]).astype(np.uint32)
    b = qb.BatchSession(m, B, cap)
    first = b.prefill(prompts)
    gen = b.decode_greedy(first, steps)
    s = qb.CachedSession(m, cap, budget=0)
    mismatched = 0
    for r in range(B):
        s.reset()
        f = int(np.argmax(s.prefill(list(prompts[r]))))
        ids = [f] + s.decode_greedy(f, steps)
        mismatched += ids != [int(first[r])] + [int(v) for v in gen[:, r]]
    assert mismatched == 0, mismatched


def test_qwen7b_decode_kernel_matches_multitoken_path(oracle):
    # The 7B shape (hd 128, 4 KV heads, untied head, INT8 per-row linears,
    # BF16 tables and KV) on one GPU: a 64-token prompt, then 16 greedy ids.
    # Against the oracle (INT8 values and row scales held in host memory,
    # the crate's x * (f32(q) * s) order): the prompt's last logits within
    # the BF16-KV tolerance and the 16 ids identical.  The persistent decode
    # kernel and the tensor-core multi-token path must also agree with each
    # other.
    import llm_inference_edu_b200 as qb
    P, steps = 64, 16
    cap = P + steps + 8
    cfg = presets.qwen_7b(cap)
    w = synthetic.weights(cfg, seed=2, dtype="bf16", lazy=True)
    m = qb.Decoder(cfg, w, linear_format="int8", table_format="bf16")
    # The oracle quantizes each lazily drawn layer itself and keeps only the
    # INT8 values and scales (~6.5 GB) plus the two BF16 tables.
    om = oracle.Model(cfg, oracle.int8_model_weights(cfg, w, "int8"))
    del w
    prompt = synthetic.prompt(cfg.vocab_size, P, seed=3)
    s = qb.CachedSession(m, cap, kv_dtype="bf16", budget=0)
    got = s.prefill(prompt)
    first = int(np.argmax(got))
    os_ = oracle.Session(om, cap, kv_bf16=True, budget=0)
    _, exp = os_.append_chunked(prompt, True)
    assert max_abs(got, exp) <= 2e-2, max_abs(got, exp)
    assert int(np.argmax(exp)) == first
    or_ids = [first]
    for _ in range(steps - 1):
        _, lg = os_.step(or_ids[-1])
        or_ids.append(int(np.argmax(lg)))
    dev = [first] + s.decode_greedy(first, steps - 1)
    assert dev == or_ids
    b = qb.BatchSession(m, 1, cap, kv_dtype="bf16")
    f = b.prefill(np.asarray(prompt, np.uint32)[None, :])
    g = b.decode_greedy(f, steps - 1)
    alt = [int(f[0])] + [int(v) for v in g[:, 0]]
    assert dev == alt
    # Same position, both paths: logits after feeding the last id.
    s_logits = s.step(dev[-1])
    b.decode_greedy(np.asarray([dev[-1]], np.uint32), 1)
    assert max_abs(s_logits, b.logits()[0]) <= 2e-2
