"""Seeded temperature / top-k sampling on the device against the oracle's
restatement of Sampler::sample (src/sampling.rs:57-110): the same ids for
the same logits and seed, over Qwen-sized vocabularies, ties and every
selection path (shared-memory and scratch-buffer sorts), and through
GenerationSession on the device logits of a 0.5B-shaped model."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

V = 151936


def _pair(oracle, t, k, seed):
    import llm_inference_edu_b200 as qb
    return qb.Sampler(qb.Sampling.Temperature(t, k, seed)), oracle.Sampler(temperature=t, top_k=k, seed=seed)


def test_reference_sampling_tests_on_device(oracle):
    # tests/sampling.rs:10-100 through the C ABI (host logits).
    import llm_inference_edu_b200 as qb
    T = qb.Sampling.Temperature
    assert qb.Sampler(qb.Sampling.Greedy).sample([2.0, 2.0, 1.0]) == 0
    assert qb.Sampler(T(1.0, 1, 42)).sample([-0.0, 0.0]) == 0
    for _ in range(100):
        assert qb.Sampler(T(1.0, 2, 42)).sample([-10.0, 0.0, 3.0, 4.0]) >= 2
    a, b = qb.Sampler(T(1.0, 2, 42)), qb.Sampler(T(1.0, 2, 42))
    with pytest.raises(qb.SamplingError) as e:
        a.sample([float("nan"), 0.0])
    assert e.value.kind == "NonFinite"
    seq = [a.sample([0.0, 1.0]) for _ in range(64)]
    assert seq == [b.sample([0.0, 1.0]) for _ in range(64)]
    a.reset()
    assert seq == [a.sample([0.0, 1.0]) for _ in range(64)]
    assert 0 in seq and 1 in seq
    o = oracle.Sampler(temperature=1.0, top_k=2, seed=42)
    assert seq == [o.sample([0.0, 1.0])[1] for _ in range(64)]
    s = qb.Sampler(T(1.0, 2, 42))
    count = sum(s.sample([0.0, math.log(3.0)]) == 1 for _ in range(10000))
    assert 7350 <= count <= 7650, count
    for bad, kind in [([], "EmptyLogits"), ([0.0], "InvalidParameters"), ([float("inf"), 0.0], "NonFinite"),
                      ([float("-inf"), 0.0], "NonFinite"), ([float("nan")], "NonFinite")]:
        with pytest.raises(qb.SamplingError) as e:
            qb.Sampler(T(1.0, 2, 42)).sample(bad)
        assert e.value.kind == kind
    tiny = float(np.array([1], dtype=np.uint32).view(np.float32)[0])
    fmax = float(np.finfo(np.float32).max)
    assert qb.Sampler(T(tiny, 2, 42)).sample([-fmax, fmax]) == 1


def test_errors_leave_the_stream_alone(oracle):
    import llm_inference_edu_b200 as qb
    s, o = _pair(oracle, 0.9, 8, 5)
    lg = np.random.default_rng(0).standard_normal(1000).astype(np.float32)
    bad = lg.copy()
    bad[777] = np.inf
    ids = []
    for i in range(20):
        if i % 3 == 0:
            with pytest.raises(qb.SamplingError):
                s.sample(bad)
        ids.append(s.sample(lg))
    assert ids == [o.sample(lg)[1] for _ in range(20)]


@pytest.mark.parametrize("t,k,draws", [(0.7, 40, 200), (1.0, 1, 50), (1.3, 4096, 40), (1.1, 5000, 20),
                                       (0.9, V, 6)])
def test_device_matches_oracle_qwen_vocab(oracle, t, k, draws):
    # Fresh logits every draw (normal, scale 2.5); k = 4096 sorts in shared
    # memory, 5000 and the whole vocabulary in the scratch buffer.
    s, o = _pair(oracle, t, k, 1234 + k)
    rng = np.random.default_rng(k)
    for d in range(draws):
        lg = (rng.standard_normal(V) * 2.5).astype(np.float32)
        assert s.sample(lg) == o.sample(lg)[1], d


@pytest.mark.parametrize("k", [3, 40, 1000, 9000])
def test_ties_take_the_lowest_ids(oracle, k):
    # Logits on a coarse grid (many equal values, -0 and +0 among them):
    # the k-th value's ties are cut by id, as the reference's total order.
    s, o = _pair(oracle, 0.5, k, 99)
    rng = np.random.default_rng(7)
    for d in range(12):
        lg = (rng.integers(-24, 25, V) / 4).astype(np.float32)
        lg[rng.integers(0, V, 500)] = -0.0
        assert s.sample(lg) == o.sample(lg)[1], d


def test_device_tensor_input(oracle):
    import torch
    s, o = _pair(oracle, 0.8, 50, 3)
    rng = np.random.default_rng(3)
    for _ in range(10):
        lg = (rng.standard_normal(V) * 3).astype(np.float32)
        assert s.sample(torch.from_numpy(lg).cuda()) == o.sample(lg)[1]


def test_generation_samples_the_device_logits(oracle):
    # 0.5B shape, INT8 linears, BF16 table, F32 KV: a sampled continuation
    # (T = 0.8, top-k 40, seed 2024) equals the oracle sampler run over the
    # same device logits (a cached session fed the same ids); reset and
    # replay restart the stream.
    import llm_inference_edu_b200 as qb
    from helpers import qwen_host_weights
    from llm_inference_edu_b200 import presets, synthetic
    P, N, cap = 32, 24, 64
    cfg = presets.qwen_0_5b(cap)
    m = qb.Decoder(cfg, qwen_host_weights("0.5b", 1, "bf16"), linear_format="int8", table_format="bf16")
    prompt = [int(v) for v in synthetic.prompt(cfg.vocab_size, P, seed=11)]
    pol = qb.Sampling.Temperature(0.8, 40, 2024)
    g = qb.GenerationSession(m, cap, pol, [], N)
    g.start(prompt)
    ids = [g.next_token() for _ in range(N)]
    assert g.next_token() is None and g.stop_reason() == "OutputLimit"
    cs = qb.CachedSession(m, cap)
    lg = cs.append(prompt)
    o = oracle.Sampler(temperature=0.8, top_k=40, seed=2024)
    want = []
    for _ in range(N):
        want.append(o.sample(lg)[1])
        lg = cs.step(want[-1])
    assert ids == want
    assert len(set(ids)) > 1
    g.reset()
    g.start(prompt)
    assert [g.next_token() for _ in range(N)] == ids
    g.replay_history(prompt, N)
    assert [g.next_token() for _ in range(N)] == ids
