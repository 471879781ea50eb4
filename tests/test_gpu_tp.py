"""Tensor parallelism on two GPUs (one process per GPU, the ranks' exchange
buffers opened through CUDA IPC): the sharded model's greedy ids must equal
the single-GPU batch's and the oracle's, and its logits (every rank's
vocabulary rows in rank order) must match both within the BF16-KV
tolerance.  Skipped on a box with one GPU."""
import socket

import numpy as np
import pytest

from helpers import max_abs, oracle_weights
from llm_inference_edu_b200 import presets, synthetic

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(size, out_dir, name, prompt_len, steps, sequences, kv):
    import torch.multiprocessing as mp

    import tp_worker
    mp.spawn(tp_worker.run, args=(size, _port(), str(out_dir), name, prompt_len, steps, sequences, kv),
             nprocs=size, join=True)
    return [np.load(out_dir / f"rank{r}.npz") for r in range(size)]


def _gather(res, key):
    # Each rank holds the rows of its vocabulary tiles, in rank order.
    for a, b in zip(res, res[1:]):
        assert a["vocab"][1] == b["vocab"][0]
    return np.concatenate([r[key] for r in res], axis=1)


def _need_gpus(n):
    import torch
    if torch.cuda.device_count() < n:
        pytest.skip(f"tensor parallelism over {n} GPUs needs {n} GPUs")


def _oracle_ids(oracle, om, cap, prompt, steps):
    s = oracle.Session(om, cap, kv_bf16=True, budget=0)
    _, lg = s.append_chunked(list(prompt), True)
    first = lg
    ids = [int(np.argmax(lg))]
    for _ in range(steps):
        _, lg = s.step(ids[-1])
        ids.append(int(np.argmax(lg)))
    return first, ids, lg


HEADS_05B = {2: [(0, 7), (7, 14)], 4: [(0, 4), (4, 7), (7, 11), (11, 14)],
             8: [(0, 2), (2, 4), (4, 6), (6, 7), (7, 9), (9, 11), (11, 13), (13, 14)]}


@pytest.mark.parametrize("size", [2, 4, 8])
def test_tp_qwen05b_matches_single_gpu_and_oracle(oracle, tmp_path, size):
    # 0.5B shape (14 query heads, 2 KV heads): at TP=2 one KV group per
    # rank; at TP=4 and 8 each KV head is replicated on 2 or 4 ranks that
    # split its 7 query heads unevenly.  INT8 linears, BF16 table and KV,
    # two sequences of 48-token prompts, 12 greedy steps.
    _need_gpus(size)
    import llm_inference_edu_b200 as qb
    from helpers import qwen_host_weights
    P, steps, B = 48, 12, 2
    res = _spawn(size, tmp_path, "0.5b", P, steps, B, "bf16")
    assert [tuple(r["heads"].tolist()) for r in res] == HEADS_05B[size]
    for r in res[1:]:
        assert np.array_equal(r["first"], res[0]["first"]) and np.array_equal(r["ids"], res[0]["ids"])
    tp_first, tp_ids = res[0]["first"], res[0]["ids"]
    lg0, lg1 = _gather(res, "lg0"), _gather(res, "lg1")
    cap = P + steps + 8
    cfg = presets.qwen_0_5b(cap)
    w = qwen_host_weights("0.5b", 1, "bf16")
    prompts = np.stack([synthetic.prompt(cfg.vocab_size, P, seed=40 + s) for s in range(B)]).astype(np.uint32)
    m = qb.Decoder(cfg, w, linear_format="int8", table_format="bf16")
    b = qb.BatchSession(m, B, cap, kv_dtype="bf16")
    first = b.prefill(prompts)
    ref0 = b.logits()
    gen = b.decode_greedy(first, steps)
    ref1 = b.logits()
    assert np.array_equal(first, tp_first) and np.array_equal(gen, tp_ids)
    assert max(max_abs(lg0, ref0), max_abs(lg1, ref1)) <= 2e-2
    om = oracle.Model(cfg, oracle_weights(oracle, cfg, w, "int8"))
    worst = 0.0
    for s in range(B):
        of, oids, ol = _oracle_ids(oracle, om, cap, prompts[s], steps)
        assert [int(tp_first[s])] + [int(v) for v in tp_ids[:, s]] == oids, s
        worst = max(worst, max_abs(lg0[s], of), max_abs(lg1[s], ol))
    assert worst <= 2e-2, worst


def test_tp2_qwen7b_matches_oracle(oracle, tmp_path):
    # The 7B shape (28 query heads, 4 KV heads: two KV groups per rank),
    # INT8 linears, untied BF16 head, BF16 KV: one 64-token prompt, then 16
    # greedy ids identical to the oracle's (INT8 values and row scales in
    # host memory), the prompt's logits within the BF16-KV tolerance.
    _need_gpus(2)
    P, steps = 64, 15
    res = _spawn(2, tmp_path, "7b", P, steps, 1, "bf16")
    for r in res[1:]:
        assert np.array_equal(r["ids"], res[0]["ids"])
    lg0 = _gather(res, "lg0")
    cap = P + steps + 8
    cfg = presets.qwen_7b(cap)
    w = synthetic.weights(cfg, seed=2, dtype="bf16", lazy=True)
    om = oracle.Model(cfg, oracle.int8_model_weights(cfg, w, "int8"))
    del w
    prompt = synthetic.prompt(cfg.vocab_size, P, seed=40)
    of, oids, _ = _oracle_ids(oracle, om, cap, prompt, steps)
    assert [int(res[0]["first"][0])] + [int(v) for v in res[0]["ids"][:, 0]] == oids
    assert max_abs(lg0[0], of) <= 2e-2
