"""CPU checks of the tensor-parallel host logic: the shard rule (heads by
KV group, KV heads replicated beyond the KV-head count, FFN columns, LM-head
tiles) and the communicator-handle exchange over two gloo ranks."""
import datetime
import socket

import pytest

from llm_inference_edu_b200 import presets


def shards(cfg, size):
    from llm_inference_edu_b200 import tp_shard_of
    return [tp_shard_of(cfg, r, size) for r in range(size)]


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_qwen7b_shards_cover_the_model_once(size):
    cfg = presets.qwen_7b()
    sh = shards(cfg, size)
    heads = [h for s in sh for h in range(*s["heads"])]
    assert heads == list(range(cfg.query_heads))
    group = cfg.query_heads // cfg.kv_heads
    for s in sh:
        # every query head's KV head is on the same rank
        kv = set(h // group for h in range(*s["heads"]))
        assert kv == set(range(*s["kv_heads"]))
    ff = [f for s in sh for f in (s["ff"][0], s["ff"][1])]
    assert ff[0] == 0 and ff[-1] == cfg.ff_dim and all(a == b for a, b in zip(ff[1:-1:2], ff[2:-1:2]))
    v = [s["vocab"] for s in sh]
    assert v[0][0] == 0 and v[-1][1] == cfg.vocab_size
    assert all(a[1] == b[0] and a[1] % 128 == 0 for a, b in zip(v, v[1:]))


def test_qwen7b_tp8_replicates_kv_heads_with_4_3_head_splits():
    sh = shards(presets.qwen_7b(), 8)
    assert [s["heads"][1] - s["heads"][0] for s in sh] == [4, 3] * 4
    assert [s["kv_heads"] for s in sh] == [(0, 1), (0, 1), (1, 2), (1, 2), (2, 3), (2, 3), (3, 4), (3, 4)]
    assert all(s["ff"][1] - s["ff"][0] == 2368 for s in sh)


def test_unsplittable_sizes_are_refused():
    from llm_inference_edu_b200 import ModelError, tp_shard_of
    for size in (3, 16):
        with pytest.raises(ModelError) as e:
            tp_shard_of(presets.qwen_7b(), 0, size)
        assert e.value.kind == "Unsupported"
    # 0.5B: 2 KV heads of 7 query heads; 4 ranks split each group 4 + 3
    sh = shards(presets.qwen_0_5b(), 4)
    assert [s["heads"] for s in sh] == [(0, 4), (4, 7), (7, 11), (11, 14)]


class _FakeComm:
    def __init__(self, rank):
        self.rank = rank
        self.got = None

    def handle(self):
        return bytes([self.rank]) * 64

    def connect(self, rank, handles):
        self.got = (rank, handles)


def _rank(rank, port, out):
    import torch.distributed as dist

    from llm_inference_edu_b200 import tp
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=30))
    try:
        c = _FakeComm(rank)
        tp.connect(c, rank, 2)
        out.put((rank, c.got))
    finally:
        dist.destroy_process_group()


def test_handles_are_exchanged_in_rank_order():
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=60) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    for r in range(2):
        rank, handles = got[r]
        assert rank == r
        assert handles == [bytes([0]) * 64, bytes([1]) * 64]
