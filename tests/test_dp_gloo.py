"""The data-parallel host logic (llm_inference_edu_b200.dp) with two gloo
ranks on CPU: sequence sharding, the max-over-ranks timing reduction, and a
rank that fails before a collective (the survivor must get an error, not
hang)."""
import multiprocessing as mp
import os
import socket

import pytest

from conftest import ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, out):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    from llm_inference_edu_b200 import dp
    topo = dp.topology_from_env()
    try:
        dp.init(topo, "gloo", timeout_s=20.0)
        if mode == "ok":
            ids = dp.sequence_ids(topo, 5)
            dp.barrier(topo)
            m = dp.max_over_ranks(topo, 1.5 + rank)
            out.put((rank, ids, m, None))
        else:  # rank 1 fails before the collective
            if rank == 1:
                raise RuntimeError("injected failure on rank 1")
            dp.max_over_ranks(topo, 1.0)
            out.put((rank, None, None, "no error"))
    except Exception as e:  # reported to the parent
        out.put((rank, None, None, type(e).__name__ + ": " + str(e)[:200]))
    finally:
        try:
            dp.shutdown(topo)
        except Exception:
            pass


def _run(mode, world=2, timeout=90):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = q.get(timeout=timeout)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


def test_topology_and_sharding_single_process():
    from llm_inference_edu_b200 import dp
    t = dp.Topology(0, 1, 0)
    assert not t.distributed and dp.sequence_ids(t, 3) == [0, 1, 2]
    assert dp.max_over_ranks(t, 2.5) == 2.5
    parts = [dp.sequence_ids(dp.Topology(r, 3, r), 8) for r in range(3)]
    assert parts == [[0, 1, 2], [3, 4, 5], [6, 7]]
    assert [dp.sequence_ids(dp.Topology(r, 4, r), 2) for r in range(4)] == [[0], [1], [], []]
    with pytest.raises(ValueError):
        dp.sequence_ids(t, -1)


def test_two_ranks_shard_and_reduce():
    res = _run("ok")
    assert res[0][3] is None and res[1][3] is None, res
    assert res[0][1] == [0, 1, 2] and res[1][1] == [3, 4]
    assert res[0][2] == 2.5 and res[1][2] == 2.5


def test_failed_rank_surfaces_as_error():
    res = _run("fail")
    assert "injected failure" in res[1][3]
    # The surviving rank's collective ends with an error (connection closed
    # or timeout), never a silent success or a hang.
    assert res[0][3] is not None and res[0][3] != "no error", res
