"""Multi-process host logic of the data-parallel replicas on CPU (gloo, world size 2): request
sharding, whole-job throughput (Σ units / max time over ranks) and result gathering, plus a rank
that fails before a collective: the others end with an error instead of waiting for ever."""
import datetime
import os
import socket

import pytest
import torch.multiprocessing as mp

from mlc_vla.replicas import shard_requests


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shards_are_disjoint_and_cover():
    for n in (0, 1, 7, 32, 33):
        for w in (1, 2, 3, 8):
            parts = [shard_requests(n, w, r) for r in range(w)]
            flat = [i for p in parts for i in p]
            assert flat == list(range(n))
            assert max(map(len, parts)) - min(map(len, parts)) <= 1
    with pytest.raises(ValueError):
        shard_requests(4, 2, 2)


def _worker(rank, world, port, q, fail_rank):
    import torch.distributed as dist

    from mlc_vla.replicas import gather_actions, shard_requests, whole_job_throughput

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        mine = shard_requests(10, world, rank)
        if rank == fail_rank:
            raise SystemExit(3)  # leaves before any collective
        # rank r "took" 100·(r+1) ms for its requests
        thr, ms = whole_job_throughput(100.0 * (rank + 1), len(mine))
        res = gather_actions([f"a{i}" for i in mine], world)
        q.put((rank, thr, ms, res))
    except SystemExit:
        raise
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", type(e).__name__, str(e)[:80]))
    finally:
        if rank != fail_rank:
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        assert not p.is_alive()
    out = []
    while not q.empty():
        out.append(q.get())
    return sorted(out, key=lambda x: x[0]), [p.exitcode for p in procs]


def test_two_ranks_throughput_and_gather():
    res, codes = _run(2)
    assert codes == [0, 0]
    assert len(res) == 2
    for rank, thr, ms, gathered in res:
        assert ms == pytest.approx(200.0)            # the slower rank bounds the job
        assert thr == pytest.approx(10 / 0.2)        # all 10 requests over 200 ms
        assert gathered == [f"a{i}" for i in range(10)]


def test_failed_rank_ends_collectives_with_an_error():
    res, codes = _run(2, fail_rank=1)
    assert codes[1] == 3
    assert len(res) == 1 and res[0][0] == 0 and res[0][1] == "error"
