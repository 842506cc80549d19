"""Tensor-parallel host plumbing on CPU: two gloo ranks share the NCCL unique id and agree on the
max-over-ranks time; the row sharding matches the library's (Q/K/V heads, gate/up rows, vocabulary)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from common_b200 import parallel


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nid = parallel.share_unique_id(lambda: bytes(range(128)))
        t = parallel.max_over_ranks(1.5 + rank)
        r, w, _ = parallel.launch_env()
        q.put((rank, nid, t, r, w))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_share_id_and_max_time():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0][1] == out[1][1] == bytes(range(128))
    assert out[0][2] == out[1][2] == 2.5
    assert [o[3] for o in out] == [0, 1] and all(o[4] == 2 for o in out)


def test_single_process_has_no_group():
    assert parallel.share_unique_id(lambda: b"x" * 128) is None
    assert parallel.max_over_ranks(3.0) == 3.0


@pytest.mark.parametrize("n,world", [(8, 2), (151936, 8), (12288, 4)])
def test_shard_rows_cover_everything(n, world):
    got = [parallel.shard_rows(n, r, world) for r in range(world)]
    assert got[0][0] == 0 and got[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
    with pytest.raises(ValueError):
        parallel.shard_rows(n + 1, 0, world)
