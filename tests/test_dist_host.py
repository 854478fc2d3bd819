"""Multi-rank host logic on CPU with the gloo backend (world size 2): request
split, row shards, max/sum over ranks, gather layout of the row-sharded linear,
and the fault path -- a rank that never reaches a collective makes the other
rank's collective fail within the short process-group timeout."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from littlebit_b200 import sharded


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, ws, port, timeout_s=20):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(ws),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _worker_basic(rank, ws, port, q):
    dist = _init(rank, ws, port)
    try:
        # max / sum over ranks
        assert sharded.max_over_ranks(1.5 + rank, ws) == 1.5 + ws - 1
        assert sharded.sum_over_ranks(rank + 1, ws) == ws * (ws + 1) / 2
        # each rank's U-row slice gathers back into the full row order
        N, k = 64, 3
        full = torch.arange(k * N, dtype=torch.float32).reshape(k, N)
        lo, hi = sharded.shard_rows(N, ws, rank)
        parts = [torch.empty(k, hi - lo) for _ in range(ws)]
        dist.all_gather(parts, full[:, lo:hi].contiguous())
        assert torch.equal(sharded.assemble_rows(parts), full)
        sharded.barrier(ws)
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent, which asserts
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _worker_fault(rank, ws, port, q):
    dist = _init(rank, ws, port, timeout_s=3)
    if rank == 1:  # leaves between steps: never joins the next collective
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # flush the message before the abrupt exit
        os._exit(0)
    try:
        sharded.barrier(ws)
        q.put((rank, "barrier returned"))
    except Exception as e:
        q.put((rank, "error: " + type(e).__name__))


def _run(target, ws=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=timeout) for _ in range(ws))
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return out


def test_split_requests_and_shards():
    for n, ws in ((64, 8), (10, 4), (3, 8), (1, 1)):
        got = [i for r in range(ws) for i in sharded.split_requests(n, ws, r)]
        assert got == list(range(n))
    assert [sharded.shard_rows(28672, 8, r) for r in (0, 7)] == [(0, 3584), (25088, 28672)]
    with pytest.raises(ValueError):
        sharded.shard_rows(100, 8, 0)


def test_gloo_two_ranks():
    out = _run(_worker_basic)
    assert out == {0: "ok", 1: "ok"}, out


def test_rank_that_leaves_fails_the_collective_not_the_process():
    out = _run(_worker_fault)
    assert out[1] == "left"
    assert out[0].startswith("error"), out
