"""Row-sharded LittleBitLinear (8192 -> 28672, rank 616, the 70B MLP shape)
over 2 GPUs with an NCCL all-gather: the gathered y equals the unsharded
layer bit for bit (every rank's V-stage is identical and a U tile's
arithmetic does not depend on which rows surround it).  Needs 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, ws, port, q):
    import datetime

    import torch.distributed as dist

    from littlebit_b200 import ops, synthetic
    from littlebit_b200.sharded import RowShardedLinear

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(9)  # same weights and inputs on every rank
        brs = synthetic.layer(8192, 28672, [616], g)
        full = synthetic.to_packed_linear(8192, 28672, brs, torch.device("cuda", rank))
        x = torch.randn(3, 8192, generator=g).cuda(rank)
        sh = RowShardedLinear(full, ws, rank)
        y = sh.forward(x)
        ref = ops.lb_linear(full, x)
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(y, ref)), float((y - ref).abs().max())))
    except Exception as e:
        q.put((rank, False, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_row_sharded_matches_unsharded_bitwise():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] for r in res), res


def _fused_worker(rank, ws, port, q):
    import datetime

    import torch.distributed as dist

    from littlebit_b200 import ops, synthetic
    from littlebit_b200.sharded import FusedRowShardedLinear

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    fsh = None
    try:
        g = torch.Generator().manual_seed(11)  # same weights and inputs on every rank
        brs = synthetic.layer(8192, 28672, [616], g)
        full = synthetic.to_packed_linear(8192, 28672, brs, torch.device("cuda", rank))
        fsh = FusedRowShardedLinear(full, ws, rank, max_tokens=8)
        ok, worst = True, 0.0
        # alternating buffer halves, ragged token counts, back-to-back calls
        for k in [1, 3, 8, 1, 5, 2, 1]:
            x = torch.randn(k, 8192, generator=g).cuda(rank)
            y = fsh.forward(x)
            ref = ops.lb_linear(full, x)
            torch.cuda.synchronize()
            ok &= bool(torch.equal(y, ref))
            worst = max(worst, float((y - ref).abs().max()))
        err = ops.device_error(torch.device("cuda", rank))
        q.put((rank, ok and err == 0, worst, err))
    except Exception as e:
        q.put((rank, False, repr(e), -1))
    finally:
        if fsh is not None:
            fsh.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_allgather_matches_unsharded_bitwise():
    """The all-gather fused into the U-stage (tagged NVLink stores, polled by
    the unpack kernel) gives every rank the unsharded layer's y bit for bit."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] for r in res), res
