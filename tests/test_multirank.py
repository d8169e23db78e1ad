"""World-size-2 gloo checks of the benchmark's rank plumbing (CPU)."""

import os
import socket

import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, ws, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(ws),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    from duplex import benchutil as bu
    import torch.distributed as dist
    bu.init_dist("gloo", timeout_s=60)
    got = bu.max_over_ranks(10.0 + rank)
    bu.barrier()
    q.put((rank, got, bu.dist_env()))
    dist.destroy_process_group()


def test_max_over_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [11.0, 11.0]
    assert res[0][2] == (2, 0, 0) and res[1][2] == (2, 1, 1)


def test_max_over_ranks_without_group():
    from duplex import benchutil as bu
    assert bu.max_over_ranks(3.5) == 3.5
