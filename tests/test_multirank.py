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
    # a rank whose replay looked 3x faster must still soak as many replays as the others
    soak = bu.soak_replays(1.0, 0.01 if rank == 0 else 0.03)
    bu.barrier()
    q.put((rank, got, bu.dist_env(), soak))
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
    assert [r[3] for r in res] == [33, 33]    # int(1.0 / 0.03) on both ranks


def test_max_over_ranks_without_group():
    from duplex import benchutil as bu
    assert bu.max_over_ranks(3.5) == 3.5
    assert bu.soak_replays(1.0, 0.25) == 4 and bu.soak_replays(0.0, 0.25) == 0
    assert bu.soak_replays(1.0, 5.0) == 1


# ------------------------------------------------------------------ expert parallelism
def _ep_worker(rank, ws, port, q):
    """One rank of the expert-parallel layer's host logic (ep_forward) on CPU/gloo, with
    the numpy oracle as the routing and local-expert steps."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(ws),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    import numpy as np
    import torch
    import torch.distributed as dist

    import oracle as O
    from duplex import synth
    from duplex.streaming.ep_moe import ep_forward
    from ep_ref import combine_ref, dispatch_pack_ref

    dist.init_process_group("gloo", rank=rank, world_size=ws)
    E, H, I, k, T_l = 8, 64, 64, 3, 5
    L = synth.moe_layer_np(seed=21, E=E, H=H, I=I, top_k=k, group=64, zero_points=True, T=ws * T_l)
    x_full = L["x"].astype(np.float32)
    x = torch.from_numpy(x_full[rank * T_l:(rank + 1) * T_l].copy())
    e0, e1 = rank * (E // ws), (rank + 1) * (E // ws)
    res = torch.from_numpy(np.random.default_rng(rank).standard_normal((T_l, H)).astype(np.float32))

    def route_fn(xt, pack):
        w, sel, _ = O.router(xt.numpy(), L["gate_w"], k, True, None, "float32")
        xb = xt.contiguous().view(torch.uint8)
        pack[:, :xb.shape[1]] = xb
        pack[:, xb.shape[1]:xb.shape[1] + 4 * k] = torch.from_numpy(sel.astype(np.int32)).view(torch.uint8)
        pack[:, xb.shape[1] + 4 * k:xb.shape[1] + 8 * k] = torch.from_numpy(w).view(torch.uint8)

    def experts_fn(x_all, sel_all, w_all):
        s = sel_all.numpy()
        w = np.where((s >= e0) & (s < e1), w_all.numpy(), 0.0).astype(np.float32)
        y = O.moe_experts_by_expert(x_all.numpy(), s, w, L["gu_packed"], L["gu_scale"],
                                    L["dn_packed"], L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
        return torch.from_numpy(y)

    out = ep_forward(x, route_fn, lambda r, s, so: dispatch_pack_ref(r, s, so, k, E, ws, 4 * H),
                     experts_fn, lambda b, so, r: combine_ref(b, so, r), k, residual=res)
    w_ref, sel_ref, _ = O.router(x_full, L["gate_w"], k, True, None, "float32")
    ref = O.moe_experts_by_expert(x_full, sel_ref, w_ref, L["gu_packed"], L["gu_scale"],
                                  L["dn_packed"], L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    ref = ref[rank * T_l:(rank + 1) * T_l] + res.numpy()
    err = float(np.abs(out.numpy() - ref).max() / np.abs(ref).max())
    q.put((rank, err, tuple(out.shape)))
    dist.destroy_process_group()


def test_expert_parallel_host_logic_gloo():
    """Two ranks, four experts each: routing, dispatch all-to-all of the rows that need
    each rank's experts, local experts, combine all-to-all of the partial rows, give each
    rank the single-process layer output for its tokens."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=180) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, shape in res:
        assert shape == (5, 64)
        assert err < 1e-5, (rank, err)


# ------------------------------------------------------------------ failure detection
def _ep_leave_worker(rank, ws, port, q):
    """Two ranks run one expert-parallel layer step; rank 1 then leaves (between steps,
    nothing in flight).  Rank 0's next step must fail with an error within the process
    group's timeout instead of hanging."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(ws),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    import datetime
    import time

    import numpy as np
    import torch
    import torch.distributed as dist

    import oracle as O
    from duplex import synth
    from duplex.streaming.ep_moe import ep_forward
    from ep_ref import combine_ref, dispatch_pack_ref

    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=5))
    E, H, I, k, T_l = 8, 64, 64, 3, 4
    L = synth.moe_layer_np(seed=22, E=E, H=H, I=I, top_k=k, group=64, zero_points=True, T=ws * T_l)
    x = torch.from_numpy(L["x"][rank * T_l:(rank + 1) * T_l].astype(np.float32))
    e0, e1 = rank * (E // ws), (rank + 1) * (E // ws)

    def route_fn(xt, pack):
        w, sel, _ = O.router(xt.numpy(), L["gate_w"], k, True, None, "float32")
        xb = xt.contiguous().view(torch.uint8)
        pack[:, :xb.shape[1]] = xb
        pack[:, xb.shape[1]:xb.shape[1] + 4 * k] = torch.from_numpy(sel.astype(np.int32)).view(torch.uint8)
        pack[:, xb.shape[1] + 4 * k:xb.shape[1] + 8 * k] = torch.from_numpy(w).view(torch.uint8)

    def experts_fn(x_all, sel_all, w_all):
        s = sel_all.numpy()
        w = np.where((s >= e0) & (s < e1), w_all.numpy(), 0.0).astype(np.float32)
        return torch.from_numpy(O.moe_experts_by_expert(
            x_all.numpy(), s, w, L["gu_packed"], L["gu_scale"], L["dn_packed"], L["dn_scale"],
            L["gu_zeros"], L["dn_zeros"]))

    def step():
        return ep_forward(x, route_fn, lambda r, s, so: dispatch_pack_ref(r, s, so, k, E, ws, 4 * H),
                          experts_fn, lambda b, so, r: combine_ref(b, so, r), k)

    step()
    if rank == 1:
        q.put((rank, "left", 0.0, ""))
        q.close()
        q.join_thread()           # flush the message before leaving
        os._exit(0)               # leaves between steps, no destroy_process_group
    time.sleep(0.5)
    t0 = time.time()
    try:
        step()
        q.put((rank, "no error", time.time() - t0, ""))
    except Exception as e:       # the peer is gone: the collective fails
        q.put((rank, "error", time.time() - t0, type(e).__name__))
    q.close()
    q.join_thread()
    os._exit(0)


def test_ep_rank_leaving_between_steps_fails_fast():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_ep_leave_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res[1][1] == "left"
    assert res[0][1] == "error", res[0]
    assert res[0][2] < 30.0        # within the 5 s group timeout plus start-up slack


def _hb_worker(rank, ws, port, q):
    """Heartbeat-gated steps: rank 1 leaves after step 1; rank 0 must learn of it on the
    host in ready(2), before launching anything of step 2."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(ws),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    import datetime
    import time

    import torch
    import torch.distributed as dist

    from duplex.health import Heartbeat, PeerLost

    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=30))
    hb = Heartbeat(timeout_s=2.0)
    t = torch.ones(4)
    hb.ready(1)
    dist.all_reduce(t)                 # step 1 of both ranks
    if rank == 1:
        q.put((rank, "left", 0.0, float(t[0])))
        q.close()
        q.join_thread()
        os._exit(0)
    t0 = time.time()
    try:
        hb.ready(2)
        q.put((rank, "no error", time.time() - t0, float(t[0])))
    except PeerLost as e:
        q.put((rank, "peer lost" if "[1]" in str(e) else str(e), time.time() - t0, float(t[0])))
    q.close()
    q.join_thread()
    os._exit(0)


def test_heartbeat_reports_a_rank_that_left_before_the_next_step():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_hb_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res[1][1] == "left" and res[1][3] == 2.0
    assert res[0][1] == "peer lost", res[0]
    assert 1.5 < res[0][2] < 15.0      # the 2 s heartbeat timeout, not the 30 s group one
