"""GPU checks of the expert-parallel pieces: duplex_moe_experts_grouped on expert shards
(partial sums over shards = the whole layer), the route-only entry point, and the
ExpertParallelMoE module over NCCL (one rank here; two ranks when two GPUs are present).
"""

import os
import socket

import numpy as np
import pytest
import torch

import oracle as O
from duplex import _lib, synth

pytestmark = pytest.mark.gpu

TOL = 2e-3


def T(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def _layer(cuda, seed, E, H, I, k, Tn, group=128):
    from duplex.streaming.fused_packed_moe import FusedPackedMoE
    L = synth.moe_layer_np(seed=seed, E=E, H=H, I=I, top_k=k, group=group, zero_points=True, T=Tn)
    x = O.round_to(L["x"].astype(np.float32), "float16")
    m = FusedPackedMoE.from_stacked(T(L["gate_w"], cuda), T(L["gu_packed"], cuda), T(L["gu_scale"], cuda),
                                    T(L["dn_packed"], cuda), T(L["dn_scale"], cuda), k,
                                    gu_zeros=T(L["gu_zeros"], cuda), dn_zeros=T(L["dn_zeros"], cuda),
                                    dtype=torch.float16)
    return L, m, x


def _shard_partial(cuda, L, m, x_t, sel, w, e0, n_loc, out_dtype=torch.float32, residual=None):
    from duplex.streaming.triton_dequant_gemv import Int4Tiles
    sl = slice(e0, e0 + n_loc)
    H = x_t.shape[1]
    gu = Int4Tiles(T(L["gu_packed"][sl], cuda), T(L["gu_scale"][sl], cuda, torch.float16),
                   T(L["gu_zeros"][sl], cuda), group=m.group, K=H, pair_halves=True)
    dn = Int4Tiles(T(L["dn_packed"][sl], cuda), T(L["dn_scale"][sl], cuda, torch.float16),
                   T(L["dn_zeros"][sl], cuda), group=m.group, K=m.inter)
    Tn, k = sel.shape
    n = _lib.ctypes.c_size_t()
    _lib.call("duplex_moe_experts_grouped_workspace_bytes", Tn, n_loc, m.num_experts, H, m.inter, k,
              m.group, 1, _lib.ctypes.byref(n))
    ws = torch.empty(n.value, dtype=torch.uint8, device=cuda)
    out = torch.empty(Tn, H, dtype=out_dtype, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.call("duplex_moe_experts_grouped", _lib.ptr(x_t), _lib.DTYPE_F16, Tn, H, _lib.ptr(sel),
              _lib.ptr(w), k, k, e0, n_loc, m.num_experts, H, m.inter, _lib.ptr(gu.buf),
              _lib.ptr(dn.buf), gu.scale_code, 1,
              m.group, _lib.ptr(residual), _lib.ptr(out), _lib.dtype_code(out_dtype), _lib.ptr(ws),
              ws.numel(), _lib.ptr(err), _lib.stream_of(x_t))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


@pytest.mark.parametrize("shards", [2, 4, 8])
def test_expert_shards_sum_to_the_layer(cuda, shards):
    """Config 4 geometry (128 experts, top-8): the fp32 partial sums of `shards`
    expert shards, added in rank order, give the whole layer."""
    L, m, x = _layer(cuda, 40 + shards, 128, 2048, 768, 8, 64)
    x_t = T(x, cuda, torch.float16)
    Tn = x.shape[0]
    out_full = torch.empty(Tn, 2048, dtype=torch.float16, device=cuda)
    w = torch.empty(Tn, 8, dtype=torch.float32, device=cuda)
    sel = torch.empty(Tn, 8, dtype=torch.int32, device=cuda)
    m.forward_grouped_into(x_t, out_full, w_out=w, sel_out=sel)
    total = torch.zeros(Tn, 2048, dtype=torch.float32, device=cuda)
    n_loc = 128 // shards
    for r in range(shards):
        total += _shard_partial(cuda, L, m, x_t, sel, w, r * n_loc, n_loc)
    ref = O.moe_experts_by_expert(x, sel.cpu().numpy(), w.cpu().numpy(), L["gu_packed"], L["gu_scale"],
                                  L["dn_packed"], L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    assert rel_err(total.cpu().numpy(), ref) <= TOL
    assert rel_err(total.cpu().numpy(), out_full.float().cpu().numpy()) <= 1e-3


def test_all_local_shard_is_the_grouped_layer_bit_for_bit(cuda):
    """One shard holding every expert, fp16 out + residual: the same kernels in the same
    order as duplex_moe_grouped, so the same bits."""
    L, m, x = _layer(cuda, 50, 32, 512, 256, 4, 100)
    x_t = T(x, cuda, torch.float16)
    Tn = x.shape[0]
    res = T(O.round_to(np.random.default_rng(3).standard_normal((Tn, 512)), "float16"), cuda, torch.float16)
    out_full = torch.empty(Tn, 512, dtype=torch.float16, device=cuda)
    w = torch.empty(Tn, 4, dtype=torch.float32, device=cuda)
    sel = torch.empty(Tn, 4, dtype=torch.int32, device=cuda)
    m.forward_grouped_into(x_t, out_full, residual=res, w_out=w, sel_out=sel)
    torch.cuda.synchronize()
    out = _shard_partial(cuda, L, m, x_t, sel, w, 0, 32, out_dtype=torch.float16, residual=res)
    assert torch.equal(out, out_full)


def test_route_grouped_matches_the_grouped_layer_routing(cuda):
    L, m, x = _layer(cuda, 51, 128, 2048, 768, 8, 200)
    x_t = T(x, cuda, torch.float16)
    Tn = x.shape[0]
    out_full = torch.empty(Tn, 2048, dtype=torch.float16, device=cuda)
    w = torch.empty(Tn, 8, dtype=torch.float32, device=cuda)
    sel = torch.empty(Tn, 8, dtype=torch.int32, device=cuda)
    m.forward_grouped_into(x_t, out_full, w_out=w, sel_out=sel)
    w2 = torch.empty_like(w)
    sel2 = torch.empty_like(sel)
    ws = torch.empty(Tn * 128 * 4, dtype=torch.uint8, device=cuda)
    g = m.gate
    _lib.call("duplex_moe_route_grouped", _lib.ptr(x_t), _lib.DTYPE_F16, Tn, _lib.ptr(g.weight), None, None,
              128, 2048, 8, 1, _lib.ptr(w2), _lib.ptr(sel2), None, 0, _lib.ptr(ws), ws.numel(), None,
              _lib.stream_of(x_t))
    torch.cuda.synchronize()
    assert torch.equal(sel, sel2) and torch.equal(w, w2)
    # the exchange rows: token bytes, ids, weights
    from duplex.streaming.ep_moe import exchange_row_bytes
    row = exchange_row_bytes(2048, 2, 8)
    pack = torch.zeros(Tn, row, dtype=torch.uint8, device=cuda)
    _lib.call("duplex_moe_route_grouped", _lib.ptr(x_t), _lib.DTYPE_F16, Tn, _lib.ptr(g.weight), None, None,
              128, 2048, 8, 1, None, None, _lib.ptr(pack), row, _lib.ptr(ws), ws.numel(), None,
              _lib.stream_of(x_t))
    torch.cuda.synchronize()
    assert torch.equal(pack[:, :4096].view(torch.float16), x_t)
    assert torch.equal(pack[:, 4096:4128].view(torch.int32), sel)
    assert torch.equal(pack[:, 4128:4160].view(torch.float32), w)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ep_rank(rank, world, port, q, T_l):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from duplex.streaming.ep_moe import ExpertParallelMoE
    from duplex.streaming.fused_packed_moe import FusedPackedMoE
    from duplex import benchutil as bu
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    os.environ.update(WORLD_SIZE=str(world), RANK=str(rank), LOCAL_RANK=str(rank))
    bu.init_nccl(dev, timeout_s=60)
    L = synth.moe_layer_np(seed=60, E=128, H=2048, I=768, top_k=8, group=128, zero_points=True,
                           T=world * T_l)
    x_full = O.round_to(L["x"].astype(np.float32), "float16")
    args = [T(L[n], dev) for n in ("gate_w", "gu_packed", "gu_scale", "dn_packed", "dn_scale")]
    ep = ExpertParallelMoE(*args, 8, gu_zeros=T(L["gu_zeros"], dev), dn_zeros=T(L["dn_zeros"], dev),
                           dtype=torch.float16, device=dev)
    x = T(x_full[rank * T_l:(rank + 1) * T_l], dev, torch.float16)
    y = ep(x)
    y2 = ep(x)                      # second call: reused buffers, same bits
    torch.cuda.synchronize()
    full = FusedPackedMoE.from_stacked(*args, 8, gu_zeros=T(L["gu_zeros"], dev), dn_zeros=T(L["dn_zeros"], dev),
                                       dtype=torch.float16, device=dev)
    y_ref = torch.empty(world * T_l, 2048, dtype=torch.float16, device=dev)
    w = torch.empty(world * T_l, 8, dtype=torch.float32, device=dev)
    sel = torch.empty(world * T_l, 8, dtype=torch.int32, device=dev)
    full.forward_grouped_into(T(x_full, dev, torch.float16), y_ref, w_out=w, sel_out=sel)
    torch.cuda.synchronize()
    mine = slice(rank * T_l, (rank + 1) * T_l)
    err = rel_err(y.float().cpu().numpy(), y_ref[mine].float().cpu().numpy())
    # the oracle: the reference's gather-bmm restated, on the routing of the same tokens
    ref = O.moe_experts_by_expert(x_full[mine], sel[mine].cpu().numpy(), w[mine].cpu().numpy(),
                                  L["gu_packed"], L["gu_scale"], L["dn_packed"], L["dn_scale"],
                                  L["gu_zeros"], L["dn_zeros"])
    oerr = rel_err(y.float().cpu().numpy(), ref)
    q.put((rank, err, ep.device_errors(), oerr, bool(torch.equal(y, y2))))
    dist.barrier()
    dist.destroy_process_group()


def _run_ranks(world, T_l):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_ep_rank, args=(r, world, port, q, T_l)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("T_l", [64, 256])
def test_expert_parallel_module_one_rank(cuda, T_l):
    """NCCL group of one: the all-to-alls degenerate to copies; the output equals the
    single-GPU grouped layer (fp32 summation-order bar) and the oracle (2e-3)."""
    for rank, err, derr, oerr, same in _run_ranks(1, T_l):
        assert err <= 1e-3 and oerr <= TOL and derr == 0 and same


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_module_two_ranks(cuda):
    """Two GPUs, 64 experts each, 32 streams per rank, dispatch / combine all-to-alls over
    NCCL (no multicast loads anywhere), against the oracle."""
    for rank, err, derr, oerr, same in _run_ranks(2, 32):
        assert err <= 1e-3 and oerr <= TOL and derr == 0 and same


def _peer_rank(rank, world, port, q):
    """The NVLink peer exchange against the NCCL all-to-alls on the same weights and
    tokens: bit-identical outputs, eagerly (three calls) and in a CUDA graph replayed."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      WORLD_SIZE=str(world), RANK=str(rank), LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from duplex import benchutil as bu
    from duplex.streaming.ep_moe import ExpertParallelMoE
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    bu.init_nccl(dev, timeout_s=60)
    L = synth.moe_layer_np(seed=62, E=128, H=2048, I=768, top_k=8, group=128, zero_points=True,
                           T=world * 32)
    args = [T(L[n], dev) for n in ("gate_w", "gu_packed", "gu_scale", "dn_packed", "dn_scale")]
    kw = dict(gu_zeros=T(L["gu_zeros"], dev), dn_zeros=T(L["dn_zeros"], dev), dtype=torch.float16,
              device=dev)
    ref = ExpertParallelMoE(*args, 8, **kw)
    mods = [ExpertParallelMoE(*args, 8, exchange="peer", **kw) for _ in range(2)]
    x = T(L["x"][rank * 32:(rank + 1) * 32], dev, torch.float16)
    res = T(np.random.default_rng(rank).standard_normal((32, 2048)).astype(np.float16), dev)
    want = ref(x, residual=res)
    eager = [mods[0](x, residual=res) for _ in range(3)]
    ok_eager = all(bool(torch.equal(y, want)) for y in eager)
    outs = [None, None]

    def step():   # two peer layers back to back, as in the bench
        outs[0] = mods[0](x, residual=res)
        outs[1] = mods[1](outs[0])
    s_ = torch.cuda.Stream(dev)
    s_.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s_):
        step()
    torch.cuda.current_stream(dev).wait_stream(s_)
    torch.cuda.synchronize()
    want1 = ref(want)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s_, capture_error_mode="thread_local"):
        step()
    ok_graph = True
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        ok_graph &= bool(torch.equal(outs[0], want)) and bool(torch.equal(outs[1], want1))
    derr = sum(m.device_errors() for m in mods)
    del g
    for m in mods:
        m.close()
    q.put((rank, ok_eager, ok_graph, derr))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_exchange_matches_the_nccl_all_to_alls(cuda, world):
    """world GPUs (skipped on a smaller box), 128 / world experts and 32 streams each."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_peer_rank, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ok_eager, ok_graph, derr in res:
        assert ok_eager and ok_graph and derr == 0, (rank, ok_eager, ok_graph, derr)


def _leave_rank(rank, world, port, q):
    """Heartbeat-gated expert-parallel steps on `world` GPUs; the last rank leaves after
    step 1 has completed (nothing of it in flight).  The others must raise PeerLost in
    ready(2), on the host, before launching any kernel or collective of step 2."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      WORLD_SIZE=str(world), RANK=str(rank), LOCAL_RANK=str(rank))
    import time

    from duplex import benchutil as bu
    from duplex.health import Heartbeat, PeerLost, abort_group, guard_step
    from duplex.streaming.ep_moe import ExpertParallelMoE
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    bu.init_nccl(dev, timeout_s=60)
    L = synth.moe_layer_np(seed=61, E=128, H=2048, I=768, top_k=8, group=128, zero_points=True,
                           T=world * 32)
    args = [T(L[n], dev) for n in ("gate_w", "gu_packed", "gu_scale", "dn_packed", "dn_scale")]
    ep = ExpertParallelMoE(*args, 8, gu_zeros=T(L["gu_zeros"], dev), dn_zeros=T(L["dn_zeros"], dev),
                           dtype=torch.float16, device=dev)
    x = T(L["x"][rank * 32:(rank + 1) * 32], dev, torch.float16)
    hb = Heartbeat(timeout_s=3.0)
    hb.ready(1)
    ep(x)
    guard_step(60.0)                     # step 1 complete on this rank
    if rank == world - 1:
        q.put((rank, "left", 0.0))
        q.close()
        q.join_thread()
        os._exit(0)
    t0 = time.time()
    try:
        hb.ready(2)
        ep(x)
        guard_step(60.0)
        res = "no error"
    except PeerLost:
        res = "peer lost"
    q.put((rank, res, time.time() - t0))
    q.close()
    q.join_thread()
    abort_group()                        # nothing in flight: the communicator just goes
    os._exit(0)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_rank_leaving_is_seen_on_the_host_before_the_next_step(cuda):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_leave_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=120)
    assert res[1][1] == "left"
    assert res[0][1] == "peer lost" and res[0][2] < 20.0, res[0]


def _guard_rank(q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()), WORLD_SIZE="1",
                      RANK="0", LOCAL_RANK="0")
    from duplex import benchutil as bu
    from duplex.health import StepTimeout, guard_step
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    bu.init_nccl(dev, timeout_s=60)
    torch.cuda._sleep(2_000_000_000)     # a slow step: ~1 s of clock64 spinning, then it ends
    try:
        guard_step(0.2)
        res = "no timeout"
    except StepTimeout:
        res = "timeout"
    torch.cuda.synchronize()             # the sleep kernel still finishes on its own
    ok = float(torch.ones(2, device=dev).sum()) == 2.0
    q.put((res, ok))
    q.close()
    q.join_thread()
    os._exit(0)


def test_guard_step_times_out_on_the_host_and_aborts_the_group(cuda):
    """A step that outlives the host timeout (a bounded sleep kernel, no fault) raises
    StepTimeout and aborts the group; the device context stays usable."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_guard_rank, args=(q,))
    p.start()
    res, ok = q.get(timeout=300)
    p.join(timeout=60)
    assert res == "timeout" and ok


@pytest.mark.parametrize("N", [1, 2, 4, 8])
def test_dispatch_pack_and_combine_kernels(cuda, N):
    """duplex_ep_dispatch_pack / duplex_ep_combine against their torch restatements:
    rows, slots and padding bit for bit; the combine within fp32 order (same order)."""
    from ep_ref import combine_ref, dispatch_pack_ref
    from duplex.streaming.ep_moe import exchange_row_bytes
    E, H, k, T_l = 128, 2048, 8, 48
    rng = np.random.default_rng(N)
    row = exchange_row_bytes(H, 2, k)
    rows = torch.from_numpy(rng.integers(0, 255, (T_l, row), dtype=np.uint8))
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T_l)]).astype(np.int32)
    rows[:, 2 * H:2 * H + 4 * k] = torch.from_numpy(ids).view(torch.uint8)
    rows[:, 2 * H + 4 * k:2 * H + 8 * k] = torch.from_numpy(
        rng.random((T_l, k), dtype=np.float32)).view(torch.uint8)
    send_ref = torch.zeros(N, T_l, row, dtype=torch.uint8)
    slot_ref = torch.empty(N, T_l, dtype=torch.int32)
    dispatch_pack_ref(rows, send_ref, slot_ref, k, E, N, 2 * H)
    rows_d = rows.to(cuda)
    send = torch.zeros(N, T_l, row, dtype=torch.uint8, device=cuda)
    slot = torch.empty(N, T_l, dtype=torch.int32, device=cuda)
    _lib.call("duplex_ep_dispatch_pack", _lib.ptr(rows_d), row, T_l, k, E, N, 2 * H, _lib.ptr(send),
              _lib.ptr(slot), _lib.stream_of(rows_d))
    torch.cuda.synchronize()
    assert torch.equal(slot.cpu(), slot_ref)
    assert torch.equal(send.cpu(), send_ref)          # padding rows included
    back = torch.from_numpy(rng.standard_normal((N, T_l, H)).astype(np.float32))
    res = torch.from_numpy(rng.standard_normal((T_l, H)).astype(np.float16))
    out = torch.empty(T_l, H, dtype=torch.float16, device=cuda)
    back_d, res_d = back.to(cuda), res.to(cuda)   # held until the kernel has run
    _lib.call("duplex_ep_combine", _lib.ptr(back_d), _lib.ptr(slot), T_l, N, H,
              _lib.ptr(res_d), _lib.ptr(out), _lib.DTYPE_F16, _lib.stream_of(out))
    torch.cuda.synchronize()
    ref = combine_ref(back, slot_ref, res.float()).to(torch.float16)
    assert torch.equal(out.cpu(), ref)
