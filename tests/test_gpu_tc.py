"""GPU parity of the tensor-core (tcgen05) grouped path: the record repack against a numpy
restatement of the record layout, the whole layer against the oracle at the config-3 batch
sizes, expert shards (expert parallelism), determinism, and agreement with the mma.sync
engine on the same routing."""

import numpy as np
import pytest
import torch

import oracle as O
from duplex import _lib, synth

pytestmark = pytest.mark.gpu


def T(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def tc_records_np(packed, scale, zeros, K, pair_halves):
    """numpy restatement of the tensor-core record layout (csrc/grouped_tc.cuh): per
    (expert, 128-row tile, 128-column chunk) int4 words [piece q][row m][4 words], word
    j = 4 q + i holding values 8 j .. 8 j + 7 with the pair (2 p, 2 p + 1) in the nibbles
    at bits 4 p and 16 + 4 p; then 128 scales; then 128 zero-point bytes (if any)."""
    E, R, _ = packed.shape
    nib = O.unpack_nibbles(packed, K).astype(np.uint32)          # [E, R, K]
    G = K // 128
    z = None if zeros is None else O.unpack_nibbles(zeros, G)     # [E, R, G]
    if pair_halves:
        I = R // 2
        m = np.arange(128)
        rows = [(m >> 4 & 1) * I + 64 * t + 16 * (m >> 5) + (m & 15) for t in range(R // 128)]
    else:
        rows = [128 * t + np.arange(128) for t in range(R // 128)]
    out = []
    for e in range(E):
        for t in range(R // 128):
            r = rows[t]
            for c in range(G):
                v = nib[e][r][:, 128 * c:128 * c + 128].reshape(128, 16, 4, 2)   # [m][j][p][lo/hi]
                words = (v[..., 0] << (4 * np.arange(4))).sum(-1) | (v[..., 1] << (16 + 4 * np.arange(4))).sum(-1)
                words = words.astype(np.uint32).reshape(128, 4, 4).transpose(1, 0, 2)  # [q][m][i]
                out.append(words.reshape(-1).view(np.uint8))
                out.append(np.ascontiguousarray(scale[e][r, c]).view(np.uint8))
                if z is not None:
                    out.append(z[e][r, c].astype(np.uint8))
    return np.concatenate(out)


@pytest.mark.parametrize("pair_halves,zp", [(True, True), (False, True), (True, False)])
def test_tc_records_layout(cuda, pair_halves, zp):
    from duplex.streaming.triton_dequant_gemv import TcRecords
    rng = np.random.default_rng(3)
    E, R, K = 2, 256, 384
    packed = O.pack4(rng.integers(0, 16, (E, R, K)))
    scale = O.round_to(rng.random((E, R, K // 128)) * 0.02 + 0.001, "float16").astype(np.float16)
    zeros = O.pack_zeros(rng.integers(0, 16, (E, R, K // 128))) if zp else None
    rec = TcRecords(T(packed, cuda), T(scale, cuda), None if zeros is None else T(zeros, cuda), group=128,
                    K=K, pair_halves=pair_halves)
    torch.cuda.synchronize()
    ref = tc_records_np(packed, scale, zeros, K, pair_halves)
    assert rec.buf.numel() == ref.size
    assert np.array_equal(rec.buf.cpu().numpy(), ref)


def _layer(cuda, seed, E, H, I, k, Tn, zp=True, dtype=torch.float16):
    from duplex.streaming.fused_packed_moe import FusedPackedMoE
    L = synth.moe_layer_np(seed=seed, E=E, H=H, I=I, top_k=k, group=128, zero_points=zp, T=Tn)
    dn = "float16" if dtype == torch.float16 else "bfloat16"
    x = O.round_to(L["x"].astype(np.float32), dn)
    z = (lambda n: T(L[n], cuda)) if zp else (lambda n: None)
    m = FusedPackedMoE.from_stacked(T(L["gate_w"], cuda, dtype), T(L["gu_packed"], cuda),
                                    T(L["gu_scale"], cuda, dtype), T(L["dn_packed"], cuda),
                                    T(L["dn_scale"], cuda, dtype), k, gu_zeros=z("gu_zeros"),
                                    dn_zeros=z("dn_zeros"), dtype=dtype, tc=True)
    assert m.gu_tc is not None
    return L, m, x


def _run(cuda, m, x, dtype, engine="tc", residual=None):
    Tn = x.shape[0]
    x_t = T(x, cuda, dtype)
    out = torch.empty(Tn, m.hidden, dtype=dtype, device=cuda)
    w = torch.empty(Tn, m.top_k, dtype=torch.float32, device=cuda)
    sel = torch.empty(Tn, m.top_k, dtype=torch.int32, device=cuda)
    m.forward_grouped_into(x_t, out, residual=residual, w_out=w, sel_out=sel, engine=engine)
    torch.cuda.synchronize()
    return out, w, sel


@pytest.mark.parametrize("Tn", [16, 64, 256, 512])
def test_tc_layer_matches_oracle_thinker_geometry(cuda, Tn):
    """Config 3 geometry (128 experts, hidden 2048, inter 768, top-8, g128 + zero points,
    fp16) at 16 / 64 / 256 / 512 streams: 16-, 16-, 32- and 64-token units."""
    L, m, x = _layer(cuda, 70 + Tn, 128, 2048, 768, 8, Tn)
    out, w, sel = _run(cuda, m, x, torch.float16)
    assert int(m.err.item()) == 0
    ref = O.moe_experts_by_expert(x, sel.cpu().numpy(), w.cpu().numpy(), L["gu_packed"], L["gu_scale"],
                                  L["dn_packed"], L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    assert rel_err(out.float().cpu().numpy(), ref) <= 2e-3


def test_tc_layer_bf16_symmetric(cuda):
    L, m, x = _layer(cuda, 81, 128, 2048, 768, 8, 96, zp=False, dtype=torch.bfloat16)
    out, w, sel = _run(cuda, m, x, torch.bfloat16)
    assert int(m.err.item()) == 0
    bf = lambda a: O.round_to(a.astype(np.float32), "bfloat16").astype(np.float32)  # noqa: E731
    ref = O.moe_experts_by_expert(x, sel.cpu().numpy(), w.cpu().numpy(), L["gu_packed"],
                                  bf(L["gu_scale"]), L["dn_packed"], bf(L["dn_scale"]))
    assert rel_err(out.float().cpu().numpy(), ref) <= 8e-3


def test_tc_small_geometry_residual(cuda):
    """32 experts, hidden 512, inter 256, top-4, 100 tokens, + residual."""
    L, m, x = _layer(cuda, 82, 32, 512, 256, 4, 100)
    res = O.round_to(np.random.default_rng(5).standard_normal((100, 512)), "float16")
    out, w, sel = _run(cuda, m, x, torch.float16, residual=T(res, cuda, torch.float16))
    assert int(m.err.item()) == 0
    ref = O.moe_experts_by_expert(x, sel.cpu().numpy(), w.cpu().numpy(), L["gu_packed"], L["gu_scale"],
                                  L["dn_packed"], L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    assert rel_err(out.float().cpu().numpy() - res.astype(np.float32), ref) <= 2e-3


def test_tc_is_deterministic_and_agrees_with_mma_engine(cuda):
    L, m, x = _layer(cuda, 83, 128, 2048, 768, 8, 200)
    a, w, sel = _run(cuda, m, x, torch.float16)
    b, _, _ = _run(cuda, m, x, torch.float16)
    assert torch.equal(a, b)
    c, w2, sel2 = _run(cuda, m, x, torch.float16, engine="mma")
    assert torch.equal(sel, sel2) and torch.equal(w, w2)
    assert rel_err(a.float().cpu().numpy(), c.float().cpu().numpy()) <= 2e-3


@pytest.mark.parametrize("shards", [2, 8])
def test_tc_expert_shards_sum_to_the_layer(cuda, shards):
    from duplex.streaming.triton_dequant_gemv import TcRecords
    L, m, x = _layer(cuda, 84 + shards, 128, 2048, 768, 8, 128)
    out_full, w, sel = _run(cuda, m, x, torch.float16)
    x_t = T(x, cuda, torch.float16)
    Tn, H, I = x.shape[0], 2048, 768
    n_loc = 128 // shards
    total = torch.zeros(Tn, H, dtype=torch.float32, device=cuda)
    for r in range(shards):
        sl = slice(r * n_loc, (r + 1) * n_loc)
        gu = TcRecords(T(L["gu_packed"][sl], cuda), T(L["gu_scale"][sl], cuda, torch.float16),
                       T(L["gu_zeros"][sl], cuda), group=128, K=H, pair_halves=True)
        dn = TcRecords(T(L["dn_packed"][sl], cuda), T(L["dn_scale"][sl], cuda, torch.float16),
                       T(L["dn_zeros"][sl], cuda), group=128, K=I)
        n = _lib.ctypes.c_size_t()
        _lib.call("duplex_moe_experts_grouped_tc_workspace_bytes", Tn, n_loc, 128, H, I, 8, 128, 1,
                  _lib.ctypes.byref(n))
        ws = torch.empty(n.value, dtype=torch.uint8, device=cuda)
        part = torch.empty(Tn, H, dtype=torch.float32, device=cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        _lib.call("duplex_moe_experts_grouped_tc", _lib.ptr(x_t), _lib.DTYPE_F16, Tn, H, _lib.ptr(sel),
                  _lib.ptr(w), 8, 8, r * n_loc, n_loc, 128, H, I, _lib.ptr(gu.buf), _lib.ptr(dn.buf),
                  gu.scale_code, 1, 128, None, _lib.ptr(part), _lib.DTYPE_F32, _lib.ptr(ws), ws.numel(),
                  _lib.ptr(err), _lib.stream_of(x_t))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        total += part
    ref = O.moe_experts_by_expert(x, sel.cpu().numpy(), w.cpu().numpy(), L["gu_packed"], L["gu_scale"],
                                  L["dn_packed"], L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    assert rel_err(total.cpu().numpy(), ref) <= 2e-3
    assert rel_err(total.cpu().numpy(), out_full.float().cpu().numpy()) <= 1e-3


@pytest.mark.parametrize("Tn", [1, 3])
def test_tc_smallest_calls(cuda, Tn):
    """One token and a ragged three: 16-column units almost entirely padding."""
    L, m, x = _layer(cuda, 90 + Tn, 128, 2048, 768, 8, Tn)
    res = O.round_to(np.random.default_rng(Tn).standard_normal((Tn, 2048)), "float16")
    out, w, sel = _run(cuda, m, x, torch.float16, residual=T(res, cuda, torch.float16))
    assert int(m.err.item()) == 0
    ref = O.moe_experts_by_expert(x, sel.cpu().numpy(), w.cpu().numpy(), L["gu_packed"], L["gu_scale"],
                                  L["dn_packed"], L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    assert rel_err(out.float().cpu().numpy() - res.astype(np.float32), ref) <= 2e-3


def test_tc_skewed_routing_splits_experts_into_many_units(cuda):
    """512 tokens that all pick experts 0-7 (router logits given): every selected expert
    holds 512 assignments, split into eight 64-token units, 120 experts idle."""
    L, m, x = _layer(cuda, 95, 128, 2048, 768, 8, 512)
    rng = np.random.default_rng(95)
    lg = rng.standard_normal((512, 128)).astype(np.float32) * 0.1
    lg[:, :8] += 10.0
    lg = O.round_to(lg, "float16").astype(np.float32)
    x_t = T(x, cuda, torch.float16)
    outs = {}
    for eng in ("tc", "mma"):
        out = torch.empty(512, 2048, dtype=torch.float16, device=cuda)
        w = torch.empty(512, 8, dtype=torch.float32, device=cuda)
        sel = torch.empty(512, 8, dtype=torch.int32, device=cuda)
        m.forward_grouped_into(x_t, out, w_out=w, sel_out=sel, logits=T(lg, cuda), engine=eng)
        torch.cuda.synchronize()
        assert int(m.err.item()) == 0
        outs[eng] = (out.float().cpu().numpy(), w.cpu().numpy(), sel.cpu().numpy())
    _, w, sel = outs["tc"]
    assert set(np.unique(sel)) == set(range(8))
    ref = O.moe_experts_by_expert(x, sel, w, L["gu_packed"], L["gu_scale"], L["dn_packed"], L["dn_scale"],
                                  L["gu_zeros"], L["dn_zeros"])
    assert rel_err(outs["tc"][0], ref) <= 2e-3
    assert rel_err(outs["mma"][0], ref) <= 2e-3


def test_tc_experts_read_packed_exchange_rows(cuda):
    """An expert-parallel rank's view: token rows, ids and weights read straight out of
    the exchange rows (row stride > H, meta stride > k) give the same bits as the dense
    inputs."""
    from duplex.streaming.ep_moe import exchange_row_bytes
    L, m, x = _layer(cuda, 97, 128, 2048, 768, 8, 96)
    Tn, H, I = 96, 2048, 768
    x_t = T(x, cuda, torch.float16)
    row = exchange_row_bytes(H, 2, 8)
    pack = torch.zeros(Tn, row, dtype=torch.uint8, device=cuda)
    lws = torch.empty(Tn * 128 * 4, dtype=torch.uint8, device=cuda)
    _lib.call("duplex_moe_route_grouped", _lib.ptr(x_t), _lib.DTYPE_F16, Tn, _lib.ptr(m.gate.weight), None, None,
              128, H, 8, 1, None, None, _lib.ptr(pack), row, _lib.ptr(lws), lws.numel(), None, _lib.stream_of(x_t))
    sel = pack[:, 2 * H:2 * H + 32].contiguous().view(torch.int32)
    w = pack[:, 2 * H + 32:2 * H + 64].contiguous().view(torch.float32)
    n = _lib.ctypes.c_size_t()
    _lib.call("duplex_moe_experts_grouped_tc_workspace_bytes", Tn, 128, 128, H, I, 8, 128, 1, _lib.ctypes.byref(n))
    ws = torch.empty(n.value, dtype=torch.uint8, device=cuda)
    outs = []
    for xp, xs, sp, wp, ms in ((x_t, H, sel, w, 8),
                               (pack, row // 2, pack[:, 2 * H:], pack[:, 2 * H + 32:], row // 4)):
        out = torch.empty(Tn, H, dtype=torch.float32, device=cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        _lib.call("duplex_moe_experts_grouped_tc", _lib.ptr(xp), _lib.DTYPE_F16, Tn, xs, _lib.ptr(sp), _lib.ptr(wp),
                  ms, 8, 0, 128, 128, H, I, _lib.ptr(m.gu_tc.buf), _lib.ptr(m.dn_tc.buf), m.gu_tc.scale_code, 1,
                  128, None, _lib.ptr(out), _lib.DTYPE_F32, _lib.ptr(ws), ws.numel(), _lib.ptr(err),
                  _lib.stream_of(x_t))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    ref = O.moe_experts_by_expert(x, sel.cpu().numpy(), w.cpu().numpy(), L["gu_packed"], L["gu_scale"],
                                  L["dn_packed"], L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    assert rel_err(outs[1].cpu().numpy(), ref) <= 2e-3
