"""GPU parity of host-resident layers (the reference's `host_resident=True`,
src/duplex/streaming/fused_packed_moe.py:130-164,233-253): the expert records live in
mapped pinned host memory and every call stages the planned experts into device slots
(duplex_moe_forward_staged).  The expert kernels read the same record bytes as on a
resident layer, so outputs, routing weights and expert ids must be bit-identical to
the resident layer's, and within the layer tolerance of the oracle."""

import numpy as np
import pytest
import torch

import oracle as O
from duplex import synth

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _pair(dev, seed, E, H, I, k, group, zp, T, act=torch.float16):
    """The same seeded layer built GPU-resident and host-resident."""
    from duplex.streaming.fused_packed_moe import FusedPackedMoE
    L = synth.moe_layer_np(seed=seed, E=E, H=H, I=I, top_k=k, group=group, zero_points=zp, T=T)

    def t(a, dt=None):
        if a is None:
            return None
        x = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        return x if dt is None else x.to(dt)

    args = (t(L["gate_w"], act), t(L["gu_packed"]), t(L["gu_scale"], act), t(L["dn_packed"]),
            t(L["dn_scale"], act), k)
    kw = dict(gu_zeros=t(L["gu_zeros"]) if zp else None, dn_zeros=t(L["dn_zeros"]) if zp else None,
              dtype=act, device=dev)
    res = FusedPackedMoE.from_stacked(*args, **kw)
    host = FusedPackedMoE.from_stacked(*args, host_resident=True, **kw)
    return L, res, host, t(L["x"], act)


def _run(m, x, staged):
    T, k = x.shape[0], m.top_k
    out = torch.empty(T, m.hidden, dtype=x.dtype, device=x.device)
    w = torch.empty(T, k, dtype=torch.float32, device=x.device)
    sel = torch.empty(T, k, dtype=torch.int32, device=x.device)
    (m.forward_staged_into if staged else m.forward_into)(x, out, w_out=w, sel_out=sel)
    return out, w, sel


@pytest.mark.parametrize("T", [1, 8])
def test_host_resident_thinker_layer_is_bit_identical_to_resident(cuda, T):
    L, res, host, x = _pair(cuda, 41, 128, 2048, 768, 8, 128, True, T)
    assert host.gu_tiles.buf.numel() == 0 and host.dn_tiles.buf.numel() == 0
    assert host.gu_host.nbytes == res.gu_tiles.buf.numel()
    ref, w_ref, sel_ref = _run(res, x, staged=False)
    for _ in range(2):          # the second call stages over the first call's slots
        got, w, sel = _run(host, x, staged=True)
        torch.cuda.synchronize()
        assert torch.equal(sel, sel_ref)
        assert torch.equal(w, w_ref)
        assert torch.equal(got, ref)
    assert host.device_errors() == 0 and res.device_errors() == 0
    # and the oracle (the reference's gather-bmm restated), within the layer bar
    w_o, sel_o, _ = O.router(L["x"], L["gate_w"], 8, True, None, "float16")
    y_o = O.moe_experts(L["x"], sel_o, w_o, L["gu_packed"], L["gu_scale"], L["dn_packed"],
                        L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    y = got.float().cpu().numpy()
    assert np.abs(y - y_o).max() <= TOL * np.abs(y_o).max()


@pytest.mark.parametrize("T", [3, 13])
def test_host_resident_reference_format_bf16(cuda, T):
    """The reference's own format (group 32, symmetric) in bf16, through forward (13
    tokens: two staged passes of 8 and 5)."""
    _, res, host, x = _pair(cuda, 42, 16, 256, 128, 4, 32, False, T, act=torch.bfloat16)
    assert torch.equal(host(x), res(x))
    assert host.device_errors() == 0


def test_host_resident_layer_under_graph_replay(cuda):
    L, res, host, x = _pair(cuda, 43, 128, 2048, 768, 8, 128, True, 2)
    xin = x.clone()
    out = torch.empty_like(x)
    host.forward_staged_into(xin, out)          # warm: workspace and slots
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            host.forward_staged_into(xin, out)
    torch.cuda.current_stream().wait_stream(s)
    gen = torch.Generator(device=cuda).manual_seed(5)
    for _ in range(3):
        x2 = torch.randn(2, 2048, device=cuda, dtype=torch.float16, generator=gen)
        xin.copy_(x2)
        g.replay()
        ref, _, _ = _run(res, x2, staged=False)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert host.device_errors() == 0


def test_installer_stages_the_layers_past_n_pinned(cuda):
    """fuse_packed_moe_blocks(n_pinned=1): the first block stays GPU resident, the second
    becomes host-resident (reference :278-319), with unchanged outputs."""
    import torch.nn as nn
    from duplex.streaming.fused_packed_moe import fuse_packed_moe_blocks
    E, H, I, k = 8, 256, 64, 2
    Ls = [synth.moe_layer_np(seed=50 + i, E=E, H=H, I=I, top_k=k, group=32, zero_points=False,
                             T=3) for i in range(2)]

    class Lin(nn.Module):
        def __init__(self, p, s, o, i):
            super().__init__()
            self.register_buffer("weight_packed", torch.from_numpy(p))
            self.register_buffer("weight_scale", torch.from_numpy(s))
            self.register_buffer("weight_shape", torch.tensor([o, i]))

    class Exp(nn.Module):
        def __init__(self, L, e):
            super().__init__()
            self.gate_proj = Lin(L["gu_packed"][e, :I].copy(), L["gu_scale"][e, :I].copy(), I, H)
            self.up_proj = Lin(L["gu_packed"][e, I:].copy(), L["gu_scale"][e, I:].copy(), I, H)
            self.down_proj = Lin(L["dn_packed"][e].copy(), L["dn_scale"][e].copy(), H, I)

    class StubSparseMoeBlock(nn.Module):
        def __init__(self, L):
            super().__init__()
            self.experts = nn.ModuleList([Exp(L, e) for e in range(E)])
            self.top_k, self.norm_topk_prob = k, True
            self.gate = nn.Linear(H, E, bias=False)
            with torch.no_grad():
                self.gate.weight.copy_(torch.from_numpy(L["gate_w"].astype(np.float32)))

    def model():
        return nn.Sequential(StubSparseMoeBlock(Ls[0]), StubSparseMoeBlock(Ls[1]))

    a, b = model(), model()
    assert fuse_packed_moe_blocks(a, dtype=torch.float16, device=cuda, verbose=False) == 2
    assert fuse_packed_moe_blocks(b, dtype=torch.float16, device=cuda, n_pinned=1,
                                  verbose=False) == 2
    assert not a[0].host_resident and not a[1].host_resident
    assert not b[0].host_resident and b[1].host_resident
    x = torch.from_numpy(Ls[0]["x"]).to(cuda)
    assert torch.equal(b(x), a(x))
