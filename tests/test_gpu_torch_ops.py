"""The TORCH_LIBRARY(duplex_b200) ops on the GPU against the oracle (they call the same
C entry points as the reference-named Python modules)."""

import numpy as np
import pytest
import torch

import oracle as O
from duplex import _lib, synth

pytestmark = pytest.mark.gpu


def test_torch_ops_match_the_oracle(cuda):
    from duplex.streaming.fused_packed_moe import FusedPackedMoE
    from duplex.streaming.triton_dequant_gemv import Int4Tiles
    ops = _lib.load_torch_ops()
    L = synth.moe_layer_np(seed=71, E=16, H=512, I=256, top_k=4, group=128, zero_points=True, T=3)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    # unpack4 and dequant: bit-exact
    up = ops.unpack4(t(L["gu_packed"][2]), 512)
    assert torch.equal(up.cpu(), torch.from_numpy(O.unpack4(L["gu_packed"][2], 512).astype(np.int32)))
    dq = ops.dequant(t(L["gu_packed"][2]), t(L["gu_scale"][2]), t(L["gu_zeros"][2]), 512, torch.float32)
    ref = O.dequant(L["gu_packed"][2], L["gu_scale"][2].astype(np.float32), 512, L["gu_zeros"][2],
                    "float32")
    assert np.array_equal(dq.cpu().numpy(), ref)
    # dequant_gemv over tile records
    tiles = Int4Tiles(t(L["gu_packed"]), t(L["gu_scale"]), t(L["gu_zeros"]), group=128, K=512)
    sel = torch.tensor([3, 9], dtype=torch.int32, device=cuda)
    x = t(L["x"][0])
    y = ops.dequant_gemv(x, tiles.buf, 16, 512, 512, 128, True, torch.float16, sel)
    yr = O.dequant_gemv(L["x"][0], L["gu_packed"], L["gu_scale"], [3, 9], L["gu_zeros"])
    assert np.abs(y.cpu().numpy() - yr).max() <= 2e-5 * np.abs(yr).max()
    # the whole decode MoE layer = the module's forward, bit for bit
    m = FusedPackedMoE.from_stacked(t(L["gate_w"]), t(L["gu_packed"]), t(L["gu_scale"]),
                                    t(L["dn_packed"]), t(L["dn_scale"]), 4, gu_zeros=t(L["gu_zeros"]),
                                    dn_zeros=t(L["dn_zeros"]), dtype=torch.float16, device=cuda)
    xs = t(L["x"])
    ws = m.workspace(3, cuda)
    out = ops.moe_forward(xs, m.gate.weight.detach(), None, m.gu_tiles.buf, m.dn_tiles.buf, 256, 4, True, 128,
                          True, ws, m.err, None, 0.0)
    ref_mod = torch.empty_like(xs)
    m.forward_into(xs, ref_mod)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_mod)
    w, selr, _ = O.router(L["x"], L["gate_w"], 4, True, None, "float16")
    yref = O.moe_experts(L["x"], selr, w, L["gu_packed"], L["gu_scale"], L["dn_packed"],
                         L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    assert np.abs(out.float().cpu().numpy() - yref).max() <= 2e-3 * np.abs(yref).max()
    assert m.device_errors() == 0


def test_route_and_talker_ops(cuda):
    """torch.ops.duplex_b200.moe_route against the oracle's router (same ids and weights,
    a token on a rounding boundary excepted), and talker_moe equal, bit for bit, to the
    module's forward."""
    import torch
    from duplex import _lib
    from duplex.streaming.fused_moe import FusedMoE
    from test_talker_moe import golden_block
    from test_gpu_talker import to_dev
    ops = torch.ops.duplex_b200
    L = synth.moe_layer_np(seed=31, T=4)
    x = torch.from_numpy(L["x"]).to(cuda)
    n = _lib.ctypes.c_size_t()
    _lib.call("duplex_moe_workspace_bytes", 4, 128, 2048, 768, 8, _lib.ctypes.byref(n))
    ws = torch.zeros(n.value, dtype=torch.uint8, device=cuda)
    w, sel = ops.moe_route(x, torch.from_numpy(L["gate_w"]).to(cuda), None, 8, True, ws)
    wr, selr, _ = O.router(L["x"], L["gate_w"], 8, True, None, "float16")
    same = [np.array_equal(a, b) for a, b in zip(sel.cpu().numpy(), selr)]
    assert sum(same) >= len(same) - 1      # a logit on a rounding boundary may flip one token
    for t in np.flatnonzero(same):
        assert np.abs(w.cpu().numpy()[t] - wr[t]).max() <= 1e-6
    m = FusedMoE(to_dev(golden_block(), cuda)).to(cuda)
    xt = torch.randn(3, m.hidden, device=cuda).to(torch.bfloat16)
    ref = m(xt)
    se = m.shared_expert
    out = ops.talker_moe(xt, m.gate.weight.detach(), m.gate_up, m.down, None, None, m.top_k,
                         m.norm_topk_prob, se.gate_proj.weight.detach(), se.up_proj.weight.detach(),
                         se.down_proj.weight.detach(), m.shared_expert_gate.weight.detach(),
                         m._workspace(3, cuda), m.err)
    assert torch.equal(out, ref)
