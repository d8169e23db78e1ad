"""GPU parity of the grouped (batched-decode) MoE path, duplex_moe_grouped, against the
numpy oracle: batches of 9 to 512 tokens through one `FusedPackedMoE` layer.

Bars as for the decode path: selected expert ids bit-exact (on exact logits, ties to
the lower id), routing weights to fp32 rounding, layer outputs
max|d| <= 2e-3 * max|y_ref| (fp16) / 8e-3 (bf16) against the fp32 dequant-then-matmul.
"""

import numpy as np
import pytest
import torch

import oracle as O
from duplex import synth

pytestmark = pytest.mark.gpu

TOL = 2e-3
TOL_BF16 = 8e-3
NAMES = {torch.float16: "float16", torch.bfloat16: "bfloat16"}


def T(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


def np_round(a, dt):
    return O.round_to(np.asarray(a, np.float32), NAMES[dt])


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def _case(cuda, seed, E, H, I, k, group, zp, Tn, act):
    from duplex.streaming.fused_packed_moe import FusedPackedMoE
    L = synth.moe_layer_np(seed=seed, E=E, H=H, I=I, top_k=k, group=group, zero_points=zp, T=Tn)
    x = np_round(L["x"], act)
    gw = np_round(L["gate_w"], act)
    gs = np_round(L["gu_scale"].astype(np.float32), act)
    ds = np_round(L["dn_scale"].astype(np.float32), act)
    m = FusedPackedMoE.from_stacked(
        T(gw, cuda, act), T(L["gu_packed"], cuda), T(gs, cuda, act), T(L["dn_packed"], cuda),
        T(ds, cuda, act), k, gu_zeros=None if not zp else T(L["gu_zeros"], cuda),
        dn_zeros=None if not zp else T(L["dn_zeros"], cuda), dtype=act)
    assert m.grouped_supported()
    return L, m, x, gw, gs, ds


def _run(m, x, cuda, act, logits=None, residual=None):
    Tn = x.shape[0]
    xt = T(x, cuda, act)
    out = torch.empty(Tn, m.hidden, dtype=act, device=cuda)
    w = torch.empty(Tn, m.top_k, dtype=torch.float32, device=cuda)
    sel = torch.empty(Tn, m.top_k, dtype=torch.int32, device=cuda)
    m.forward_grouped_into(xt, out, residual=residual, w_out=w, sel_out=sel, logits=logits)
    torch.cuda.synchronize()
    return out, w.cpu().numpy(), sel.cpu().numpy()


def _check_routing(x, gw, k, name, w, sel, max_flip_frac=0.02):
    """Selection against the oracle's router: tokens whose fp16/bf16 logits round the
    same way select the same ids in the same order with the same weights.  A logit
    whose fp32 sum lands on the other side of a rounding boundary than the float64
    one moves that token's softmax by one ulp of the logit (or flips a near-tie);
    at most max_flip_frac of the tokens may differ that way."""
    w_ref, sel_ref, _ = O.router(x, gw, k, True, None, name)
    same = (sel == sel_ref).all(1) & np.isclose(w, w_ref, rtol=2e-6, atol=1e-7).all(1)
    assert (~same).sum() <= max(1, int(max_flip_frac * len(sel))), f"{(~same).sum()} flips"


@pytest.mark.parametrize("Tn", [9, 64, 200])
@pytest.mark.parametrize("group,zp", [(64, False), (128, True)])
@pytest.mark.parametrize("act", [torch.float16, torch.bfloat16])
def test_grouped_small_vs_oracle(cuda, Tn, group, zp, act):
    """16 experts, top-4: at 200 tokens each expert holds ~50 tokens, 3 units."""
    L, m, x, gw, gs, ds = _case(cuda, 300 + Tn, 16, 256, 128, 4, group, zp, Tn, act)
    out, w, sel = _run(m, x, cuda, act)
    _check_routing(x, gw, 4, NAMES[act], w, sel)
    ref = O.moe_experts_by_expert(x, sel, w, L["gu_packed"], gs, L["dn_packed"], ds,
                                  L["gu_zeros"] if zp else None, L["dn_zeros"] if zp else None)
    assert rel_err(out.float().cpu().numpy(), ref) <= (TOL if act == torch.float16 else TOL_BF16)
    assert m.device_errors() == 0


@pytest.mark.parametrize("Tn", [64, 256])
def test_grouped_thinker_geometry_vs_oracle(cuda, Tn):
    """Config 3: 128 experts, hidden 2048, inter 768, top-8, group 128 with zero points,
    fp16, 64 and 256 decode streams."""
    L, m, x, gw, gs, ds = _case(cuda, 7, 128, 2048, 768, 8, 128, True, Tn, torch.float16)
    out, w, sel = _run(m, x, cuda, torch.float16)
    _check_routing(x, gw, 8, "float16", w, sel)
    ref = O.moe_experts_by_expert(x, sel, w, L["gu_packed"], gs, L["dn_packed"], ds,
                                  L["gu_zeros"], L["dn_zeros"])
    assert rel_err(out.float().cpu().numpy(), ref) <= TOL
    assert m.device_errors() == 0


def test_grouped_exact_logits_selection_bit_exact(cuda):
    """Logits on a 1/16 grid with many exact ties, passed in: ids in the oracle's order
    (descending, ties to the lower id) and its weights."""
    E, k, Tn = 64, 8, 96
    L, m, x, gw, gs, ds = _case(cuda, 5, E, 256, 128, k, 64, False, Tn, torch.float16)
    rng = np.random.default_rng(6)
    lg = (rng.integers(-24, 24, size=(Tn, E)) / 16.0).astype(np.float32)
    out, w, sel = _run(m, x, cuda, torch.float16, logits=T(lg, cuda))
    w_ref, sel_ref, _ = O.router(lg, np.eye(E, dtype=np.float32), k, True, None, "float16")
    assert np.array_equal(sel, sel_ref)
    np.testing.assert_allclose(w, w_ref, rtol=2e-6, atol=1e-7)
    ref = O.moe_experts_by_expert(x, sel_ref, w_ref, L["gu_packed"], gs, L["dn_packed"], ds)
    assert rel_err(out.float().cpu().numpy(), ref) <= TOL


def test_grouped_skewed_routing_many_units(cuda):
    """Every token picks experts 0..3: each of them gets 150 tokens = 8 units of <= 20,
    the other experts none."""
    E, k, Tn = 32, 4, 150
    L, m, x, gw, gs, ds = _case(cuda, 8, E, 256, 192, k, 64, True, Tn, torch.float16)
    rng = np.random.default_rng(9)
    lg = rng.uniform(-1, 0, size=(Tn, E)).astype(np.float32)
    lg[:, :k] = 4.0 + rng.uniform(0, 1, size=(Tn, k))
    lg = lg.astype(np.float16).astype(np.float32)       # logits come rounded to fp16
    out, w, sel = _run(m, x, cuda, torch.float16, logits=T(lg, cuda))
    assert set(np.unique(sel)) == set(range(k))
    w_ref, sel_ref, _ = O.router(lg, np.eye(E, dtype=np.float32), k, True, None, "float16")
    assert np.array_equal(sel, sel_ref)
    ref = O.moe_experts_by_expert(x, sel_ref, w_ref, L["gu_packed"], gs, L["dn_packed"], ds,
                                  L["gu_zeros"], L["dn_zeros"])
    assert rel_err(out.float().cpu().numpy(), ref) <= TOL
    assert m.device_errors() == 0


def test_grouped_residual_and_module_forward(cuda):
    """forward() of more than 8 tokens takes the grouped path; the residual is added
    in fp32 before the one rounding."""
    act = torch.float16
    L, m, x, gw, gs, ds = _case(cuda, 11, 16, 256, 128, 4, 128, True, 40, act)
    res = np_round(np.random.default_rng(2).standard_normal((40, 256)), act)
    out, w, sel = _run(m, x, cuda, act, residual=T(res, cuda, act))
    ref = O.moe_experts_by_expert(x, sel, w, L["gu_packed"], gs, L["dn_packed"], ds,
                                  L["gu_zeros"], L["dn_zeros"]) + res
    assert rel_err(out.float().cpu().numpy(), ref) <= TOL
    y = m(T(x, cuda, act).view(2, 20, 256))
    assert y.shape == (2, 20, 256)
    out2, _, _ = _run(m, x, cuda, act)
    assert torch.equal(y.view(40, 256), out2)


def test_grouped_agrees_with_decode_path(cuda):
    """At 8 tokens both paths apply: same routing, outputs within the fp32 order bar."""
    act = torch.float16
    L, m, x, gw, gs, ds = _case(cuda, 12, 128, 2048, 768, 8, 128, True, 8, act)
    out_g, w_g, sel_g = _run(m, x, cuda, act)
    xt = T(x, cuda, act)
    out_d = torch.empty_like(out_g)
    w_d = torch.empty(8, 8, dtype=torch.float32, device=cuda)
    sel_d = torch.empty(8, 8, dtype=torch.int32, device=cuda)
    m.forward_into(xt, out_d, w_out=w_d, sel_out=sel_d)
    torch.cuda.synchronize()
    same = (sel_g == sel_d.cpu().numpy()).all(1)
    assert (~same).sum() <= 1       # the two routers sum the logits in different orders
    np.testing.assert_allclose(w_g[same], w_d.cpu().numpy()[same], rtol=2e-6, atol=1e-7)
    assert rel_err(out_g.float().cpu().numpy()[same], out_d.float().cpu().numpy()[same]) <= 1e-3


def test_grouped_deterministic_and_graph_capture(cuda):
    """Every reduction runs in a fixed order: repeated eager calls and a CUDA-graph
    replay give bit-identical outputs."""
    act = torch.float16
    L, m, x, gw, gs, ds = _case(cuda, 13, 64, 512, 256, 8, 128, True, 128, act)
    xt = T(x, cuda, act)
    a, _, _ = _run(m, x, cuda, act)
    b, _, _ = _run(m, x, cuda, act)
    assert torch.equal(a, b)
    out = torch.empty_like(a)
    m.forward_grouped_into(xt, out)          # workspace allocated before capture
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    out.zero_()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            m.forward_grouped_into(xt, out)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, a)
    assert m.device_errors() == 0
