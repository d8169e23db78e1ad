"""GPU parity of the clock-path stack (fused qkv, o, MoE per layer, RMSNorm inputs)
against the numpy restatement -- at a small geometry and at the Thinker geometry the
bench times -- plus graph replay, the host-buffer decode call, and the bounded-wait
timeout path of the persistent kernel."""

import numpy as np
import pytest
import torch

from duplex import synth
from oracle.clock_oracle import clock_layer

pytestmark = pytest.mark.gpu


def small_layers(n, seed=3, H=256, q=256, kv=64, E=16, I=128, top_k=4, group=128):
    rng = np.random.Generator(np.random.PCG64(seed))
    out = []
    for l in range(n):
        a = synth.linear_np(rng, q + 2 * kv, H, group, True)
        b = synth.linear_np(rng, H, q, group, True)
        m = synth.moe_layer_np(seed=seed * 100 + l, E=E, H=H, I=I, top_k=top_k, group=group)
        d = dict(qkv_packed=a["packed"], qkv_scale=a["scale"], qkv_zeros=a["zeros"],
                 o_packed=b["packed"], o_scale=b["scale"], o_zeros=b["zeros"])
        for k in ("gate_w", "gu_packed", "gu_scale", "gu_zeros", "dn_packed", "dn_scale",
                  "dn_zeros"):
            d[k] = m[k]
        out.append(d)
    return out


@pytest.mark.parametrize("T", [1, 3, 8])
@pytest.mark.parametrize("fused", [True, False])
def test_clock_stack_vs_oracle(cuda, T, fused):
    from duplex.clock import ClockStack
    layers = small_layers(3)
    st = ClockStack.from_arrays(layers, top_k=4, device=cuda, T=T, fused=fused)
    x = np.random.default_rng(1).standard_normal((T, 256)).astype(np.float16)
    out = torch.zeros(T, 256, device=cuda, dtype=torch.float16)
    st.step_into(torch.from_numpy(x).to(cuda), out)
    h = x.astype(np.float32)
    for d in layers:
        h, _ = clock_layer(h, d, 4)
    y = out.float().cpu().numpy()
    assert np.isfinite(y).all()
    assert np.abs(y - h).max() <= 2e-3 * np.abs(h).max()
    assert st.device_errors() == 0


def test_clock_stack_graph_and_decode(cuda):
    from duplex.clock import ClockStack
    st = ClockStack.synthetic(n_layers=2, seed=0, device=cuda)
    st.capture()
    x = torch.randn(1, 2048, device=cuda, dtype=torch.float16)
    eager = torch.zeros_like(x)
    st.step_into(x, eager)
    xh = x.cpu().pin_memory()
    oh = torch.empty(1, 2048, dtype=torch.float16).pin_memory()
    st.decode(xh, oh)
    torch.cuda.synchronize()
    assert torch.equal(oh, eager.cpu())
    assert torch.isfinite(eager).all()
    assert st.device_errors() == 0


def test_persistent_matches_kernel_chain_thinker_geometry(cuda):
    """The one-launch stack and the 5-kernels-per-layer chain agree at Thinker geometry."""
    from duplex.clock import ClockStack
    a = ClockStack.synthetic(n_layers=3, seed=5, device=cuda, fused=True)
    b = ClockStack(a.layers, fused=False, device=cuda)
    x = torch.randn(1, 2048, device=cuda, dtype=torch.float16,
                    generator=torch.Generator(device=cuda).manual_seed(3))
    ya, yb = torch.zeros_like(x), torch.zeros_like(x)
    a.step_into(x, ya)
    b.step_into(x, yb)
    torch.cuda.synchronize()
    ya, yb = ya.float().cpu().numpy(), yb.float().cpu().numpy()
    assert np.isfinite(ya).all()
    assert np.abs(ya - yb).max() <= 2e-3 * np.abs(yb).max()
    assert a.device_errors() == 0


@pytest.mark.parametrize("T", [1, 4])
def test_moe_chain_vs_oracle(cuda, T):
    """x -> MoE(rms(x)) over three layers in one launch against the numpy oracle
    chained layer by layer (each layer's output rounded to fp16, as on the GPU), and
    one layer of it against the per-layer module call."""
    from duplex.clock import MoEChain
    from duplex.streaming.fused_packed_moe import FusedPackedMoE
    from oracle.clock_oracle import moe_layer, rms_norm
    from oracle.moe_oracle import round_to
    moes, arrays = [], []
    for l in range(3):
        L = synth.moe_layer_np(seed=40 + l, E=32, H=512, I=128, top_k=4, group=128, T=1)
        arrays.append(L)
        t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
        moes.append(FusedPackedMoE.from_stacked(t(L["gate_w"]), t(L["gu_packed"]), t(L["gu_scale"]),
                                                t(L["dn_packed"]), t(L["dn_scale"]), 4,
                                                gu_zeros=t(L["gu_zeros"]), dn_zeros=t(L["dn_zeros"]),
                                                dtype=torch.float16, device=cuda, stack=True))
    x = torch.randn(T, 512, device=cuda, dtype=torch.float16,
                    generator=torch.Generator(device=cuda).manual_seed(7))
    chain = MoEChain(moes, rms_eps=1e-6, residual=False, T=T)
    got = torch.zeros_like(x)
    chain.forward_into(x, got)
    one = MoEChain(moes[:1], rms_eps=1e-6, residual=False, T=T)
    got1 = torch.zeros_like(x)
    one.forward_into(x, got1)
    mod1 = torch.zeros_like(x)
    moes[0].forward_into(x, mod1, rms_eps=1e-6)
    torch.cuda.synchronize()
    h = x.float().cpu().numpy()
    for L in arrays:
        y, _ = moe_layer(rms_norm(h, 1e-6), L, 4)
        h = np.asarray(round_to(y, "float16"), np.float32)
    g = got.float().cpu().numpy()
    assert np.abs(g - h).max() <= 2e-3 * np.abs(h).max()
    g1, m1 = got1.float().cpu().numpy(), mod1.float().cpu().numpy()
    assert np.abs(g1 - m1).max() <= 2e-3 * np.abs(m1).max()
    assert chain.p.device_errors() == 0 and one.p.device_errors() == 0


def thinker_layers(n, seed, moe_only=False):
    """n seeded layers at the Thinker geometry (hidden 2048, q|k|v 5120, o 2048 x 4096,
    128 experts, top-8, inter 768, group 128 with zero points)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = []
    for l in range(n):
        m = synth.moe_layer_np(seed=seed * 100 + l)
        d = {k: m[k] for k in ("gate_w", "gu_packed", "gu_scale", "gu_zeros", "dn_packed",
                               "dn_scale", "dn_zeros")}
        if not moe_only:
            a = synth.linear_np(rng, 5120, 2048, 128, True)
            b = synth.linear_np(rng, 2048, 4096, 128, True)
            d.update(qkv_packed=a["packed"], qkv_scale=a["scale"], qkv_zeros=a["zeros"],
                     o_packed=b["packed"], o_scale=b["scale"], o_zeros=b["zeros"])
        out.append(d)
    return out


@pytest.mark.parametrize("T", [1, 8])
def test_clock_stack_vs_oracle_thinker_geometry(cuda, T):
    """The persistent kernel the bench times, at the Thinker geometry (its fixed-geometry
    inner loops), against the oracle chained layer by layer."""
    from duplex.clock import ClockStack
    layers = thinker_layers(2, seed=11)
    st = ClockStack.from_arrays(layers, top_k=8, device=cuda, T=T, fused=True)
    x = np.random.default_rng(21).standard_normal((T, 2048)).astype(np.float16)
    out = torch.zeros(T, 2048, device=cuda, dtype=torch.float16)
    st.step_into(torch.from_numpy(x).to(cuda), out)
    h = x.astype(np.float32)
    for d in layers:
        h, _ = clock_layer(h, d, 8, threads=8)
    y = out.float().cpu().numpy()
    assert np.isfinite(y).all()
    assert np.abs(y - h).max() <= 2e-3 * np.abs(h).max()
    assert st.device_errors() == 0


@pytest.mark.parametrize("T", [1, 8])
def test_moe_chain_vs_oracle_thinker_geometry(cuda, T):
    """Three config-0 MoE layers (x -> MoE(rms(x))) in one launch against the oracle,
    each layer's output rounded to fp16 as on the GPU."""
    from duplex.clock import MoEChain
    from duplex.streaming.fused_packed_moe import FusedPackedMoE
    from oracle.clock_oracle import moe_layer, rms_norm
    from oracle.moe_oracle import round_to
    arrays = thinker_layers(3, seed=12, moe_only=True)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    moes = [FusedPackedMoE.from_stacked(t(L["gate_w"]), t(L["gu_packed"]), t(L["gu_scale"]),
                                        t(L["dn_packed"]), t(L["dn_scale"]), 8,
                                        gu_zeros=t(L["gu_zeros"]), dn_zeros=t(L["dn_zeros"]),
                                        dtype=torch.float16, device=cuda, stack=True)
            for L in arrays]
    x = torch.randn(T, 2048, device=cuda, dtype=torch.float16,
                    generator=torch.Generator(device=cuda).manual_seed(17))
    chain = MoEChain(moes, rms_eps=1e-6, residual=False, T=T)
    got = torch.zeros_like(x)
    chain.forward_into(x, got)
    again = torch.zeros_like(x)
    chain.forward_into(x, again)
    torch.cuda.synchronize()
    h = x.float().cpu().numpy()
    for L in arrays:
        y, _ = moe_layer(rms_norm(h, 1e-6), L, 8, threads=8)
        h = np.asarray(round_to(y, "float16"), np.float32)
    g = got.float().cpu().numpy()
    assert np.isfinite(g).all()
    assert np.abs(g - h).max() <= 2e-3 * np.abs(h).max()
    assert torch.equal(got, again)          # fixed-order sums: bit-identical launches
    assert chain.p.device_errors() == 0


def test_stack_wait_gives_up_with_status(cuda):
    """A grid barrier that cannot complete (test flag) gives up after its short bound:
    the launch returns, the error word holds DUPLEX_DEVERR_TIMEOUT and the grid-barrier
    site, and the device stays usable (the next launch is correct)."""
    from duplex import _lib
    from duplex.clock import MoEChain
    from duplex.streaming.fused_packed_moe import FusedPackedMoE
    L = synth.moe_layer_np(seed=50, E=32, H=512, I=128, top_k=4, group=128, T=1)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    moes = [FusedPackedMoE.from_stacked(t(L["gate_w"]), t(L["gu_packed"]), t(L["gu_scale"]),
                                        t(L["dn_packed"]), t(L["dn_scale"]), 4,
                                        gu_zeros=t(L["gu_zeros"]), dn_zeros=t(L["dn_zeros"]),
                                        dtype=torch.float16, device=cuda, stack=True)
            for _ in range(2)]
    chain = MoEChain(moes, rms_eps=1e-6, residual=False, T=1)
    x = torch.randn(1, 512, device=cuda, dtype=torch.float16,
                    generator=torch.Generator(device=cuda).manual_seed(3))
    ok = torch.zeros_like(x)
    chain.forward_into(x, ok)
    torch.cuda.synchronize()
    assert chain.p.device_errors() == 0
    bad = torch.zeros_like(x)
    chain.p.run(x, bad, wait_limit_cycles=2_000_000, test_flags=1)   # ~1 ms bound
    torch.cuda.synchronize()
    e = chain.p.device_errors()
    assert e & _lib.DEVERR_TIMEOUT
    assert (e >> 8) & 0xFF == 4                    # site 4: the grid barrier
    again = torch.zeros_like(x)
    chain.forward_into(x, again)
    torch.cuda.synchronize()
    assert chain.p.device_errors() == 0
    assert torch.equal(again, ok)
