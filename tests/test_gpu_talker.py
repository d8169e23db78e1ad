"""GPU parity of the Talker MoE kernels (csrc/talker.cu) through the drop-in FusedMoE:

* against the reference's own FusedMoE.forward (golden vectors, bf16 and q8,
  src/duplex/streaming/fused_moe.py:40-141);
* against a torch fp32 restatement of the same op at the Talker geometry (128 experts,
  hidden 1024, inter 384, top-8, a shared expert), T = 1 and 8, bf16 and fp16, with and
  without q8;
* against transformers' own fused-expert Talker block.
Bars: the kernel rounds to the act dtype after each step as the reference does, so the
output differs from fp32 by a few roundings of the act dtype: 2e-2 max|y| for bf16
(8 bits of mantissa), 4e-3 for fp16."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from test_talker_moe import G, bf16, golden_block

pytestmark = pytest.mark.gpu

BAR = {torch.bfloat16: 2e-2, torch.float16: 4e-3}


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max())


def to_dev(block, dev):
    for m in [block.gate, block.shared_expert_gate, block.shared_expert] + list(block.experts):
        m.to(dev)
    return block


@pytest.mark.parametrize("q8", [False, True])
def test_talker_vs_reference_golden(cuda, q8):
    from duplex.streaming.fused_moe import FusedMoE
    m = FusedMoE(to_dev(golden_block(), cuda), q8=q8).to(cuda)
    T, H = int(G["dims"][5]), int(G["dims"][1])
    x = bf16(G["x"]).to(cuda)
    y = m(x.view(1, T, H)).view(T, H)
    ref = bf16(G["y_q8" if q8 else "y"])
    assert rel(y, ref) <= BAR[torch.bfloat16], rel(y, ref)
    assert m.device_errors() == 0


def fp32_talker(x, gate_w, gate_up, down, gu_s, dn_s, shg, shu, shd, sgw, k, norm):
    """The op in fp32, no intermediate rounding (weights dequantised as round(q s))."""
    dt = x.dtype
    if gu_s is not None:
        gate_up = (gate_up.to(dt) * gu_s[..., None]).float()
        down = (down.to(dt) * dn_s[..., None]).float()
    x, gate_up, down = x.float(), gate_up.float(), down.float()
    logits = (x @ gate_w.float().T).to(dt).float()
    p = torch.softmax(logits, dim=-1)
    w, sel = torch.topk(p, k, dim=-1)
    if norm:
        w = w / w.sum(-1, keepdim=True)
    I = gate_up.shape[1] // 2
    out = torch.zeros_like(x)
    for t in range(x.shape[0]):
        for j in range(k):
            e = int(sel[t, j])
            h = gate_up[e] @ x[t]
            a = F.silu(h[:I]) * h[I:]
            out[t] += w[t, j] * (down[e] @ a)
    if shg is not None:
        sh = shd.float() @ (F.silu(shg.float() @ x.T) * (shu.float() @ x.T))
        out += torch.sigmoid(x @ sgw.float().T) * sh.T
    return out


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T", [1, 8])
@pytest.mark.parametrize("q8", [False, True])
def test_talker_geometry_vs_fp32(cuda, dt, T, q8):
    from duplex.streaming.fused_moe import quantize_q8
    from duplex import _lib
    E, H, I, S, k = 128, 1024, 384, 768, 8
    g = torch.Generator(device=cuda).manual_seed(T * 7 + q8)
    r = lambda *s, sc=0.04: (torch.randn(*s, generator=g, device=cuda) * sc).to(dt)  # noqa: E731
    x, gate_w = r(T, H, sc=1.0), r(E, H, sc=0.03)
    gate_up, down = r(E, 2 * I, H), r(E, H, I)
    shg, shu, shd, sgw = r(S, H), r(S, H), r(H, S), r(1, H)
    gu_s = dn_s = None
    if q8:
        gate_up, gu_s = quantize_q8(gate_up)
        down, dn_s = quantize_q8(down)
    n = _lib.ctypes.c_size_t()
    _lib.call("duplex_talker_moe_workspace_bytes", T, E, H, I, k, S, _lib.ctypes.byref(n))
    ws = torch.zeros(n.value, dtype=torch.uint8, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.empty(T, H, dtype=dt, device=cuda)
    sel = torch.empty(T, k, dtype=torch.int32, device=cuda)
    for _ in range(2):   # the second call reuses the workspace: same bits
        _lib.call("duplex_talker_moe_forward", _lib.ptr(x), _lib.dtype_code(dt), T, _lib.ptr(gate_w),
                  E, H, I, k, 0, _lib.ptr(gate_up), _lib.ptr(down), 1 if q8 else 0, _lib.ptr(gu_s),
                  _lib.ptr(dn_s), _lib.ptr(shg), _lib.ptr(shu), _lib.ptr(shd), S, _lib.ptr(sgw),
                  _lib.ptr(out), None, _lib.ptr(sel), _lib.ptr(ws), ws.numel(), _lib.ptr(err),
                  _lib.stream_of(x))
        torch.cuda.synchronize()
        if _ == 0:
            first = out.clone()
    assert torch.equal(first, out)
    ref = fp32_talker(x, gate_w, gate_up, down, gu_s, dn_s, shg, shu, shd, sgw, k, False)
    assert rel(out, ref) <= BAR[dt], rel(out, ref)
    # the selection: logits rounded to the act dtype, larger first, ties to the lower id
    lg = (x.float() @ gate_w.float().T).to(dt).float()
    want = torch.argsort(-lg, dim=-1, stable=True)[:, :k]
    assert torch.equal(sel.long().cpu(), want.cpu())
    assert int(err.item()) == 0


def test_transformers_talker_block_vs_its_own_forward(cuda):
    from duplex.streaming.fused_moe import fuse_moe_blocks
    from transformers.models.qwen3_omni_moe import modeling_qwen3_omni_moe as tm
    from transformers.models.qwen3_omni_moe.configuration_qwen3_omni_moe import (
        Qwen3OmniMoeTalkerTextConfig)
    cfg = Qwen3OmniMoeTalkerTextConfig(num_experts=32, hidden_size=256, moe_intermediate_size=128,
                                       num_experts_per_tok=4, norm_topk_prob=False,
                                       intermediate_size=512, num_hidden_layers=1,
                                       num_attention_heads=4, num_key_value_heads=2)
    cfg.shared_expert_intermediate_size = 192
    torch.manual_seed(3)
    blk = tm.Qwen3OmniMoeTalkerTextSparseMoeBlock(cfg)
    with torch.no_grad():
        for p in blk.parameters():
            p.copy_(torch.randn(p.shape) * 0.05)
    blk = blk.to(cuda, torch.float32)
    x = torch.randn(1, 5, 256, device=cuda)
    with torch.no_grad():
        ref = blk(x)
    model = torch.nn.Module()
    model.mlp = blk.to(torch.float16)
    assert fuse_moe_blocks(model, verbose=False) == 1
    y = model.mlp(x.half())
    assert rel(y, ref) <= BAR[torch.float16], rel(y, ref)
