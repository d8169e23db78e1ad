"""Talker MoE drop-in (duplex.streaming.fused_moe) on the CPU: the int8 quantisation and
the expert stacking against the reference's own FusedMoE (golden vectors made by
tests/golden/make_talker_golden.py from src/duplex/streaming/fused_moe.py:40-141)."""

from types import SimpleNamespace as NS

import numpy as np
import torch
import torch.nn as nn

from conftest import GOLDEN

G = np.load(GOLDEN / "talker_fused_moe.npz")


def bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


class MLP(nn.Module):
    def __init__(self, gate, up, down):
        super().__init__()
        self.gate_proj = nn.Linear(gate.shape[1], gate.shape[0], bias=False)
        self.up_proj = nn.Linear(up.shape[1], up.shape[0], bias=False)
        self.down_proj = nn.Linear(down.shape[1], down.shape[0], bias=False)
        with torch.no_grad():
            self.gate_proj.weight = nn.Parameter(gate.clone())
            self.up_proj.weight = nn.Parameter(up.clone())
            self.down_proj.weight = nn.Parameter(down.clone())


def golden_block():
    """The golden block in the reference's layout (per-expert ModuleList)."""
    E, H, I, S, K, T = (int(v) for v in G["dims"])
    gu, dn = bf16(G["gate_up"]), bf16(G["down"])
    gate = nn.Linear(H, E, bias=False)
    gate.weight = nn.Parameter(bf16(G["gate_w"]).clone())
    sgate = nn.Linear(H, 1, bias=False)
    sgate.weight = nn.Parameter(bf16(G["sh_gate_w"]).clone())
    return NS(experts=nn.ModuleList([MLP(gu[e, :I], gu[e, I:], dn[e]) for e in range(E)]),
              top_k=K, norm_topk_prob=False, gate=gate,
              shared_expert=MLP(bf16(G["sh_gate"]), bf16(G["sh_up"]), bf16(G["sh_down"])),
              shared_expert_gate=sgate)


def test_q8_quantisation_is_the_reference_bit_for_bit():
    from duplex.streaming.fused_moe import FusedMoE
    m = FusedMoE(golden_block(), q8=True)
    assert torch.equal(m.gate_up, torch.from_numpy(G["gate_up_q8"]))
    assert torch.equal(m.down, torch.from_numpy(G["down_q8"]))
    assert torch.equal(m.gate_up_s, bf16(G["gate_up_s"]))
    assert torch.equal(m.down_s, bf16(G["down_s"]))


def test_stacking_is_gate_rows_then_up_rows():
    from duplex.streaming.fused_moe import FusedMoE
    m = FusedMoE(golden_block())
    assert torch.equal(m.gate_up, bf16(G["gate_up"])) and torch.equal(m.down, bf16(G["down"]))
    assert (m.num_experts, m.hidden, m.inter, m.top_k, m.norm_topk_prob) == (8, 64, 32, 2, False)


def test_fuse_moe_blocks_skips_packed_and_takes_transformers_fused_blocks():
    from types import SimpleNamespace
    from duplex.streaming.fused_moe import FusedMoE, fuse_moe_blocks
    from transformers.models.qwen3_omni_moe import modeling_qwen3_omni_moe as tm
    cfg = SimpleNamespace(num_experts=8, hidden_size=64, moe_intermediate_size=32, hidden_act="silu",
                          num_experts_per_tok=2, norm_topk_prob=False,
                          shared_expert_intermediate_size=48, intermediate_size=96)
    tb = tm.Qwen3OmniMoeTalkerTextSparseMoeBlock(cfg)

    class Packed(nn.Module):                     # an int4 block: left to the packed path
        pass
    pb = Packed()
    pb.experts = [SimpleNamespace(gate_proj=SimpleNamespace(weight_packed=1))]
    type(pb).__name__ = "PackedSparseMoeBlock"
    model = nn.Module()
    model.a = tb
    model.b = pb
    n = fuse_moe_blocks(model, verbose=False)
    assert n == 1 and isinstance(model.a, FusedMoE) and model.b is pb
    assert model.a.top_k == 2 and model.a.norm_topk_prob is False and model.a.inter == 32
