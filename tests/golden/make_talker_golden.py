"""Golden vectors of the reference's Talker MoE, `FusedMoE.forward`
(src/duplex/streaming/fused_moe.py:40-141), for tests/test_gpu_talker.py.

Run with the reference's package importable, e.g.

    PYTHONPATH=<reference>/src python tests/golden/make_talker_golden.py --out tests/golden

It builds a small Talker-shaped block in the transformers-4 layout the reference
consumes (a ModuleList of experts with gate_proj / up_proj / down_proj Linears, a
shared expert MLP and its sigmoid gate; E 8, hidden 64, inter 32, shared inter 48,
top-2, norm_topk_prob False as the Talker's config), seeded bf16 weights, and records
the reference's forward on the CPU for 3 tokens with q8 off and on (its int8
quantisation included) as bf16 bit patterns.
"""

import argparse
from pathlib import Path
from types import SimpleNamespace as NS

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

E, H, I, S, K, T = 8, 64, 32, 48, 2, 3


class MLP(nn.Module):
    def __init__(self, inter):
        super().__init__()
        self.gate_proj = nn.Linear(H, inter, bias=False)
        self.up_proj = nn.Linear(H, inter, bias=False)
        self.down_proj = nn.Linear(inter, H, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


def block(seed=9):
    g = torch.Generator().manual_seed(seed)
    b = NS(experts=nn.ModuleList([MLP(I) for _ in range(E)]), top_k=K, norm_topk_prob=False,
           gate=nn.Linear(H, E, bias=False), shared_expert=MLP(S),
           shared_expert_gate=nn.Linear(H, 1, bias=False))
    with torch.no_grad():
        for m in [b.gate, b.shared_expert_gate, b.shared_expert] + list(b.experts):
            for p in m.parameters():
                p.copy_(torch.randn(p.shape, generator=g) * 0.08)
    for m in [b.gate, b.shared_expert_gate, b.shared_expert] + list(b.experts):
        m.to(torch.bfloat16)
    return b


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    from duplex.streaming.fused_moe import FusedMoE  # the reference's module
    b = block()
    x = (torch.randn(T, H, generator=torch.Generator().manual_seed(10))).to(torch.bfloat16)
    rec = {"x": bits(x), "gate_w": bits(b.gate.weight.detach()),
           "sh_gate_w": bits(b.shared_expert_gate.weight.detach()),
           "sh_gate": bits(b.shared_expert.gate_proj.weight.detach()),
           "sh_up": bits(b.shared_expert.up_proj.weight.detach()),
           "sh_down": bits(b.shared_expert.down_proj.weight.detach()),
           "gate_up": bits(torch.stack([torch.cat([e.gate_proj.weight, e.up_proj.weight])
                                        for e in b.experts]).detach()),
           "down": bits(torch.stack([e.down_proj.weight for e in b.experts]).detach()),
           "dims": np.array([E, H, I, S, K, T], dtype=np.int64)}
    with torch.no_grad():
        for q8 in (False, True):
            m = FusedMoE(block(), q8=q8)
            rec["y_q8" if q8 else "y"] = bits(m(x.view(1, T, H)).view(T, H))
            if q8:
                rec["gate_up_q8"] = m.gate_up.numpy()
                rec["down_q8"] = m.down.numpy()
                rec["gate_up_s"] = bits(m.gate_up_s.squeeze(-1))
                rec["down_s"] = bits(m.down_s.squeeze(-1))
    out = Path(a.out) / "talker_fused_moe.npz"
    np.savez_compressed(out, **rec)
    print("wrote", out)


if __name__ == "__main__":
    main()
