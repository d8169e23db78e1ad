"""The reference's own torch CPU path of the MoE layer, timed on the host cores.

Run as a script with the reference's package first on PYTHONPATH (baseline/_ref):
`import duplex` is then the reference, not this repository.  It builds the reference's
`FusedPackedMoE` (src/duplex/streaming/fused_packed_moe.py:86-182) at the Thinker
geometry (128 experts, hidden 2048, inter 768, top-8) from a duck-typed block of
per-expert packed linears (random symmetric int4, group 128, fp32 scales, the
reference's only format: no zero points), on the CPU in fp32, with `HAVE_TRITON`
False so that `forward` takes its torch gather-bmm branch (:265-275), and times that
forward on one decode token (the branch materialises [T, k, 2I, H] dense weights, so
the reference's serving loop feeds it one token at a time).  Prints one JSON object:
seconds per token-layer (median), the torch thread count, the runs.
"""

import argparse
import json
import statistics
import time
from types import SimpleNamespace as NS

import torch
import torch.nn as nn

E, H, I, K_TOP, GROUP = 128, 2048, 768, 8, 128


def _linear(packed, scale, out_f, in_f):
    return NS(weight_packed=packed, weight_scale=scale, weight_shape=torch.tensor([out_f, in_f]))


def build(seed=7):
    import duplex.streaming.fused_packed_moe as ref  # the reference's module
    ref.HAVE_TRITON = False
    g = torch.Generator().manual_seed(seed)
    rint = lambda *s: torch.randint(-2**31, 2**31 - 1, s, generator=g, dtype=torch.int64).to(torch.int32)  # noqa: E731
    rs = lambda *s: torch.randn(*s, generator=g).abs_() * 0.01  # noqa: E731
    gp, upk, dp = rint(E, I, H // 8), rint(E, I, H // 8), rint(E, H, I // 8)
    gs, us, ds = rs(E, I, H // GROUP), rs(E, I, H // GROUP), rs(E, H, I // GROUP)
    experts = [NS(gate_proj=_linear(gp[e], gs[e], I, H), up_proj=_linear(upk[e], us[e], I, H),
                  down_proj=_linear(dp[e], ds[e], H, I)) for e in range(E)]
    gate = nn.Linear(H, E, bias=False)
    with torch.no_grad():
        gate.weight.normal_(0.0, 0.02, generator=g)
    block = NS(experts=experts, top_k=K_TOP, norm_topk_prob=True, gate=gate)
    return ref.FusedPackedMoE(block, dtype=torch.float32, device="cpu"), g


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--runs", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    a = ap.parse_args()
    m, g = build()
    ts = []
    with torch.no_grad():
        for i in range(a.warmup + a.runs):
            x = torch.randn(1, H, generator=g)
            t0 = time.perf_counter()
            m(x)
            if i >= a.warmup:
                ts.append(time.perf_counter() - t0)
    print(json.dumps({"s_per_token_layer": statistics.median(ts), "runs": ts,
                      "threads": torch.get_num_threads(), "dtype": "float32",
                      "format": "group 128 symmetric (the reference has no zero points)"}),
          flush=True)


if __name__ == "__main__":
    main()
