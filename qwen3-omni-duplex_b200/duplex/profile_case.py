"""Run a fixed decode case for an external profiler (ncu) or a quick timing.

    python -m duplex.profile_case --stack clock --layers 4 --steps 4
    python -m duplex.profile_case --stack moe --layers 24 --steps 20 --time
    python -m duplex.profile_case --stack grouped --tokens 256 --layers 4 --steps 40 --time
    python -m duplex.profile_case --stack grouped --engine mma --tokens 256 --layers 4 --steps 40 --time

Builds seeded synthetic Thinker-geometry layers (hidden 2048, 128 experts, top-8,
int4 group 128 with zero points, fp16) and runs `--steps` launches of the persistent
kernel: the clock path (`ClockStack`: q|k|v, o, MoE per layer) or the MoE chain
(`MoEChain`: MoE only); or `--steps` grouped MoE calls (`duplex_moe_grouped`, batched
decode of `--tokens` streams, on the tcgen05 or the mma.sync expert engine), cycling
over `--layers` distinct layers so that no
call finds its experts in L2.  With --time it prints the time per step (per layer)
measured with CUDA events over the last half of the steps, and for the grouped path
the bytes of the experts it selected; device errors are always checked.
"""

from __future__ import annotations

import argparse

import torch

from .clock import ClockStack, MoEChain


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--stack", choices=["clock", "moe", "grouped"], default="clock")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--time", action="store_true")
    ap.add_argument("--engine", choices=["tc", "mma"], default="tc", help="grouped expert engine")
    a = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    if a.stack == "grouped":
        return grouped(a, dev)
    st = ClockStack.synthetic(n_layers=a.layers, seed=1, device=dev, T=a.tokens)
    x = torch.randn(a.tokens, st.hidden, device=dev, dtype=torch.float16,
                    generator=torch.Generator(device=dev).manual_seed(0))
    out = torch.zeros_like(x)
    if a.stack == "clock":
        run, errs = (lambda: st.step_into(x, out)), st.device_errors
    else:
        chain = MoEChain([L.moe for L in st.layers], residual=True, T=a.tokens)
        run, errs = (lambda: chain.forward_into(x, out)), chain.p.device_errors
    half = max(1, a.steps // 2)
    for _ in range(a.steps - half):
        run()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(half):
        run()
    e1.record()
    torch.cuda.synchronize(dev)
    err = errs()
    if a.time:
        us = e0.elapsed_time(e1) * 1e3 / half
        print(f"{a.stack}: {us:.1f} us/launch, {us / a.layers:.2f} us/layer, device errors {err}")
    if err:
        print(f"device error word {err:#x}")
        return 1
    return 0


def grouped(a, dev) -> int:
    from . import synth
    from .streaming.fused_packed_moe import FusedPackedMoE
    gen = torch.Generator(device=dev).manual_seed(1)
    layers = []
    for _ in range(a.layers):
        m = synth.moe_layer_torch(gen, device=dev)
        layers.append(FusedPackedMoE.from_stacked(
            m["gate_w"], m["gu_packed"], m["gu_scale"], m["dn_packed"], m["dn_scale"],
            synth.THINKER_ACTIVE, gu_zeros=m["gu_zeros"], dn_zeros=m["dn_zeros"],
            dtype=torch.float16, device=dev, tc=a.engine == "tc"))
        del m
    x = torch.randn(a.tokens, layers[0].hidden, device=dev, dtype=torch.float16, generator=gen)
    out = torch.empty_like(x)
    sel = torch.empty(a.tokens, layers[0].top_k, dtype=torch.int32, device=dev)
    half = max(1, a.steps // 2)
    for s in range(a.steps - half):
        layers[s % a.layers].forward_grouped_into(x, out, sel_out=sel, engine=a.engine)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(half):
        layers[s % a.layers].forward_grouped_into(x, out, engine=a.engine)
    e1.record()
    torch.cuda.synchronize(dev)
    err = 0
    for m in layers:
        err |= m.device_errors()
    if a.time:
        us = e0.elapsed_time(e1) * 1e3 / half
        L0 = layers[0]
        gu, dn = (L0.gu_tc, L0.dn_tc) if a.engine == "tc" else (L0.gu_tiles, L0.dn_tiles)
        per_expert = (gu.buf.numel() + dn.buf.numel()) / L0.num_experts
        n_sel = int(torch.unique(sel).numel())
        mb = n_sel * per_expert / 1e6
        print(f"grouped[{a.engine}] T={a.tokens}: {us:.1f} us/layer, {n_sel} experts selected, "
              f"{mb:.1f} MB of experts -> {mb / us:.2f} TB/s, device errors {err}")
    if err:
        print(f"device error word {err:#x}")
        return 1
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
