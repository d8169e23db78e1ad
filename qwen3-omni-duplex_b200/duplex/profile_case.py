"""Run a fixed decode case for an external profiler (ncu) or a quick timing.

    python -m duplex.profile_case --stack clock --layers 4 --steps 4
    python -m duplex.profile_case --stack moe --layers 24 --steps 20 --time

Builds seeded synthetic Thinker-geometry layers (hidden 2048, 128 experts, top-8,
int4 group 128 with zero points, fp16) and runs `--steps` launches of the persistent
kernel: the clock path (`ClockStack`: q|k|v, o, MoE per layer) or the MoE chain
(`MoEChain`: MoE only).  With --time it prints us/layer measured with CUDA events over
the last half of the steps; device errors are always checked.
"""

from __future__ import annotations

import argparse

import torch

from .clock import ClockStack, MoEChain


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--stack", choices=["clock", "moe"], default="clock")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--time", action="store_true")
    a = ap.parse_args(argv)
    dev = torch.device("cuda:0")
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


if __name__ == "__main__":
    raise SystemExit(main())
