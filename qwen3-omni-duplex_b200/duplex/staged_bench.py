"""Host-resident layer line (`bench.py --workload staged`): the reference's
`host_resident=True` layers (src/duplex/streaming/fused_packed_moe.py:130-164,233-253),
whose expert records stay in host memory and are staged per call, at the Thinker
geometry of config 0 (128 experts, hidden 2048, inter 768, top-8, group 128 with zero
points, fp16) for T = 1 and 8 tokens.

Four distinct host-resident layers (4 x 314 MB of mapped pinned host memory) run back to
back in one CUDA graph; µs per layer = replay time / 4.  The bound is the host link: the
line reports the staged bytes per layer (the planned experts' gate|up and down records)
over the time, against a plain pinned host-to-device cudaMemcpyAsync of 256 MB timed in
the same process (the link's copy bandwidth).
"""

from __future__ import annotations

import argparse
import json

LAYERS = 4


def main(argv=None) -> int:
    import torch
    from duplex import synth
    from duplex.streaming.fused_packed_moe import FusedPackedMoE

    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    K, W = max(1, args.steps), max(3, args.warmup)

    layers = []
    for li in range(LAYERS):
        gen = torch.Generator(device=dev).manual_seed(3000 + li)
        m = synth.moe_layer_torch(gen, device=dev)
        layers.append(FusedPackedMoE.from_stacked(
            m["gate_w"], m["gu_packed"], m["gu_scale"], m["dn_packed"], m["dn_scale"],
            synth.THINKER_ACTIVE, gu_zeros=m["gu_zeros"], dn_zeros=m["dn_zeros"],
            dtype=torch.float16, device=dev, host_resident=True))
        del m
    torch.cuda.empty_cache()
    per_expert = (layers[0].gu_host.nbytes + layers[0].dn_host.nbytes) // layers[0].num_experts

    # the host link's copy bandwidth: pinned host -> device, 256 MB, CUDA events
    nb = 256 << 20
    src = torch.empty(nb, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nb, dtype=torch.uint8, device=dev)
    for _ in range(2):
        dst.copy_(src, non_blocking=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(4):
        dst.copy_(src, non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    h2d_gbs = 4 * nb / (e0.elapsed_time(e1) * 1e-3) / 1e9
    del src, dst

    rows = []
    for T in (1, 8):
        gen = torch.Generator(device=dev).manual_seed(11 + T)
        x = torch.randn(T, synth.THINKER_HIDDEN, device=dev, dtype=torch.float16, generator=gen)
        outs = [torch.empty_like(x) for _ in layers]
        sels = [torch.empty(T, synth.THINKER_ACTIVE, dtype=torch.int32, device=dev) for _ in layers]

        def step():
            for L, o, s in zip(layers, outs, sels):
                L.forward_staged_into(x, o, sel_out=s)

        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step()
        for _ in range(W):
            g.replay()
        torch.cuda.synchronize(dev)
        e0.record()
        for _ in range(K):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1e3 / (K * LAYERS)
        distinct = sum(int(torch.unique(sl).numel()) for sl in sels) / LAYERS
        staged = distinct * per_expert
        gbs = staged / (us * 1e-6) / 1e9
        derr = sum(L.device_errors() for L in layers)
        rows.append({"tokens": T, "us_per_layer": us, "experts_staged_per_layer": distinct,
                     "staged_bytes_per_layer": staged, "host_link_GBps": gbs,
                     "frac_of_h2d_copy": gbs / h2d_gbs, "device_errors": derr})
        del g
    print(json.dumps({
        "metric": "host-resident int4 MoE layer µs/layer (experts staged from host memory)",
        "unit": "us/layer", "higher_is_better": False, "steps": K, "warmup": W,
        "dtype": "int4 weights x f16 activations, f32 accumulate",
        "data": "synthetic (seeded; BASELINE config-0 distributions)",
        "config": {"workload": "host-resident Thinker MoE layer (config-0 geometry), "
                               f"{LAYERS} distinct layers in one CUDA graph",
                   "experts": 128, "top_k": 8, "hidden": 2048, "moe_inter": 768,
                   "group": 128, "zero_points": True},
        "h2d_copy_GBps": h2d_gbs,
        "h2d_copy_note": "pinned host -> device cudaMemcpyAsync of 256 MB (the host link's peak)",
        "rows": rows,
        "gpu_launches_per_layer": 4,
        "gpu_launches_note": "router, stage (host -> device slots), gate|up, down",
    }), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
