"""Config 3 benchmark: batched decode through one Thinker MoE layer (one JSON line).

    python -m duplex.batched_bench [--streams 256] [--layers 8] [--steps 20] [--warmup 3]
                                   [--engine auto|tc|mma] [--dtype bf16|fp16]

T concurrent streams (64 or 256 in the configuration) through one int4 MoE layer
(128 experts, hidden 2048, inter 768, top-8, group 128 with zero points), routed by
random router logits ~N(0,1) as the configuration specifies, on the grouped path
(`FusedPackedMoE.forward_grouped_into`). `--layers` distinct seeded layers are
called in rotation so that no call finds its experts in L2 (8 layers: ~2.5 GB). A
step is one call per layer, captured in one CUDA graph; the time is CUDA events
around K replays. The roofline unit is one layer call: the record bytes of the
experts its routing selects, over its time, against the measured HBM copy bandwidth.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from . import synth
from .streaming.fused_packed_moe import FusedPackedMoE

HBM_GBS = 6545.3  # MEASURED_PEAKS.json hbm_gbs (fallback when the file is absent)


def _peak() -> tuple[float, str]:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return HBM_GBS, "measured (copied)"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--streams", type=int, default=256)
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--engine", choices=["auto", "tc", "mma"], default="auto")
    ap.add_argument("--dtype", choices=["bf16", "fp16"], default="bf16")
    a = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    dt = torch.bfloat16 if a.dtype == "bf16" else torch.float16
    T = a.streams
    layers, logits = [], []
    for li in range(a.layers):
        gen = torch.Generator(device=dev).manual_seed(3000 + li)
        m = synth.moe_layer_torch(gen, device=dev, dtype=dt)
        layers.append(FusedPackedMoE.from_stacked(
            m["gate_w"], m["gu_packed"], m["gu_scale"], m["dn_packed"], m["dn_scale"],
            synth.THINKER_ACTIVE, gu_zeros=m["gu_zeros"], dn_zeros=m["dn_zeros"], dtype=dt,
            device=dev, tc=a.engine != "mma"))
        del m
        # router logits ~N(0,1), rounded to the activation dtype as the router's output is
        lg = torch.randn(T, layers[-1].num_experts, device=dev, generator=gen)
        logits.append(lg.to(dt).float())
    torch.cuda.empty_cache()
    engine = layers[0].grouped_engine(T) if a.engine == "auto" else a.engine
    gen = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(T, layers[0].hidden, device=dev, dtype=dt, generator=gen)
    outs = [torch.empty_like(x) for _ in layers]
    sels = [torch.empty(T, layers[0].top_k, dtype=torch.int32, device=dev) for _ in layers]

    def step():
        for li, L in enumerate(layers):
            L.forward_grouped_into(x, outs[li], sel_out=sels[li], logits=logits[li], engine=engine)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(max(a.warmup, 1)):
            step()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        step()
    for _ in range(a.warmup):
        g.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / a.steps
    us_layer = ms * 1e3 / a.layers
    err = 0
    for L in layers:
        err |= L.device_errors()
    # record bytes of the experts each layer's routing selected
    L0 = layers[0]
    gu, dn = (L0.gu_tc, L0.dn_tc) if engine == "tc" else (L0.gu_tiles, L0.dn_tiles)
    per_expert = (gu.buf.numel() + dn.buf.numel()) / L0.num_experts
    n_sel = [int(torch.unique(sl).numel()) for sl in sels]
    bytes_layer = sum(n_sel) / len(n_sel) * per_expert
    peak, kind = _peak()
    achieved = bytes_layer / (us_layer * 1e-6) / 1e9
    del g
    print(json.dumps({
        "metric": "config 3 batched decode MoE layer, tokens/s",
        "value": T / (us_layer * 1e-6), "unit": "tokens/s", "n_gpus": 1, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "us_per_layer": us_layer, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": f"int4 weights x {a.dtype} activations, f32 accumulate",
        "data": "synthetic (seeded weights, config 0 distributions; router logits ~N(0,1))",
        "config": {"workload": f"config 3: {T} streams through one Thinker MoE layer, {a.layers} "
                               "distinct layers in rotation (working set above L2)",
                   "streams": T, "layers_in_rotation": a.layers, "engine": engine, "experts": 128,
                   "top_k": 8, "group": 128, "zero_points": True, "graph": "one CUDA graph per step"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": kind,
                     "bytes_per_layer": bytes_layer, "experts_selected": sum(n_sel) / len(n_sel)},
        "device_errors": err}))
    return 1 if err else 0


if __name__ == "__main__":
    raise SystemExit(main())
