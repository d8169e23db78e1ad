"""Expert-parallel decode benchmark: a 48-layer Thinker MoE stack at
256 concurrent streams, experts split evenly over N ranks (one per GPU, NCCL).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m duplex.ep_bench [--layers 48]
        [--streams 256] [--steps 20] [--warmup 3]

Each rank holds its 128/N experts of every layer (seeded synthetic weights in the
config 0 distributions: int4 group 128 with zero points, fp16) and 256/N streams.  A
step takes every stream one token through the 48 layers: per layer local routing,
all-gather of tokens and selections, the rank's experts (grouped int4 kernels),
reduce-scatter of the fp32 partial sums.  The layers run back to back on the same
input (the attention blocks between them are outside this config), so a step does
exactly the per-layer work of a real stack.  The whole step is captured in one CUDA
graph per rank; time is CUDA events around K replays, max over ranks.

Prints one JSON line (rank 0): tokens/s for all streams, us/layer, and the per-rank
weight bytes the selected local experts stream per layer against the HBM peak.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
from pathlib import Path

import torch
import torch.distributed as dist

from . import synth
from .streaming.ep_moe import ExpertParallelMoE

ROOT = Path(__file__).resolve().parents[2]


def hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--streams", type=int, default=256)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29541")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    if a.streams % world:
        raise SystemExit(f"{a.streams} streams do not split over {world} ranks")
    T_l = a.streams // world
    layers = []
    for li in range(a.layers):
        gen = torch.Generator(device=dev).manual_seed(1000 + li)  # identical on every rank
        m = synth.moe_layer_torch(gen, device=dev)
        layers.append(ExpertParallelMoE(m["gate_w"], m["gu_packed"], m["gu_scale"], m["dn_packed"],
                                        m["dn_scale"], synth.THINKER_ACTIVE, gu_zeros=m["gu_zeros"],
                                        dn_zeros=m["dn_zeros"], dtype=torch.float16, device=dev))
        del m
    torch.cuda.empty_cache()
    gen = torch.Generator(device=dev).manual_seed(7 + rank)
    x = torch.randn(T_l, synth.THINKER_HIDDEN, device=dev, dtype=torch.float16, generator=gen)
    outs = [torch.empty_like(x) for _ in layers]

    def step():
        for li, L in enumerate(layers):
            outs[li].copy_(L(x))

    # selected-expert bytes per layer on this rank (for the roofline), from one routing
    per_expert = (layers[0].gu_tiles.buf.numel() + layers[0].dn_tiles.buf.numel()) / layers[0].E_local
    x_all = torch.empty(world * T_l, x.shape[1], dtype=x.dtype, device=dev)
    dist.all_gather_into_tensor(x_all, x)
    _, sel = layers[0].route(x_all)
    loc = sel[(sel >= layers[0].e_begin) & (sel < layers[0].e_begin + layers[0].E_local)]
    n_local_sel = int(torch.unique(loc).numel())
    bytes_layer = n_local_sel * per_expert

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(a.warmup):
            step()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        step()
    g.replay()
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record()
    for _ in range(a.steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = torch.tensor([e0.elapsed_time(e1) / a.steps], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    derr = 0
    for L in layers:
        derr |= L.device_errors()
    peak, kind = hbm_peak()
    us_layer = ms * 1e3 / a.layers
    line = {
        "metric": "config 4 expert-parallel decode: 48-layer Thinker MoE stack, tokens/s",
        "value": a.streams / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "us_per_layer": us_layer, "higher_is_better": True,
        "scaling": "strong", "dtype": "int4 weights x f16 activations, f32 accumulate",
        "data": "synthetic (seeded; config 0 distributions)",
        "config": {"workload": "config 4: 48 Thinker MoE layers, 256 decode streams, experts "
                               f"split over {world} GPU(s) (NCCL all-gather + reduce-scatter)",
                   "layers": a.layers, "streams": a.streams, "streams_per_gpu": T_l,
                   "experts_per_gpu": layers[0].E_local, "top_k": synth.THINKER_ACTIVE, "group": 128,
                   "zero_points": True, "graph": "one CUDA graph per rank per step"},
        "per_gpu_hbm": {"bytes_per_layer": bytes_layer, "GBps": bytes_layer / (us_layer * 1e3),
                        "frac": bytes_layer / (us_layer * 1e3) / peak, "peak": peak, "peak_kind": kind,
                        "local_experts_selected": n_local_sel},
        "device_errors": derr,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del g
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
