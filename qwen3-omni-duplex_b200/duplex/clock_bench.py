"""Config 2 line: the clock path (int4 linears of Thinker layers 0-23 for one decode
token: fused q|k|v, o, router + 128-expert top-8 MoE; group 128 with zero points,
fp16) as one launch of the persistent kernel per token; `bench.py --workload clock`.

The default bench line is config 4 (bench.py); this keeps config 2 as a line of its
own with the same contract: tokens/s, us/layer, the config-0 MoE layer as the roofline
unit, the end-to-end figure through `ClockStack.decode()` with pinned host buffers, the
CPU oracle on a bounded sample (one clock layer per step for --impl reference), and
SM clocks sampled around the timed region.  With N ranks every rank runs an
independent replica (batch-1 decode does not shard).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
for _p in (str(ROOT), str(ROOT / "qwen3-omni-duplex_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "int4 MoE+GEMV µs/layer @batch1, % HBM peak; decode tok/s at 1/2/4/8 GPUs"
N_LAYERS = 24
HIDDEN = 2048
TRAFFIC = ROOT / "profiles" / "traffic.txt"


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic(key):
    """A figure of the committed ncu summary profiles/traffic.txt (key = value lines)."""
    if TRAFFIC.exists():
        for line in TRAFFIC.read_text().splitlines():
            k, _, v = line.partition("=")
            if k.strip() == key:
                return float(v.split()[0])
    return None


def config_block(n_gpus, batch=1):
    return {
        "workload": "config 2 clock path: int4 linears of Thinker layers 0-23 (fused qkv, o, "
                    "router + 128-expert top-8 MoE), one decode token",
        "layers": N_LAYERS, "hidden": HIDDEN, "experts": 128, "top_k": 8, "moe_inter": 768,
        "q_heads": 32, "kv_heads": 4, "head_dim": 128, "group": 128, "zero_points": True,
        "batch": batch, "activations": "fp16",
        "parallelism": "replicas" if n_gpus == 1 else f"{n_gpus} replicas (batch-1 decode)",
        "l2": "no flush: each step streams ~720 MB of distinct weights (> 126 MB L2)",
    }


# ------------------------------------------------------------------ CPU (oracle) arms
def cpu_layer_sample(seed=5):
    """One full-geometry clock-path layer as numpy arrays (same distributions)."""
    import numpy as np
    from duplex import synth
    rng = np.random.Generator(np.random.PCG64(seed))
    qkv = synth.linear_np(rng, 5120, HIDDEN, 128, True)
    o = synth.linear_np(rng, HIDDEN, 4096, 128, True)
    m = synth.moe_layer_np(seed=seed + 1, T=1)
    d = dict(qkv_packed=qkv["packed"], qkv_scale=qkv["scale"], qkv_zeros=qkv["zeros"],
             o_packed=o["packed"], o_scale=o["scale"], o_zeros=o["zeros"])
    for k in ("gate_w", "gu_packed", "gu_scale", "gu_zeros", "dn_packed", "dn_scale", "dn_zeros"):
        d[k] = m[k]
    return d, m["x"].astype(np.float32)


def time_cpu_layers(n_samples, n_warm=1):
    from oracle.clock_oracle import clock_layer
    threads = os.cpu_count() or 1
    d, h = cpu_layer_sample()
    for _ in range(n_warm):
        clock_layer(h, d, 8, threads=threads)
    ts = []
    for _ in range(n_samples):
        t0 = time.perf_counter()
        clock_layer(h, d, 8, threads=threads)
        ts.append(time.perf_counter() - t0)
    return ts, threads


def cpu_baseline_block(n_samples=3):
    ts, threads = time_cpu_layers(n_samples)
    t_layer = sorted(ts)[len(ts) // 2]
    return {"value": 1.0 / (N_LAYERS * t_layer), "unit": "tokens/s", "cores": threads,
            "kind": "port",
            "sample": f"{n_samples} of the 24 layers (median {t_layer * 1e3:.0f} ms/layer), "
                      "numpy port of the reference's dequant + gather-bmm path, experts on a "
                      f"{threads}-thread pool; tokens/s = 1/(24 x t_layer)"}


def run_reference(args):
    """The oracle on the host cores, rank 0 alone: each step one clock-path layer for one
    token (so ms_per_step is a step's real time); tokens/s = 1 / (24 x ms_per_step)."""
    ws, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    K, W = max(1, args.steps), max(0, args.warmup)
    ts, threads = time_cpu_layers(K, n_warm=W)
    t_layer = sum(ts) / len(ts)
    value = 1.0 / (N_LAYERS * t_layer)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": K,
        "warmup": W, "ms_per_step": t_layer * 1e3, "step_unit": "one clock-path layer of the 24",
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4 x f32 (numpy port, fp16-rounded activations)",
        "data": "synthetic (seeded)", "config": config_block(ws), "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": "each step one of the 24 clock-path layers (numpy port of the "
                                   "reference's torch dequant + gather-bmm path); tokens/s = "
                                   "1 / (24 x ms_per_step)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
def run_ours(args):
    import torch
    from duplex import benchutil as bu
    from duplex.clock import ClockStack, moe_bytes

    n_gpus = args.gpus
    ws, rank, local = bu.dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        bu.init_dist("nccl")
    K, W = args.steps, max(3, args.warmup)

    stack = ClockStack.synthetic(n_layers=N_LAYERS, seed=1234 + rank, device=dev)
    pool = torch.randn(64, 1, HIDDEN, device=dev, dtype=torch.float16,
                       generator=torch.Generator(device=dev).manual_seed(77 + rank))
    stack.capture()

    def step(i):
        stack.x_in.copy_(pool[i % 64])
        stack.replay()

    for i in range(W):
        step(i)
    torch.cuda.synchronize(dev)

    # clocks: sampled over a soak of the same loop bracketing the timed steps
    sampler = bu.ClockSampler(bu.visible_gpu_indices(max(1, ws))).start() if rank == 0 else None
    t_soak = time.perf_counter()
    i = 0
    while time.perf_counter() - t_soak < args.soak:
        step(i)
        i += 1
        if i % 64 == 0:
            torch.cuda.synchronize(dev)
    torch.cuda.synchronize(dev)

    bu.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        step(i)
    e1.record()
    torch.cuda.synchronize(dev)
    bu.barrier()
    ms = bu.max_over_ranks(e0.elapsed_time(e1), dev)
    ms_step = ms / K
    value = ws * K / (ms / 1e3)

    # end to end through the public decode() call, host buffers
    xh = torch.randn(64, 1, HIDDEN, dtype=torch.float16).pin_memory()
    oh = torch.empty(64, 1, HIDDEN, dtype=torch.float16).pin_memory()
    for i in range(W):
        stack.decode(xh[i % 64], oh[i % 64])
    torch.cuda.synchronize(dev)
    bu.barrier()
    torch.cuda.synchronize(dev)
    e0.record()
    for i in range(K):
        stack.decode(xh[i % 64], oh[i % 64])
    e1.record()
    torch.cuda.synchronize(dev)
    bu.barrier()
    ms_e2e = bu.max_over_ranks(e0.elapsed_time(e1), dev)
    e2e_value = ws * K / (ms_e2e / 1e3)

    # roofline unit: the decode MoE layer (router, top-k, gate|up, down, combine) of
    # config 0, timed over the 24 distinct MoE layers of the stack in one persistent
    # launch: x -> MoE(rms(x)) layer after layer
    from duplex.clock import MoEChain
    moes = [L.moe for L in stack.layers]
    chain = MoEChain(moes, rms_eps=1e-6, residual=False)
    hx = torch.zeros(1, HIDDEN, device=dev, dtype=torch.float16)
    hout = torch.zeros(1, HIDDEN, device=dev, dtype=torch.float16)

    def moe_chain():
        chain.forward_into(hx, hout)

    moe_chain()
    torch.cuda.synchronize(dev)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    gm = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(gm, stream=s):
            moe_chain()
    torch.cuda.current_stream(dev).wait_stream(s)
    for i in range(W):
        hx.copy_(pool[i % 64])
        gm.replay()
    torch.cuda.synchronize(dev)
    bu.barrier()
    torch.cuda.synchronize(dev)
    Km = max(K, 50)
    e0.record()
    for i in range(Km):
        hx.copy_(pool[i % 64])
        gm.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    bu.barrier()
    ms_moe = bu.max_over_ranks(e0.elapsed_time(e1), dev)
    us_moe = ms_moe * 1e3 / (Km * N_LAYERS)
    mb = moe_bytes(moes[0])

    # drain the soak sampler after a short tail of load
    t_tail = time.perf_counter()
    i = 0
    while time.perf_counter() - t_tail < 0.3:
        step(i)
        i += 1
    torch.cuda.synchronize(dev)
    clocks = sampler.stop().summary() if sampler else None
    errors = stack.device_errors()

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_block(args.cpu_samples)

    peak, peak_kind = peaks()
    achieved = mb / (us_moe * 1e-6) / 1e9
    bytes_step = stack.bytes_per_step()
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": K,
        "warmup": W, "ms_per_step": ms_step, "us_per_layer": ms_step * 1e3 / N_LAYERS,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4 weights x f16 activations, f32 accumulate",
        "data": "synthetic (seeded; BASELINE config distributions)",
        "config": config_block(ws),
        "step_hbm": {"bytes": bytes_step, "GBps": bytes_step / (ms_step * 1e-3) / 1e9,
                     "frac": bytes_step / (ms_step * 1e-3) / 1e9 / peak},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic("moe_layer_dram_bytes"),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of a "
                                       "4-layer MoE-chain launch / 4 (profiles/traffic.txt)",
                     "kernel": "decode MoE layer (router, top-k, gate|up, down, combine) in the "
                               "persistent clustered stack kernel, config 0 geometry, batch 1, 24 "
                               "distinct layers per launch",
                     "us_per_launch": us_moe, "algorithmic_bytes": mb,
                     "peak_kind": f"{peak_kind} (copy bandwidth, MEASURED_PEAKS.json)"},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": HIDDEN * 2,
                "d2h_bytes_per_step": HIDDEN * 2},
        "gpu_launches": stack.kernels_per_step() * K,
        "clocks": clocks,
        "device_errors": errors,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del gm
    stack.graph = None
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--soak", type=float, default=1.0)
    ap.add_argument("--cpu-samples", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
