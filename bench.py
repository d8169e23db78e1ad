"""Benchmark: int4 MoE + dequant-GEMV decode on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Headline workload ("decode tok/s at 1/2/4/8 GPUs"): a 48-layer
Thinker MoE stack for 256 concurrent decode streams, the 128 experts of every layer
split evenly over the N GPUs (one process per GPU, NCCL): per layer each rank routes
its 256/N streams, one all-to-all dispatches every token to the ranks that hold its
experts, the rank's experts run as grouped int4 kernels, one all-to-all returns the
partial sums to the token's owner, which adds them.  A step is every stream through
the 48 layers (each layer on the same input: the attention blocks between them are
outside this config), one CUDA graph per rank.  Seeded synthetic weights in the
config-0 distributions (int4 group 128 with zero points, fp16).  value = 256 * steps /
max-over-ranks time; the per-GPU working set (314/N MB of experts per layer x 48) is
far larger than the 126 MB L2.

Beside it, on every rank (reported from the max over ranks):
  roofline  the decode MoE layer of config 0 (batch 1: router, top-8 of 128, gate|up,
            SiLU, down, combine) timed inside the persistent kernel over 24 distinct
            layers (MoEChain): algorithmic bytes per layer / time, against the measured
            HBM copy bandwidth; DRAM traffic per layer from the committed ncu summary;
  clock     config 2: the int4 linears of Thinker layers 0-23 for one token (fused
            q|k|v, o, MoE), one launch of the persistent kernel per token;
  e2e       the headline through the module's forward with pinned host buffers: H2D of
            the step's tokens, the 48 layers, D2H of the last layer's output;
  cpu_baseline  (rank 0, N = 1) the oracle (numpy restatement of the reference's
            dequant + gather-bmm) on two layer samples of the same workload.

--workload clock | batched | gemv | talker | staged select the other configs' lines
(clock: config 2 as the headline; batched: config 3, duplex/batched_bench.py; gemv:
config 1, duplex/gemv_bench.py; talker: the Talker's bf16 / int8 MoE,
duplex/talker_bench.py; staged: host-resident layers, duplex/staged_bench.py).

--impl reference times the reference algorithm on the host cores for the headline
workload: rank 0 alone (other ranks exit), each step one of the 48 layers for all 256
streams through the oracle's by-expert restatement of the reference's gather-bmm
(fused_packed_moe.py:265-275), so ms_per_step is the real time of a step;
tokens/s = 256 / (48 x ms_per_step).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "qwen3-omni-duplex_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "int4 MoE+GEMV µs/layer @batch1, % HBM peak; decode tok/s at 1/2/4/8 GPUs"
EP_LAYERS, EP_STREAMS = 48, 256
CLOCK_LAYERS = 24
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


def ep_config(n, exchange="peer"):
    how = ("dispatch and combine as NVLink peer stores from the pack and return kernels, "
           "with flags" if exchange == "peer" else "all-to-all dispatch and combine over NCCL")
    return {"workload": "config 4: 48-layer Thinker MoE stack, 256 decode streams, the 128 "
                        f"experts of every layer split over {n} GPU(s); "
                        + (how if n > 1 else "one GPU: no exchange"),
            "exchange": exchange if n > 1 else None,
            "layers": EP_LAYERS, "streams": EP_STREAMS, "streams_per_gpu": EP_STREAMS // n,
            "experts": 128, "experts_per_gpu": 128 // n, "top_k": 8, "hidden": HIDDEN,
            "moe_inter": 768, "group": 128, "zero_points": True, "activations": "fp16",
            "parallelism": f"ep{n}", "graph": "one CUDA graph per rank per step",
            "l2": "no flush: a step streams 48 x 314/N MB of distinct experts (> 126 MB L2)"}


def ep_launches_per_layer(n, exchange="peer"):
    """Our kernels launched per layer of the config-4 step: route (router, top-k), expert
    stage (bucketing, gate|up, down, expert combine), rank combine; at N > 1 the dispatch
    pack, and with the peer exchange the dispatch wait, the give-back put and its wait."""
    if n == 1:
        return 7
    return 11 if exchange == "peer" else 8


# ------------------------------------------------------------------ CPU (oracle) arms
def cpu_layer_sample(seed=5, T=EP_STREAMS):
    from duplex import synth
    return synth.moe_layer_np(seed=seed, T=T)


def time_cpu_layer(L):
    """One layer of the headline workload through the oracle: routing and the by-expert
    gather-bmm restatement for all streams.  Returns seconds."""
    import numpy as np
    import oracle as O
    x = L["x"].astype(np.float32)
    t0 = time.perf_counter()
    w, sel, _ = O.router(x, L["gate_w"], 8, True, None, "float16")
    O.moe_experts_by_expert(x, sel, w, L["gu_packed"], L["gu_scale"], L["dn_packed"],
                            L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    return time.perf_counter() - t0


def cpu_threads():
    try:
        import torch
        return torch.get_num_threads()
    except Exception:  # pragma: no cover
        return os.cpu_count() or 1


def reference_torch_cpu():
    """The reference's own torch FusedPackedMoE CPU path (baseline/_ref), one decode token
    per forward as its serving loop feeds it, in its own process (duplex/ref_cpu_bench.py);
    None when the reference is not installed."""
    import subprocess
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "duplex" / "streaming" / "fused_packed_moe.py").exists():
        return None
    script = ROOT / "qwen3-omni-duplex_b200" / "duplex" / "ref_cpu_bench.py"
    r = subprocess.run([sys.executable, str(script)], capture_output=True, text=True,
                       env=dict(os.environ, PYTHONPATH=str(ref)), timeout=600)
    if r.returncode != 0:
        return {"unavailable": ((r.stderr or r.stdout).strip().splitlines() or ["?"])[-1][:200]}
    d = json.loads(r.stdout.strip().splitlines()[-1])
    t = d["s_per_token_layer"]
    return {"value": 1.0 / (EP_LAYERS * t), "unit": "tokens/s", "cores": d["threads"],
            "kind": "reference",
            "sample": f"the reference's FusedPackedMoE.forward (torch gather-bmm branch, fp32, "
                      f"HAVE_TRITON off) on one token of one Thinker-geometry layer, median of "
                      f"{len(d['runs'])} ({t:.3f} s); tokens/s = 1 / (48 x t): it serves one "
                      "token per forward"}


def cpu_baseline_block(n_samples=2):
    L = cpu_layer_sample()
    ts = [time_cpu_layer(L) for _ in range(n_samples)]
    t = sorted(ts)[len(ts) // 2]
    out = {"value": EP_STREAMS / (EP_LAYERS * t), "unit": "tokens/s", "cores": cpu_threads(),
           "kind": "port",
           "sample": f"{n_samples} samples of one layer x 256 streams (median {t:.2f} s), numpy "
                     "restatement of the reference's dequant + gather-bmm (oracle/), by expert; "
                     "tokens/s = 256 / (48 x t_layer)"}
    out["reference_torch"] = reference_torch_cpu()
    return out


def run_reference(args):
    ws, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    K, W = max(1, args.steps), max(0, args.warmup)
    L = cpu_layer_sample()
    for _ in range(W):
        time_cpu_layer(L)
    ts = [time_cpu_layer(L) for _ in range(K)]
    t = sum(ts) / len(ts)
    value = EP_STREAMS / (EP_LAYERS * t)
    sample = ("each step: one of the 48 layers for all 256 streams (routing + by-expert "
              "gather-bmm), numpy restatement of the reference's torch path (oracle/); "
              "tokens/s = 256 / (48 x ms_per_step)")
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": K,
        "warmup": W, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int4 x f32 (numpy port, fp16-rounded activations)",
        "data": "synthetic (seeded)", "config": ep_config(ws), "impl": "reference",
        "step_unit": "one layer of the 48 (all 256 streams)",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cpu_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
def init_group(local):
    """NCCL group of the torchrun ranks (a group of one without torchrun), with a
    180 s collective timeout watched by torch's NCCL watchdog (duplex.benchutil)."""
    import torch
    import torch.distributed as dist
    from duplex import benchutil as bu
    bu.init_nccl(torch.device("cuda", local), timeout_s=180)
    return dist


def time_graph(g, K, dev, pre=None):
    """CUDA-event time of K replays (max over ranks), ms total."""
    import torch
    from duplex import benchutil as bu
    torch.cuda.synchronize(dev)
    bu.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        if pre:
            pre(i)
        g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    bu.barrier()
    return bu.max_over_ranks(e0.elapsed_time(e1), dev)


def capture(fn, dev):
    import torch
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    # thread-local capture: CUDA calls of other threads (NCCL's, torch's watchdog) may
    # run meanwhile without invalidating the capture
    with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
        fn()
    torch.cuda.synchronize(dev)
    return g


def run_ours(args):
    import torch
    from duplex import benchutil as bu, synth
    from duplex.streaming.ep_moe import ExpertParallelMoE

    _, _, local = bu.dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = init_group(local)
    ws, rank = dist.get_world_size(), dist.get_rank()
    if EP_STREAMS % ws or 128 % ws:
        raise SystemExit(f"{ws} GPUs do not split 256 streams / 128 experts")
    K, W = args.steps, max(3, args.warmup)
    T_l = EP_STREAMS // ws

    # ---------------------------------------------------------------- config 4
    layers = []
    for li in range(EP_LAYERS):
        gen = torch.Generator(device=dev).manual_seed(1000 + li)  # identical on every rank
        m = synth.moe_layer_torch(gen, device=dev)
        layers.append(ExpertParallelMoE(m["gate_w"], m["gu_packed"], m["gu_scale"], m["dn_packed"],
                                        m["dn_scale"], synth.THINKER_ACTIVE, gu_zeros=m["gu_zeros"],
                                        dn_zeros=m["dn_zeros"], dtype=torch.float16, device=dev,
                                        exchange=args.exchange))
        del m
    torch.cuda.empty_cache()
    gen = torch.Generator(device=dev).manual_seed(7 + rank)
    x = torch.randn(T_l, HIDDEN, device=dev, dtype=torch.float16, generator=gen)
    outs = [None] * EP_LAYERS

    def step():
        for li, L in enumerate(layers):
            outs[li] = L(x)

    g = capture(step, dev)
    for _ in range(W):
        g.replay()
    # clocks sampled around a soak of the same loop and the timed region
    sampler = bu.ClockSampler(bu.visible_gpu_indices(ws)).start() if rank == 0 else None
    # every step exchanges with the other ranks, so all ranks replay the same number of
    # times: the soak length comes from one replay timed on every rank (max over ranks)
    # (--soak 0, the same on every rank, skips it: the launch sequence stays W + K replays)
    if args.soak > 0:
        torch.cuda.synchronize(dev)
        bu.barrier()
        t_one = time.perf_counter()
        g.replay()
        torch.cuda.synchronize(dev)
        n_soak = bu.soak_replays(args.soak, time.perf_counter() - t_one, dev)
        for _ in range(n_soak):
            g.replay()
        torch.cuda.synchronize(dev)
    ms = time_graph(g, K, dev)
    ms_step = ms / K
    value = EP_STREAMS * K / (ms / 1e3)
    derr = sum(L.device_errors() for L in layers)

    # per-GPU bytes of the selected local experts per layer (HBM roofline of the stage)
    per_expert = (layers[0].gu_tiles.buf.numel() + layers[0].dn_tiles.buf.numel()) / layers[0].E_local
    x_all = torch.empty(ws * T_l, HIDDEN, dtype=x.dtype, device=dev)
    dist.all_gather_into_tensor(x_all, x)
    _, sel = layers[0].route(x_all)
    loc = sel[(sel >= layers[0].e_begin) & (sel < layers[0].e_begin + layers[0].E_local)]
    ep_bytes = int(torch.unique(loc).numel()) * per_expert

    # end to end through the module: pinned host tokens in, last layer's output out
    xh = torch.randn(T_l, HIDDEN, dtype=torch.float16).pin_memory()
    oh = torch.empty(T_l, HIDDEN, dtype=torch.float16).pin_memory()

    torch.cuda.synchronize(dev)
    bu.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        x.copy_(xh, non_blocking=True)
        g.replay()
        oh.copy_(outs[-1], non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    bu.barrier()
    ms_e2e = bu.max_over_ranks(e0.elapsed_time(e1), dev)
    e2e_value = EP_STREAMS * K / (ms_e2e / 1e3)
    clocks = sampler.stop().summary() if sampler else None
    del g
    for L in layers:
        L.close()
    layers.clear()
    outs = None
    torch.cuda.empty_cache()

    # ---------------------------------------------------------------- configs 2 and 0
    from duplex.clock import ClockStack, MoEChain, moe_bytes
    stack = ClockStack.synthetic(n_layers=CLOCK_LAYERS, seed=1234 + rank, device=dev)
    pool = torch.randn(64, 1, HIDDEN, device=dev, dtype=torch.float16,
                       generator=torch.Generator(device=dev).manual_seed(77 + rank))
    gc = stack.capture()
    for i in range(W):
        stack.x_in.copy_(pool[i % 64])
        gc.replay()
    ms_c = time_graph(gc, K, dev, pre=lambda i: stack.x_in.copy_(pool[i % 64]))
    clock = {"value": K / (ms_c / 1e3), "unit": "tokens/s per GPU",
             "us_per_layer": ms_c * 1e3 / (K * CLOCK_LAYERS),
             "workload": "config 2: int4 linears of Thinker layers 0-23 (fused q|k|v, o, "
                         "router + 128-expert top-8 MoE), one decode token, one launch",
             "bytes_per_token": stack.bytes_per_step()}
    moes = [Lc.moe for Lc in stack.layers]
    chain = MoEChain(moes, rms_eps=1e-6, residual=False)
    hx = torch.zeros(1, HIDDEN, device=dev, dtype=torch.float16)
    hout = torch.zeros(1, HIDDEN, device=dev, dtype=torch.float16)
    gm = capture(lambda: chain.forward_into(hx, hout), dev)
    for i in range(W):
        hx.copy_(pool[i % 64])
        gm.replay()
    Km = max(K, 50)
    ms_m = time_graph(gm, Km, dev, pre=lambda i: hx.copy_(pool[i % 64]))
    us_moe = ms_m * 1e3 / (Km * CLOCK_LAYERS)
    mb = moe_bytes(moes[0])
    derr += stack.device_errors() + chain.p.device_errors()
    del gm, gc
    stack.graph = None

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_block(args.cpu_samples)

    peak, peak_kind = peaks()
    achieved = mb / (us_moe * 1e-6) / 1e9
    us_layer = ms_step * 1e3 / EP_LAYERS
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": K,
        "warmup": W, "ms_per_step": ms_step, "us_per_layer": us_layer,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4 weights x f16 activations, f32 accumulate",
        "data": "synthetic (seeded; BASELINE config distributions)",
        "config": ep_config(ws, args.exchange),
        "ep_hbm": {"bytes_per_layer_per_gpu": ep_bytes,
                   "GBps": ep_bytes / (us_layer * 1e3), "frac": ep_bytes / (us_layer * 1e3) / peak,
                   "note": "bytes of the selected local experts (tile records) per layer per GPU"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic("moe_layer_dram_bytes"),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of a "
                                       "4-layer MoE-chain launch / 4 (profiles/traffic.txt)",
                     "kernel": "decode MoE layer (config 0: router, top-8 of 128, gate|up, "
                               "down, combine), batch 1, inside the persistent clustered stack "
                               "kernel over 24 distinct layers",
                     "us_per_launch": us_moe, "algorithmic_bytes": mb,
                     "peak_kind": f"{peak_kind} (copy bandwidth, MEASURED_PEAKS.json)"},
        "clock": clock,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "tokens/s",
                "h2d_bytes_per_step": T_l * HIDDEN * 2, "d2h_bytes_per_step": T_l * HIDDEN * 2},
        "gpu_launches": ep_launches_per_layer(ws, args.exchange) * EP_LAYERS * K,
        "gpu_launches_note": "per layer: router, top-k, bucketing, gate|up, down, expert combine, "
                             "rank combine; at N > 1 also the dispatch pack, and with the peer "
                             "exchange its wait, the give-back put and its wait (the NCCL form "
                             "adds 2 all-to-alls instead)",
        "clocks": clocks,
        "device_errors": derr,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--soak", type=float, default=1.0, help="seconds of load before timing")
    ap.add_argument("--cpu-samples", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["ep", "clock", "batched", "gemv", "talker", "staged"],
                    default="ep",
                    help="ep: config 4, the default line (see the module docstring); clock: "
                         "config 2 as the line (duplex/clock_bench.py); batched: config 3 "
                         "(duplex/batched_bench.py); gemv: config 1 (duplex/gemv_bench.py); "
                         "talker: the Talker MoE (duplex/talker_bench.py); staged: host-resident "
                         "layers (duplex/staged_bench.py)")
    ap.add_argument("--streams", type=int, default=256, help="batched: concurrent streams")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="config 4 at N > 1: dispatch / combine over NVLink peer stores (one "
                         "pack-and-send kernel, flags, bounded waits) or NCCL all-to-alls")
    args = ap.parse_args()
    if args.workload == "batched" and args.impl == "ours":
        from duplex import batched_bench
        raise SystemExit(batched_bench.main(["--streams", str(args.streams), "--steps", str(args.steps),
                                             "--warmup", str(args.warmup)]))
    if args.workload == "gemv":
        from duplex import gemv_bench
        raise SystemExit(gemv_bench.main(["--steps", str(args.steps), "--warmup", str(args.warmup),
                                          "--impl", args.impl]))
    if args.workload == "staged":
        from duplex import staged_bench
        raise SystemExit(staged_bench.main(["--steps", str(args.steps), "--warmup", str(args.warmup)]))
    if args.workload == "talker":
        from duplex import talker_bench
        raise SystemExit(talker_bench.main(["--steps", str(args.steps), "--warmup", str(args.warmup)]))
    if args.workload == "clock":
        from duplex import clock_bench
        raise SystemExit(clock_bench.main(["--steps", str(args.steps), "--warmup", str(args.warmup),
                                           "--impl", args.impl]))
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
