"""Config 1 line: the dense int4 dequant-GEMV sweep (`bench.py --workload gemv`).

Shapes of the Thinker's attention linears and the lm_head -- q 2048 -> 4096, k / v
2048 -> 512, o 4096 -> 2048, the fused q|k|v 2048 -> 5120 the clock path uses, lm_head
2048 -> 151936 -- at B = 1, 2, 4, 8 fp16 rows, through `TritonPackedLinear.forward`
(one launch of `duplex_packed_linear` per call), in two formats:
  * BASELINE's: group 128 with 4-bit zero points, fp16 scales;
  * the reference's: group 32, symmetric (nibble - 8), as its Triton kernel reads it.
Each timed replay cycles over enough distinct copies of the weights that the working
set exceeds 300 MB (> the 126 MB L2), in one CUDA graph; per call = replay time /
copies.  GB/s counts the algorithmic bytes of a call (nibbles, scales, zero points,
x and y) against the measured HBM copy bandwidth.

When the reference is installed in baseline/_ref, its own `TritonPackedLinear` (the
Triton `_dq_gemv_kernel`, one launch per row; src/duplex/streaming/
triton_dequant_gemv.py:125-159) is timed on the same B200 on the same group-32
symmetric weights, in a separate process (both packages are named `duplex`), by
`ref_triton_bench.py`; its compiled cache is never read.  `--impl reference` prints
that arm alone.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
REF = ROOT / "baseline" / "_ref"
SHAPES = [("q", 4096, 2048), ("k", 512, 2048), ("v", 512, 2048), ("o", 2048, 4096),
          ("qkv", 5120, 2048), ("lm_head", 151936, 2048)]
BATCHES = [1, 2, 4, 8]
WORKSET = 300e6


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def call_bytes(R, K, B, group, zp):
    G = -(-K // group)
    n = R * K // 2 + R * G * 2 + B * K * 2 + B * R * 2
    if zp:
        n += R * G // 2
    return n


def weight_bytes(R, K, group, zp):
    return call_bytes(R, K, 0, group, zp)


def _capture(fn, dev):
    import torch
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fn()
    torch.cuda.synchronize(dev)
    return g


def time_replays(g, steps, warmup, dev):
    import torch
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / steps


def ours(steps, warmup, group, zp, dev):
    """Per (shape, B): microseconds per call of TritonPackedLinear.forward."""
    from types import SimpleNamespace as NS

    import torch
    from duplex import synth
    from duplex.streaming.triton_dequant_gemv import TritonPackedLinear
    gen = torch.Generator(device=dev).manual_seed(11)
    rows = []
    for name, R, K in SHAPES:
        copies = max(2, math.ceil(WORKSET / weight_bytes(R, K, group, zp)))
        lins = []
        for _ in range(copies):
            w = synth.linear_torch(gen, R, K, group, zp, dev)
            mod = NS(weight_packed=w["packed"], weight_scale=w["scale"], weight_zeros=w["zeros"],
                     weight_shape=torch.tensor([R, K]), bias=None)
            lins.append(TritonPackedLinear(mod, dev))
            del w, mod
        for B in BATCHES:
            x = torch.randn(B, K, device=dev, dtype=torch.float16, generator=gen)
            outs = [torch.empty(B, R, device=dev, dtype=torch.float16) for _ in lins]
            g = _capture(lambda: [lin.forward(x, out=o) for lin, o in zip(lins, outs)], dev)
            ms = time_replays(g, steps, warmup, dev)
            rows.append({"shape": name, "R": R, "K": K, "B": B,
                         "us_per_call": ms * 1e3 / copies, "copies": copies})
            del g, outs
        del lins
        torch.cuda.empty_cache()
    return rows


def reference_triton(steps, warmup):
    """The reference's Triton kernel in its own process; (rows, None) or (None, reason)."""
    if not (REF / "duplex" / "streaming" / "triton_dequant_gemv.py").exists():
        return None, "reference not installed in baseline/_ref"
    script = Path(__file__).resolve().parent / "ref_triton_bench.py"
    env = dict(os.environ, PYTHONPATH=str(REF))
    r = subprocess.run([sys.executable, str(script), "--steps", str(steps), "--warmup",
                        str(warmup)], capture_output=True, text=True, env=env, timeout=1200)
    if r.returncode != 0:
        tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
        return None, f"reference Triton arm failed: {tail[0][:200]}"
    return json.loads(r.stdout.strip().splitlines()[-1]), None


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    a = ap.parse_args(argv)
    peak, kind = peaks()
    metric = "config 1: dense int4 dequant-GEMV sweep (q, k/v, o, fused qkv, lm_head; B 1-8)"
    if a.impl == "reference":
        ref, why = reference_triton(a.steps, max(3, a.warmup))
        line = {"metric": metric, "impl": "reference", "unit": "GB/s", "higher_is_better": True}
        if ref is None:
            line["unavailable"] = why
        else:
            tot_b = sum(call_bytes(r["R"], r["K"], r["B"], 32, False) for r in ref)
            tot_t = sum(r["us_per_call"] for r in ref)
            line.update(value=tot_b / (tot_t * 1e3), sweep=ref,
                        note="the reference's TritonPackedLinear (Triton _dq_gemv_kernel, one "
                             "launch per row), group 32 symmetric, on this B200")
        print(json.dumps(line), flush=True)
        return 0

    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    W = max(3, a.warmup)
    main_rows = ours(a.steps, W, 128, True, dev)
    g32_rows = ours(a.steps, W, 32, False, dev)
    for r in main_rows:
        b = call_bytes(r["R"], r["K"], r["B"], 128, True)
        r["GBps"] = b / (r["us_per_call"] * 1e3)
        r["frac"] = r["GBps"] / peak
    ref, why = reference_triton(a.steps, W)
    for r in g32_rows:
        b = call_bytes(r["R"], r["K"], r["B"], 32, False)
        r["GBps"] = b / (r["us_per_call"] * 1e3)
        r["frac"] = r["GBps"] / peak
        if ref:
            m = next(x for x in ref if x["shape"] == r["shape"] and x["B"] == r["B"])
            r["ref_triton_us"] = m["us_per_call"]
            r["speedup_vs_ref_triton"] = m["us_per_call"] / r["us_per_call"]
    tot_b = sum(call_bytes(r["R"], r["K"], r["B"], 128, True) for r in main_rows)
    tot_t = sum(r["us_per_call"] for r in main_rows)
    line = {
        "metric": metric, "value": tot_b / (tot_t * 1e3), "unit": "GB/s (all calls of the sweep)",
        "n_gpus": 1, "steps": a.steps, "warmup": W, "higher_is_better": True,
        "dtype": "int4 weights x f16 activations, f32 accumulate", "data": "synthetic (seeded)",
        "config": {"workload": "config 1 dense int4 GEMV sweep", "format": "group 128 + zero points",
                   "batches": BATCHES, "shapes": [s[0] for s in SHAPES],
                   "l2": f"each replay cycles distinct weight copies (> {WORKSET / 1e6:.0f} MB)"},
        "peak": peak, "peak_kind": kind,
        "sweep": main_rows,
        "g32_symmetric": g32_rows,
        "reference_triton": ref if ref else {"unavailable": why},
    }
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.path.insert(0, str(ROOT / "qwen3-omni-duplex_b200"))
    raise SystemExit(main())
