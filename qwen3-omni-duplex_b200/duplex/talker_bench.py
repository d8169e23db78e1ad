"""Talker MoE line (`bench.py --workload talker`): the Talker's MoE block (the reference's
FusedMoE, src/duplex/streaming/fused_moe.py:40-141) at its geometry -- 128 experts,
hidden 1024, expert inter 384, top-8, norm_topk_prob off, a shared expert of inter 2048
(the config's dense intermediate size; the checkpoint sets the real one) with its
sigmoid gate -- for T = 1 and 8 tokens, bf16 weights and the reference's q8 int8 format.

20 distinct layers (the Talker's depth; ~634 MB of bf16 weights, far beyond the 126 MB
L2) run back to back in one CUDA graph; µs per layer = replay time / 20.  GB/s counts the
bytes a layer must read: the router, the selected experts' rows (8 distinct experts
per token; at T = 8 the distinct experts of the seeded routing), their int8 scales, the
shared expert, and the tokens in and out.

When the reference is installed in baseline/_ref, its own FusedMoE.forward (torch gather
+ bmm on the GPU) is timed on the same B200 on the same shapes, in its own process
(`--reference`), graph-captured the same way.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
REF = ROOT / "baseline" / "_ref"
E, H, I, S, K, LAYERS = 128, 1024, 384, 2048, 8, 20


def layer_tensors(gen, dev, dt):
    import torch
    r = lambda *s, sc=0.04: (torch.randn(*s, generator=gen, device=dev) * sc).to(dt)  # noqa: E731
    return {"gate_w": r(E, H, sc=0.03), "gate_up": r(E, 2 * I, H), "down": r(E, H, I),
            "sh_gate": r(S, H), "sh_up": r(S, H), "sh_down": r(H, S), "sgw": r(1, H)}


def layer_bytes(distinct, q8):
    eb = 1 if q8 else 2
    n = E * H * 2 + distinct * 3 * I * H * eb + 3 * S * H * 2 + H * 2
    if q8:
        n += distinct * (2 * I + H) * 2
    return n


def capture(fn, dev):
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


def time_graph(g, steps, warmup, dev):
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


def ours(steps, warmup, dev):
    import torch
    from duplex import _lib
    from duplex.streaming.fused_moe import quantize_q8
    dt = torch.bfloat16
    gen = torch.Generator(device=dev).manual_seed(5)
    layers = [layer_tensors(gen, dev, dt) for _ in range(LAYERS)]
    rows = []
    for q8 in (False, True):
        if q8:
            for L in layers:
                L["gq"], L["gs"] = quantize_q8(L["gate_up"])
                L["dq"], L["ds"] = quantize_q8(L["down"])
        for T in (1, 8):
            x = torch.randn(T, H, generator=gen, device=dev).to(dt)
            n = _lib.ctypes.c_size_t()
            _lib.call("duplex_talker_moe_workspace_bytes", T, E, H, I, K, S, _lib.ctypes.byref(n))
            ws = [torch.zeros(n.value, dtype=torch.uint8, device=dev) for _ in layers]
            err = torch.zeros(1, dtype=torch.int32, device=dev)
            outs = [torch.empty(T, H, dtype=dt, device=dev) for _ in layers]
            sel = torch.empty(T, K, dtype=torch.int32, device=dev)

            def run():
                s = _lib.stream_of(x)   # the capturing stream
                for L, w, o in zip(layers, ws, outs):
                    gu, dn = (L["gq"], L["dq"]) if q8 else (L["gate_up"], L["down"])
                    _lib.call("duplex_talker_moe_forward", _lib.ptr(x), _lib.dtype_code(dt), T,
                              _lib.ptr(L["gate_w"]), E, H, I, K, 0, _lib.ptr(gu), _lib.ptr(dn),
                              1 if q8 else 0, _lib.ptr(L.get("gs") if q8 else None),
                              _lib.ptr(L.get("ds") if q8 else None), _lib.ptr(L["sh_gate"]),
                              _lib.ptr(L["sh_up"]), _lib.ptr(L["sh_down"]), S, _lib.ptr(L["sgw"]),
                              _lib.ptr(o), None, _lib.ptr(sel), _lib.ptr(w), w.numel(),
                              _lib.ptr(err), s)
            g = capture(run, dev)
            ms = time_graph(g, steps, warmup, dev)
            # distinct experts of each layer's routing of x, averaged over the layers
            nd = [int(torch.topk((x.float() @ L["gate_w"].float().T).to(dt).float(), K,
                                 dim=-1).indices.unique().numel()) for L in layers]
            distinct = sum(nd) / len(nd)
            rows.append({"format": "q8" if q8 else "bf16", "T": T, "us_per_layer": ms * 1e3 / LAYERS,
                         "bytes_per_layer": layer_bytes(distinct, q8), "distinct_experts": distinct,
                         "device_errors": int(err.item())})
            del g
    return rows


def reference(steps, warmup):
    """The reference's FusedMoE on the GPU in its own process; (rows, None) or (None, why)."""
    if not (REF / "duplex" / "streaming" / "fused_moe.py").exists():
        return None, "reference not installed in baseline/_ref"
    env = dict(os.environ, PYTHONPATH=str(REF))
    r = subprocess.run([sys.executable, __file__, "--reference", "--steps", str(steps), "--warmup",
                        str(warmup)], capture_output=True, text=True, env=env, timeout=1500)
    if r.returncode != 0:
        tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
        return None, f"reference arm failed: {tail[0][:200]}"
    return json.loads(r.stdout.strip().splitlines()[-1]), None


def reference_main(steps, warmup):
    """Runs with the reference's package first on sys.path: `import duplex` is the reference."""
    from types import SimpleNamespace as NS

    import torch
    import torch.nn as nn
    from duplex.streaming.fused_moe import FusedMoE  # the reference's
    dev = torch.device("cuda", 0)
    dt = torch.bfloat16
    gen = torch.Generator(device=dev).manual_seed(5)

    class MLP(nn.Module):
        def __init__(self, g, u, d):
            super().__init__()
            self.gate_proj, self.up_proj, self.down_proj = (nn.Linear(1, 1, bias=False) for _ in range(3))
            self.gate_proj.weight, self.up_proj.weight, self.down_proj.weight = (
                nn.Parameter(t, requires_grad=False) for t in (g, u, d))

        def forward(self, x):
            return self.down_proj(torch.nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))

    rows = []
    for q8 in (False, True):
        mods = []
        for _ in range(LAYERS):
            L = layer_tensors(gen, dev, dt)
            gate = nn.Linear(H, E, bias=False).to(dev, dt)
            gate.weight = nn.Parameter(L["gate_w"], requires_grad=False)
            sg = nn.Linear(H, 1, bias=False).to(dev, dt)
            sg.weight = nn.Parameter(L["sgw"], requires_grad=False)
            experts = [NS(gate_proj=NS(weight=L["gate_up"][e, :I]), up_proj=NS(weight=L["gate_up"][e, I:]),
                          down_proj=NS(weight=L["down"][e])) for e in range(E)]
            blk = NS(experts=experts, top_k=K, norm_topk_prob=False, gate=gate,
                     shared_expert=MLP(L["sh_gate"], L["sh_up"], L["sh_down"]), shared_expert_gate=sg)
            mods.append(FusedMoE(blk, q8=q8))
            del L, experts, blk
        for T in (1, 8):
            x = torch.randn(1, T, H, generator=gen, device=dev).to(dt)
            outs = [None] * LAYERS

            def run():
                with torch.no_grad():
                    for i, m in enumerate(mods):
                        outs[i] = m(x)
            g = capture(run, dev)
            ms = time_graph(g, steps, warmup, dev)
            rows.append({"format": "q8" if q8 else "bf16", "T": T, "us_per_layer": ms * 1e3 / LAYERS})
            del g
        del mods
        torch.cuda.empty_cache()
    print(json.dumps(rows), flush=True)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--reference", action="store_true")
    a = ap.parse_args(argv)
    W = max(3, a.warmup)
    if a.reference:
        reference_main(a.steps, W)
        return 0
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak_p = ROOT / "MEASURED_PEAKS.json"
    peak = float(json.loads(peak_p.read_text())["hbm_gbs"]) if peak_p.exists() else 6650.0
    rows = ours(a.steps, W, dev)
    for r in rows:
        r["GBps"] = r["bytes_per_layer"] / (r["us_per_layer"] * 1e3)
        r["frac"] = r["GBps"] / peak
    ref, why = reference(a.steps, W)
    if ref:
        for r in rows:
            m = next(x for x in ref if x["format"] == r["format"] and x["T"] == r["T"])
            r["ref_us_per_layer"] = m["us_per_layer"]
            r["speedup_vs_ref"] = m["us_per_layer"] / r["us_per_layer"]
    head = next(r for r in rows if r["format"] == "bf16" and r["T"] == 1)
    line = {"metric": "Talker MoE layer (bf16 experts + shared expert), µs/layer @ batch 1",
            "value": head["us_per_layer"], "unit": "us/layer", "higher_is_better": False,
            "n_gpus": 1, "steps": a.steps, "warmup": W, "dtype": "bf16 (q8: int8 weights)",
            "data": "synthetic (seeded)",
            "config": {"workload": "Talker MoE, 20 distinct layers per graph replay", "experts": E,
                       "hidden": H, "moe_inter": I, "shared_inter": S, "top_k": K,
                       "l2": f"{LAYERS} distinct layers per replay (> 126 MB)"},
            "peak": peak, "rows": rows,
            "reference_fused_moe": ref if ref else {"unavailable": why}}
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    if "--reference" not in sys.argv:
        sys.path.insert(0, str(ROOT / "qwen3-omni-duplex_b200"))
    raise SystemExit(main())
