"""The reference's own GPU kernel on this B200, for the config-1 line (gemv_bench.py).

Run as a script with the reference's package first on PYTHONPATH (baseline/_ref):
`import duplex` is then the reference, not this repository.  For every config-1 shape
and B = 1, 2, 4, 8 it times the reference's `TritonPackedLinear.forward` (its Triton
`_dq_gemv_kernel`, one launch per row, then a stack and a cast;
src/duplex/streaming/triton_dequant_gemv.py:125-159) on random group-32 symmetric
weights (the only format that kernel reads), cycling distinct weight copies (> 300 MB)
inside one CUDA graph, as gemv_bench.py times this repository's kernel.  Prints one
JSON list.  Triton's compiled cache is left unread.
"""

import argparse
import json
import math
from types import SimpleNamespace as NS

import torch

SHAPES = [("q", 4096, 2048), ("k", 512, 2048), ("v", 512, 2048), ("o", 2048, 4096),
          ("qkv", 5120, 2048), ("lm_head", 151936, 2048)]
BATCHES = [1, 2, 4, 8]
WORKSET = 300e6


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args()
    from duplex.streaming.triton_dequant_gemv import TritonPackedLinear  # the reference's
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(11)
    rows = []
    for name, R, K in SHAPES:
        wbytes = R * K // 2 + R * (K // 32) * 2
        copies = max(2, math.ceil(WORKSET / wbytes))
        lins = []
        for _ in range(copies):
            packed = torch.randint(-2**31, 2**31 - 1, (R, K // 8), generator=gen, device=dev,
                                   dtype=torch.int64).to(torch.int32)
            scale = (torch.randn(R, K // 32, generator=gen, device=dev).abs_() * 0.01).half()
            mod = NS(weight_packed=packed, weight_scale=scale, weight_shape=torch.tensor([R, K]),
                     bias=None)
            lins.append(TritonPackedLinear(mod, dev))
            del packed, scale, mod
        for B in BATCHES:
            x = torch.randn(B, K, device=dev, dtype=torch.float16, generator=gen)
            outs = [None] * copies

            def run():
                for i, lin in enumerate(lins):
                    outs[i] = lin(x)

            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                run()                       # compiles the kernel on the first shape
            torch.cuda.current_stream(dev).wait_stream(s)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                run()
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
            rows.append({"shape": name, "R": R, "K": K, "B": B, "us_per_call": ms * 1e3 / copies,
                         "copies": copies})
            del g
        del lins
        torch.cuda.empty_cache()
    print(json.dumps(rows), flush=True)


if __name__ == "__main__":
    main()
