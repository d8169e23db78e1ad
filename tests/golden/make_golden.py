"""Generate golden vectors by running the REFERENCE's own torch code.

Run in a container where the reference project is checked out (read-only):

    python tests/golden/make_golden.py --ref /path/to/qwen3-omni-duplex

It imports `duplex.streaming.fused_packed_moe` / `triton_dequant_gemv` /
`quant.dequant` from the reference's `src/`, forces the torch path
(`HAVE_TRITON = False`, because the Triton branch is taken even for CPU tensors,
fused_packed_moe.py:222), feeds it a duck-typed SparseMoeBlock built from seeded
synthetic tensors, and writes `golden_*.npz` next to this script.  The GPU box
never runs this; it only reads the committed `.npz` files.

compressed-tensors >= 0.15 moved `unpack_from_int32`; the reference's import at
quant/dequant.py:52-54 is shimmed to the new module so `dequantize_weight` runs.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _load_synth():
    p = REPO / "qwen3-omni-duplex_b200" / "duplex" / "synth.py"
    spec = importlib.util.spec_from_file_location("_duplex_synth", p)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _import_reference(ref_root: str):
    sys.path.insert(0, str(Path(ref_root) / "src"))
    # shim the moved compressed-tensors helper (quant/dequant.py:52-54)
    import compressed_tensors.compressors.pack_quantized.helpers as h
    name = "compressed_tensors.compressors.quantized_compressors.pack_quantized"
    if name not in sys.modules:
        parent = "compressed_tensors.compressors.quantized_compressors"
        if parent not in sys.modules:
            sys.modules[parent] = types.ModuleType(parent)
        mod = types.ModuleType(name)
        mod.unpack_from_int32 = h.unpack_from_int32
        sys.modules[name] = mod
    import duplex.streaming.fused_packed_moe as fpm
    import duplex.streaming.triton_dequant_gemv as tdg
    import duplex.quant.dequant as dq
    fpm.HAVE_TRITON = False
    return fpm, tdg, dq, h


def _block(torch, nn, layer, dtype_scale, top_k):
    """Duck-typed SparseMoeBlock (fused_packed_moe.py:108-123) from stacked arrays."""
    from types import SimpleNamespace as NS
    E, I, H = layer["E"], layer["I"], layer["H"]
    gp, gs = layer["gu_packed"], layer["gu_scale"]
    dp, ds = layer["dn_packed"], layer["dn_scale"]

    def lin(p, s, out_f, in_f):
        return NS(weight_packed=torch.from_numpy(np.ascontiguousarray(p)),
                  weight_scale=torch.from_numpy(np.ascontiguousarray(s)).to(dtype_scale),
                  weight_shape=torch.tensor([out_f, in_f]))

    experts = [NS(gate_proj=lin(gp[e, :I], gs[e, :I], I, H),
                  up_proj=lin(gp[e, I:], gs[e, I:], I, H),
                  down_proj=lin(dp[e], ds[e], H, I)) for e in range(E)]
    gate = nn.Linear(H, E, bias=False)
    with torch.no_grad():
        gate.weight.copy_(torch.from_numpy(layer["gate_w"].astype(np.float32)))
    return NS(experts=experts, top_k=top_k, norm_topk_prob=True, gate=gate)


def _route(torch, F, mod, x):
    """The reference's routing lines (fused_packed_moe.py:195-199), verbatim semantics."""
    w = F.softmax(mod.gate(x), dim=1, dtype=torch.float)
    w, sel = torch.topk(w, mod.top_k, dim=-1)
    if mod.norm_topk_prob:
        w = w / w.sum(dim=-1, keepdim=True)
    return w, sel


def moe_case(torch, nn, F, fpm, synth, seed, E, H, I, top_k, group, T, dtypes):
    layer = synth.moe_layer_np(seed=seed, E=E, H=H, I=I, top_k=top_k, group=group,
                               zero_points=False, T=T)
    out = dict(seed=np.int64(seed), E=np.int64(E), H=np.int64(H), I=np.int64(I),
               top_k=np.int64(top_k), group=np.int64(group), T=np.int64(T))
    for name, dt in dtypes:
        blk = _block(torch, nn, layer, torch.float16, top_k)
        mod = fpm.FusedPackedMoE(blk, dtype=dt, device="cpu")
        x = torch.from_numpy(layer["x"].astype(np.float32)).to(dt)
        with torch.no_grad():
            y = mod(x)
            w, sel = _route(torch, F, mod, x)
        out[f"y_{name}"] = y.float().numpy()
        out[f"w_{name}"] = w.float().numpy()
        out[f"sel_{name}"] = sel.numpy().astype(np.int64)
    return layer, out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("DUPLEX_REFERENCE"),
                    help="checkout of the reference project (or set DUPLEX_REFERENCE)")
    ap.add_argument("--skip-large", action="store_true")
    a = ap.parse_args()
    if not a.ref:
        ap.error("give --ref (or DUPLEX_REFERENCE): the reference checkout to run")

    import torch
    import torch.nn as nn
    import torch.nn.functional as F
    torch.manual_seed(0)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    fpm, tdg, dq, ct_helpers = _import_reference(a.ref)
    synth = _load_synth()
    rng = np.random.Generator(np.random.PCG64(1234))

    # ---- (1) unpack4 on random words, and compressed-tensors equivalence
    words = rng.integers(0, 2**32, size=(5, 24), dtype=np.uint64).astype(np.uint32).view(np.int32)
    up = fpm.unpack4(torch.from_numpy(words), 190).numpy()
    ct = ct_helpers.unpack_from_int32(torch.from_numpy(words), 4, torch.Size([5, 190])).numpy()
    assert np.array_equal(up, ct.astype(up.dtype)), "unpack4 != unpack_from_int32"
    packed_back = ct_helpers.pack_to_int32(torch.from_numpy(ct.astype(np.int8)), 4).numpy()
    np.savez_compressed(HERE / "golden_unpack.npz", words=words, unpack4_190=up,
                        ct_unpack=ct.astype(np.int32), ct_pack=packed_back.astype(np.int32))

    # ---- (2) _dequant in three scale dtypes, two group sizes
    dq_out = {}
    for gname, G in (("g32", 8), ("g128", 2)):
        pk = rng.integers(0, 2**32, size=(3, 40, 32), dtype=np.uint64).astype(np.uint32).view(np.int32)
        sc = (np.abs(rng.standard_normal((3, 40, G))) * 0.01).astype(np.float16)
        dq_out[f"{gname}_packed"] = pk
        dq_out[f"{gname}_scale_f16"] = sc
        for dname, dt in (("f32", torch.float32), ("f16", torch.float16), ("bf16", torch.bfloat16)):
            s_t = torch.from_numpy(sc).to(dt)
            w = fpm.FusedPackedMoE._dequant(torch.from_numpy(pk), s_t, 256)
            dq_out[f"{gname}_{dname}"] = w.float().numpy()
    np.savez_compressed(HERE / "golden_dequant.npz", **dq_out)

    # ---- (3) dequantize_weight (2-D, compressed-tensors unpack) in three dtypes
    from types import SimpleNamespace as NS
    pk = rng.integers(0, 2**32, size=(48, 256 // 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
    sc = (np.abs(rng.standard_normal((48, 256 // 32))) * 0.01).astype(np.float16)
    m = NS(weight_packed=torch.from_numpy(pk), weight_scale=torch.from_numpy(sc),
           weight_shape=torch.tensor([48, 256]))
    dw = {"packed": pk, "scale": sc}
    for dname, dt in (("f32", torch.float32), ("f16", torch.float16), ("bf16", torch.bfloat16)):
        dw[dname] = dq.dequantize_weight(m, dtype=dt).float().numpy()
    np.savez_compressed(HERE / "golden_dequantize_weight.npz", **dw)

    # ---- (4) reference_gemv (E=1 dense and gathered), fp16 scales cast to fp32 inside
    E, R, K = 6, 96, 256
    pk = rng.integers(0, 2**32, size=(E, R, K // 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
    sc = (np.abs(rng.standard_normal((E, R, K // 32))) * 0.01).astype(np.float16)
    x = rng.standard_normal(K).astype(np.float16)
    sel = np.array([4, 1, 5], dtype=np.int32)
    y = tdg.reference_gemv(torch.from_numpy(x), torch.from_numpy(pk), torch.from_numpy(sc),
                           torch.from_numpy(sel).long(), group=32).numpy()
    np.savez_compressed(HERE / "golden_gemv.npz", packed=pk, scale=sc, x=x, sel=sel, y=y)

    # ---- (5) MoE forward, small geometry (inputs stored), fp32 and fp16 modules
    dts = [("f32", torch.float32), ("f16", torch.float16)]
    for group in (32, 128):
        layer, out = moe_case(torch, nn, F, fpm, synth, 7 + group, 16, 256, 128, 4, group, 3, dts)
        for k in ("x", "gate_w", "gu_packed", "gu_scale", "dn_packed", "dn_scale"):
            out[k] = layer[k]
        np.savez_compressed(HERE / f"golden_moe_small_g{group}.npz", **out)

    # ---- (6) MoE forward at Thinker geometry (config-0 shapes, symmetric format).
    # Inputs are NOT stored (300 MB); `duplex.synth.moe_layer_np(seed, ...)` regenerates them.
    if not a.skip_large:
        for group in (128, 32):
            _, out = moe_case(torch, nn, F, fpm, synth, 0, 128, 2048, 768, 8, group, 1,
                              [("f32", torch.float32)])
            np.savez_compressed(HERE / f"golden_moe_thinker_g{group}.npz", **out)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
