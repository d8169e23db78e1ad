"""Numpy restatement of one clock-path layer (TEST INFRASTRUCTURE / CPU baseline).

Composition follows the reference's clock path (src/duplex/streaming/clock.py:132-197):
the packed attention linears (`TritonPackedLinear.forward`,
triton_dequant_gemv.py:151-159) and `FusedPackedMoE.forward`
(fused_packed_moe.py:191-275) of one Thinker layer, with the attention core left
out and the decoder layer's RMSNorms kept weightless (Qwen3 RMSNorm semantics:
x.float() * rsqrt(mean(x^2) + eps), rounded back to the activation dtype).
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .moe_oracle import dequant, packed_linear, round_to, router


def rms_norm(x, eps, dtype="float16"):
    x32 = np.asarray(x, np.float32)
    var = (x32.astype(np.float64) ** 2).mean(axis=-1, keepdims=True)
    inv = (1.0 / np.sqrt(var + eps)).astype(np.float32)
    return np.asarray(round_to(x32 * inv, dtype), np.float32)


def _expert_pair(args):
    xt, e, w_e, gu_p, gu_s, gu_z, dn_p, dn_s, dn_z, H, I, act_dtype = args
    gu = dequant(gu_p[e], np.asarray(gu_s[e], np.float32), H,
                 None if gu_z is None else gu_z[e], "float32")
    h = gu @ xt
    g, u = h[:I], h[I:]
    act = np.asarray(round_to((g / (np.float32(1.0) + np.exp(-g))) * u, act_dtype), np.float32)
    dn = dequant(dn_p[e], np.asarray(dn_s[e], np.float32), I,
                 None if dn_z is None else dn_z[e], "float32")
    return w_e * (dn @ act)


def moe_layer(x, d, top_k, threads=1, logits_dtype="float16", act_dtype="float16"):
    """MoE of one layer for x [T, H] (fp32 experts, act rounded to the act dtype as in
    the reference's kernel path, fused_packed_moe.py:257).  `threads` parallelises the
    selected experts (numpy releases the GIL in its kernels)."""
    x = np.asarray(x, np.float32)
    T, H = x.shape
    I = d["gu_packed"].shape[1] // 2
    w, sel, _ = router(x, d["gate_w"], top_k, True, None, logits_dtype)
    out = np.zeros((T, d["dn_packed"].shape[1]), np.float32)
    pool = ThreadPoolExecutor(threads) if threads > 1 else None
    for t in range(T):
        jobs = [(x[t], int(sel[t, j]), np.float32(w[t, j]), d["gu_packed"], d["gu_scale"],
                 d.get("gu_zeros"), d["dn_packed"], d["dn_scale"], d.get("dn_zeros"), H, I,
                 act_dtype)
                for j in range(top_k)]
        ys = list(pool.map(_expert_pair, jobs)) if pool else [_expert_pair(j) for j in jobs]
        out[t] = np.sum(ys, axis=0)
    if pool:
        pool.shutdown()
    return out, sel


def clock_layer(h, d, top_k, eps=1e-6, dtype="float16", threads=1):
    """One clock-path layer: qkv(rms(h)) -> h1 = h + o(q) -> h' = h1 + MoE(rms(h1))."""
    h = np.asarray(h, np.float32)
    xn = rms_norm(h, eps, dtype)
    qkv = np.asarray(packed_linear(xn, d["qkv_packed"], d["qkv_scale"], d.get("qkv_zeros"),
                                   None, dtype), np.float32)
    q = qkv[:, : d["o_packed"].shape[1] * 8]
    o = np.asarray(packed_linear(q, d["o_packed"], d["o_scale"], d.get("o_zeros"), None, dtype),
                   np.float32)
    h1 = np.asarray(round_to(o + h, dtype), np.float32)
    y, sel = moe_layer(rms_norm(h1, eps, dtype), d, top_k, threads, dtype, dtype)
    return np.asarray(round_to(y + h1, dtype), np.float32), sel
