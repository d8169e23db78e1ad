"""Numpy restatement of the reference's int4 dequant / gather-bmm MoE path.

TEST INFRASTRUCTURE: imported only by tests, `__graft_entry__.smoke()` and the
CPU arms of `bench.py`.  Every function cites the reference line(s) it follows
(paths relative to the reference project root).

Dtypes are named by strings: "float32", "float16", "bfloat16".  numpy has no
bfloat16, so bf16 values are carried in float32 arrays whose values are exactly
bf16-representable (`round_to(x, "bfloat16")` rounds to nearest-even).

Packing order (compressed-tensors `pack_to_int32`, packed_dim=1, as restated by the
reference at `src/duplex/streaming/fused_packed_moe.py:54-65` and
`src/duplex/streaming/triton_dequant_gemv.py:12-14`): unpacked column `i + 8*m` is
nibble `i` (bits 4i..4i+3) of int32 word `m`.  A stored nibble is `q + 8` for the
symmetric format, i.e. the reference reads value = nibble - 8.

Zero points (no counterpart in the reference, which is symmetric): a `zeros`
tensor `[..., R, ceil(G/8)]` int32 packs one 4-bit zero point per (row, group) in the
same nibble order along the group axis; value = nibble - zero.  `zeros=None`
means zero == 8 everywhere, which reproduces the reference bit-exactly.
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

import numpy as np

__all__ = [
    "PACK", "round_to", "np_dtype", "pack4", "unpack_nibbles", "unpack4",
    "pack_zeros", "unpack_zeros", "dequant", "dequantize_weight", "router",
    "moe_experts", "moe_experts_by_expert", "moe_forward", "dequant_gemv", "packed_linear",
    "silu",
]

PACK = 8          # nibbles per int32 word (fused_packed_moe.py:33-34)
NUM_BITS = 4


# --------------------------------------------------------------------------- dtypes
def np_dtype(name: str):
    return {"float32": np.float32, "float16": np.float16,
            "bfloat16": np.float32, "float64": np.float64}[name]


def _round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), kept in float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    lsb = (u >> 16) & 1
    u = (u + 0x7FFF + lsb) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32)
    return np.where(nan, x, out).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round (once, to nearest-even) into `dtype`; bf16 stays in a float32 carrier."""
    if dtype == "bfloat16":
        return _round_bf16(np.asarray(x, dtype=np.float32))
    return np.asarray(x).astype(np_dtype(dtype))


# --------------------------------------------------------------------------- packing
def pack4(nibbles: np.ndarray) -> np.ndarray:
    """[..., 8C] values 0..15 -> [..., C] int32 in the reference packing order.

    Inverse of `unpack_nibbles`; restates compressed-tensors `pack_to_int32`
    (used by the reference's checkpoints, `quant/dequant.py:52-63`).
    """
    n = np.asarray(nibbles).astype(np.uint32) & 0xF
    *lead, cols = n.shape
    assert cols % PACK == 0, "pack4 needs a multiple of 8 columns"
    n = n.reshape(*lead, cols // PACK, PACK)
    shifts = (np.arange(PACK, dtype=np.uint32) * NUM_BITS)
    words = np.bitwise_or.reduce(n << shifts, axis=-1).astype(np.uint32)
    return words.view(np.int32)


def unpack_nibbles(packed: np.ndarray, out_cols: int) -> np.ndarray:
    """[..., C] int32 -> [..., out_cols] uint8 nibbles 0..15 (fused_packed_moe.py:62-64)."""
    p = np.asarray(packed).astype(np.int32).view(np.uint32)
    shifts = np.arange(PACK, dtype=np.uint32) * NUM_BITS
    u = (p[..., None] >> shifts) & 0xF                      # [..., C, 8]
    u = u.reshape(*p.shape[:-1], p.shape[-1] * PACK)
    return u[..., :out_cols].astype(np.uint8)


def unpack4(packed: np.ndarray, out_cols: int) -> np.ndarray:
    """Reference `unpack4` (fused_packed_moe.py:54-65): signed int4 in [-8, 7], int32."""
    return unpack_nibbles(packed, out_cols).astype(np.int32) - (1 << (NUM_BITS - 1))


def pack_zeros(z: np.ndarray) -> np.ndarray:
    """[..., R, G] zero points 0..15 -> [..., R, ceil(G/8)] int32 (pad groups with 0)."""
    z = np.asarray(z)
    G = z.shape[-1]
    gp = -(-G // PACK) * PACK
    if gp != G:
        pad = [(0, 0)] * (z.ndim - 1) + [(0, gp - G)]
        z = np.pad(z, pad)
    return pack4(z)


def unpack_zeros(zeros: np.ndarray, G: int) -> np.ndarray:
    return unpack_nibbles(zeros, G).astype(np.int32)


# --------------------------------------------------------------------------- dequant
def dequant(packed, scale, cols: int, zeros=None, scale_dtype: str | None = None):
    """`FusedPackedMoE._dequant` (fused_packed_moe.py:183-189), zero-point generalised.

    packed [..., R, C] int32, scale [..., R, G] -> [..., R, cols] in the scale dtype.
    q = nibble - zero is an exact small integer; q.to(dt) * scale is one rounding of
    the exact product into dt, which is what torch computes for f32/f16/bf16.
    The group size is inferred from scale.shape[-1] exactly as the reference does.
    """
    scale = np.asarray(scale)
    dt = scale_dtype or ("float16" if scale.dtype == np.float16 else
                         "float64" if scale.dtype == np.float64 else "float32")
    nib = unpack_nibbles(packed, cols).astype(np.int32)         # [..., R, cols]
    lead = nib.shape[:-1]
    G = scale.shape[-1]
    if cols % G != 0:
        raise ValueError(f"cols {cols} not divisible by {G} scale groups")
    if zeros is None:
        z = np.full(lead + (G,), 8, dtype=np.int32)
    else:
        z = unpack_zeros(zeros, G)
    q = nib.reshape(*lead, G, cols // G) - z[..., None]         # exact ints in [-15, 15]
    if dt == "float16":
        w = (q.astype(np.float32) * scale.astype(np.float32)[..., None]).astype(np.float16)
    elif dt == "bfloat16":
        w = _round_bf16(q.astype(np.float32) * scale.astype(np.float32)[..., None])
    elif dt == "float64":
        w = q.astype(np.float64) * scale.astype(np.float64)[..., None]
    else:
        w = q.astype(np.float32) * scale.astype(np.float32)[..., None]
    return w.reshape(*lead, cols)


def dequantize_weight(packed, scale, shape, dtype: str = "float32", zeros=None):
    """2-D `dequantize_weight` (quant/dequant.py:40-77): [out, in/8] + [out, G] -> [out, in].

    Mirrors the grouped branch (:67-74, scale is cast to `dtype` first) and the
    per-channel branch (:75-76).  Raises ValueError exactly where the reference does
    (:69-72, with its fixed GROUP_SIZE = 32 check).
    """
    out_f, in_f = (int(v) for v in shape)
    scale = np.asarray(scale)
    nib = unpack_nibbles(packed, in_f).astype(np.int32)
    if scale.ndim == 2 and scale.shape[1] > 1:
        G = scale.shape[1]
        if G * 32 < in_f:
            raise ValueError(f"scale groups {G} x 32 < in_features {in_f}")
        s = round_to(scale.astype(np.float32), dtype)
        z = np.full((out_f, G), 8, np.int32) if zeros is None else unpack_zeros(zeros, G)
        q = nib.reshape(out_f, G, -1) - z[..., None]
        w = round_to(q.astype(np.float32) * np.asarray(s, np.float32)[..., None], dtype)
        return w.reshape(out_f, -1)[:, :in_f]
    s = round_to(scale.astype(np.float32).reshape(-1, 1), dtype)
    q = nib - 8
    return round_to(q.astype(np.float32) * np.asarray(s, np.float32), dtype)


# --------------------------------------------------------------------------- router
def router(x, gate_w, top_k: int, norm_topk_prob: bool = True, gate_b=None,
           logits_dtype: str = "float32"):
    """Router of `FusedPackedMoE.forward` (fused_packed_moe.py:195-199).

    logits = gate(x) in the module dtype (nn.Linear: fp32-or-better accumulation,
    one rounding into the module dtype), softmax in fp32, top-k, renormalise.
    Selection is by logit value, descending, ties to the LOWER expert index
    (softmax is monotone, so this is the top-k of the fp32 probabilities).
    Returns (w [T, k] float32, sel [T, k] int64, logits [T, E] float32).
    """
    x = np.asarray(x, dtype=np.float64).reshape(-1, np.shape(x)[-1])
    W = np.asarray(gate_w, dtype=np.float64)
    lg = x @ W.T
    if gate_b is not None:
        lg = lg + np.asarray(gate_b, dtype=np.float64)
    lg = np.asarray(round_to(lg.astype(np.float32) if logits_dtype != "float64" else lg,
                             logits_dtype), dtype=np.float32)
    T, E = lg.shape
    # stable sort on (-logit) keeps the lower index first among equal logits
    order = np.argsort(-lg, axis=1, kind="stable")
    sel = order[:, :top_k].astype(np.int64)
    m = lg.max(axis=1, keepdims=True)
    p = np.exp((lg - m).astype(np.float32)).astype(np.float32)
    p = (p / p.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    w = np.take_along_axis(p, sel, axis=1)
    if norm_topk_prob:
        w = (w / w.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return w.astype(np.float32), sel, lg


def silu(v):
    v = np.asarray(v, dtype=np.float32)
    return (v / (np.float32(1.0) + np.exp(-v))).astype(np.float32)


# --------------------------------------------------------------------------- experts
def moe_experts(x, sel, w, gu_packed, gu_scale, dn_packed, dn_scale,
                gu_zeros=None, dn_zeros=None, compute: str = "float32"):
    """Torch gather-bmm forward (fused_packed_moe.py:265-275), expert half.

    x [T, H]; sel/w [T, k]; gu_packed [E, 2I, H/8]; dn_packed [E, H, I/8].
    gu = dequant(gu_packed[sel]) ; h = gu @ x ; act = silu(g) * u ;
    y = dequant(dn_packed[sel]) @ act ; out = sum_j w_j * y_j.
    `compute` is the module dtype of the fp32 oracle ("float32"), or "float64".
    Returns out [T, H] in the compute dtype.
    """
    ct = np_dtype(compute)
    x = np.asarray(x, dtype=np.float32).astype(ct)
    T, H = x.shape
    I2 = gu_packed.shape[-2]
    I = I2 // 2
    Ki = dn_packed.shape[-1] * PACK
    out = np.zeros((T, dn_packed.shape[-2]), dtype=ct)
    sdt = "float64" if compute == "float64" else "float32"
    for t in range(T):
        st = np.asarray(sel[t])
        gz = None if gu_zeros is None else gu_zeros[st]
        dz = None if dn_zeros is None else dn_zeros[st]
        gu = dequant(gu_packed[st], np.asarray(gu_scale[st], np.float32).astype(ct), H, gz, sdt)
        h = np.matmul(gu, x[t])                                     # [k, 2I]
        g, u = h[:, :I], h[:, I:]
        act = (g / (ct(1.0) + np.exp(-g))) * u                      # silu(g) * u
        dn = dequant(dn_packed[st], np.asarray(dn_scale[st], np.float32).astype(ct), Ki, dz, sdt)
        y = np.matmul(dn, act[:, :Ki, None])[..., 0]               # [k, H]
        out[t] = (y * np.asarray(w[t], dtype=ct)[:, None]).sum(axis=0)
    return out


def moe_experts_by_expert(x, sel, w, gu_packed, gu_scale, dn_packed, dn_scale,
                          gu_zeros=None, dn_zeros=None, threads=1):
    """`moe_experts` in fp32 with one dequantisation per selected expert, shared by every
    token that selects it (the reference's per-token loop of fused_packed_moe.py:265-275,
    reordered so that batches of hundreds of tokens finish in seconds).  Same values up
    to fp32 summation order: each token's slots are added in ascending expert order.
    `threads` > 1 computes the experts on a thread pool (numpy releases the GIL in its
    kernels); their outputs are still added in ascending expert order."""
    x = np.asarray(x, dtype=np.float32)
    sel = np.asarray(sel)
    w = np.asarray(w, dtype=np.float32)
    T, H = x.shape
    I = gu_packed.shape[-2] // 2
    Ki = dn_packed.shape[-1] * PACK
    out = np.zeros((T, dn_packed.shape[-2]), dtype=np.float32)

    def one(e):
        t_idx, j_idx = np.nonzero(sel == e)
        gz = None if gu_zeros is None else gu_zeros[e]
        dz = None if dn_zeros is None else dn_zeros[e]
        gu = dequant(gu_packed[e], np.asarray(gu_scale[e], np.float32), H, gz, "float32")
        h = x[t_idx] @ gu.T                                          # [n, 2I]
        g, u = h[:, :I], h[:, I:]
        act = (g / (np.float32(1.0) + np.exp(-g))) * u
        dn = dequant(dn_packed[e], np.asarray(dn_scale[e], np.float32), Ki, dz, "float32")
        return t_idx, (act[:, :Ki] @ dn.T) * w[t_idx, j_idx][:, None]   # [n, H]

    experts = np.unique(sel)
    if threads > 1:
        with ThreadPoolExecutor(threads) as pool:
            results = list(pool.map(one, experts))
    else:
        results = [one(e) for e in experts]
    for t_idx, y in results:
        np.add.at(out, t_idx, y)  # a token may list e twice
    return out


def moe_forward(x, gate_w, top_k, gu_packed, gu_scale, dn_packed, dn_scale,
                gu_zeros=None, dn_zeros=None, norm_topk_prob=True, gate_b=None,
                logits_dtype="float32", compute="float32"):
    """Whole `FusedPackedMoE.forward` torch path (fused_packed_moe.py:191-199,265-275)."""
    w, sel, _ = router(x, gate_w, top_k, norm_topk_prob, gate_b, logits_dtype)
    return moe_experts(x, sel, w, gu_packed, gu_scale, dn_packed, dn_scale,
                       gu_zeros, dn_zeros, compute), w, sel


# --------------------------------------------------------------------------- GEMV
def dequant_gemv(x, packed, scale, sel, zeros=None):
    """`dequant_gemv` semantics (triton_dequant_gemv.py:85-113; checker `reference_gemv`
    :116-122): y[j, r] = sum_c W[sel[j], r, c] * x_j[c] in fp32, W dequantised in fp32.

    x is [K] (shared by every selected expert) or [k, K] (one row per slot).
    Returns [k, R] float32.
    """
    sel = np.asarray(sel).reshape(-1)
    x = np.asarray(x, dtype=np.float32)
    K = x.shape[-1]
    z = None if zeros is None else np.asarray(zeros)[sel]
    W = dequant(np.asarray(packed)[sel], np.asarray(scale, np.float32)[sel], K, z, "float32")
    if x.ndim == 1:
        return np.matmul(W, x).astype(np.float32)
    return np.einsum("jrc,jc->jr", W, x, dtype=np.float32).astype(np.float32)


def packed_linear(x, packed, scale, zeros=None, bias=None, out_dtype: str = "float16"):
    """`TritonPackedLinear.forward` (triton_dequant_gemv.py:151-159): per row an fp32
    dequant-GEMV, then `.to(x.dtype)`, then `+ bias` in x dtype (two roundings)."""
    x = np.asarray(x, dtype=np.float32)
    lead, K = x.shape[:-1], x.shape[-1]
    flat = x.reshape(-1, K)
    W = dequant(np.asarray(packed)[None], np.asarray(scale, np.float32)[None], K,
                None if zeros is None else np.asarray(zeros)[None], "float32")[0]
    y = np.matmul(flat, W.T).astype(np.float32)
    y = round_to(y, out_dtype)
    if bias is not None:
        y = round_to(np.asarray(y, np.float32) + np.asarray(bias, np.float32), out_dtype)
    return np.asarray(y).reshape(*lead, W.shape[0])
