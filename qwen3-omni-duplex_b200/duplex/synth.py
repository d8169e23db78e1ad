"""Seeded synthetic int4 weights and activations at Thinker geometry.

The reference ships no fixtures; its benches draw synthetic weights at the
model's geometry (`src/duplex/bench/clock.py:144-150`).  The distributions here
follow the benchmark configs: activations ~N(0,1), router weights ~N(0,0.02),
nibbles uniform 0..15 (so a packed int32 word is a uniform random 32-bit
pattern), scales |N(0,1)|*0.01 per group, zero points uniform 0..15 per group
(or absent: the reference's symmetric format, value = nibble - 8).

Two generators with the same distributions:
  * `moe_layer_np` / `linear_np`: numpy PCG64, bit-reproducible on any host, used
    for parity cases that a CPU checker must see;
  * `moe_layer_torch` / `linear_torch`: torch generator on the target device, used
    to fill many GB of benchmark weights quickly.
"""

from __future__ import annotations

import numpy as np

THINKER_HIDDEN = 2048      # reference src/duplex/config.py:14-21
THINKER_EXPERTS = 128
THINKER_ACTIVE = 8
THINKER_MOE_INTER = 768
THINKER_Q_HEADS = 32
THINKER_KV_HEADS = 4
HEAD_DIM = 128


def _ceil_div(a, b):
    return -(-a // b)


def _np_words(rng, shape):
    return rng.integers(0, 2**32, size=shape, dtype=np.uint64).astype(np.uint32).view(np.int32)


def linear_np(rng, R, K, group=128, zero_points=True, scale_dtype=np.float16):
    """One packed int4 linear [R, K]: dict(packed [R,K/8] i32, scale [R,G], zeros|None)."""
    G = _ceil_div(K, group)
    packed = _np_words(rng, (R, K // 8))
    scale = (np.abs(rng.standard_normal((R, G))) * 0.01).astype(scale_dtype)
    zeros = _np_words(rng, (R, _ceil_div(G, 8))) if zero_points else None
    if zeros is not None and G % 8:
        # keep the padding nibbles of the last word zero
        keep = np.uint32((1 << (4 * (G % 8))) - 1)
        z = zeros.view(np.uint32).copy()
        z[..., -1] &= keep
        zeros = z.view(np.int32)
    return dict(packed=packed, scale=scale, zeros=zeros, R=R, K=K, group=group)


def moe_layer_np(seed=0, E=THINKER_EXPERTS, H=THINKER_HIDDEN, I=THINKER_MOE_INTER,
                 top_k=THINKER_ACTIVE, group=128, zero_points=True, T=1,
                 x_dtype=np.float16, scale_dtype=np.float16):
    """A full MoE block's worth of seeded numpy tensors plus T input tokens."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((T, H)).astype(x_dtype)
    gate_w = (rng.standard_normal((E, H)) * 0.02).astype(x_dtype)
    gu = linear_np(rng, E * 2 * I, H, group, zero_points, scale_dtype)
    dn = linear_np(rng, E * H, I, group, zero_points, scale_dtype)

    def stack(d, R):
        z = None if d["zeros"] is None else d["zeros"].reshape(E, R, -1)
        return d["packed"].reshape(E, R, -1), d["scale"].reshape(E, R, -1), z

    gp, gs, gz = stack(gu, 2 * I)
    dp, ds, dz = stack(dn, H)
    return dict(x=x, gate_w=gate_w, gu_packed=gp, gu_scale=gs, gu_zeros=gz,
                dn_packed=dp, dn_scale=ds, dn_zeros=dz, E=E, H=H, I=I,
                top_k=top_k, group=group)


# ------------------------------------------------------------------ device generators
def _torch():
    import torch
    return torch


def _t_words(gen, shape, device):
    torch = _torch()
    return torch.randint(-2**31, 2**31 - 1, shape, generator=gen, device=device,
                         dtype=torch.int64).to(torch.int32)


def linear_torch(gen, R, K, group=128, zero_points=True, device="cuda",
                 scale_dtype=None, lead=()):
    """Same distributions as `linear_np`, drawn on `device` (leading dims `lead`)."""
    torch = _torch()
    scale_dtype = scale_dtype or torch.float16
    G = _ceil_div(K, group)
    packed = _t_words(gen, (*lead, R, K // 8), device)
    scale = (torch.randn((*lead, R, G), generator=gen, device=device).abs_() * 0.01).to(scale_dtype)
    zeros = None
    if zero_points:
        zeros = _t_words(gen, (*lead, R, _ceil_div(G, 8)), device)
        if G % 8:
            keep = (1 << (4 * (G % 8))) - 1
            zeros[..., -1] &= keep
    return dict(packed=packed, scale=scale, zeros=zeros, R=R, K=K, group=group)


def moe_layer_torch(gen, E=THINKER_EXPERTS, H=THINKER_HIDDEN, I=THINKER_MOE_INTER,
                    group=128, zero_points=True, device="cuda", dtype=None):
    torch = _torch()
    dtype = dtype or torch.float16
    gate_w = (torch.randn((E, H), generator=gen, device=device) * 0.02).to(dtype)
    gu = linear_torch(gen, 2 * I, H, group, zero_points, device, dtype, lead=(E,))
    dn = linear_torch(gen, H, I, group, zero_points, device, dtype, lead=(E,))
    return dict(gate_w=gate_w, gu_packed=gu["packed"], gu_scale=gu["scale"],
                gu_zeros=gu["zeros"], dn_packed=dn["packed"], dn_scale=dn["scale"],
                dn_zeros=dn["zeros"], E=E, H=H, I=I, group=group)
