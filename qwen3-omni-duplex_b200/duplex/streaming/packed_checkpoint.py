"""Packed int4 Thinker checkpoints -> the stacked expert layout of FusedPackedMoE.

The reference's checkpoint (compressed-tensors pack-quantized Qwen3-Omni) stores every
expert linear as a triplet `<layer>.mlp.experts.<i>.<gate|up|down>_proj.weight_{packed,
scale,shape}`: packed [R, K/8] int32 (nibble i of word m is column 8m + i), scale [R, K/g],
shape [2] = (R, K).  Its loader puts the triplets on per-expert Linear modules
(src/duplex/loader.py:31-55, src/duplex/streaming/clock.py:65-103), and
`fuse_packed_moe_blocks` stacks them from there (src/duplex/streaming/fused_packed_moe.py:
68-80, 117-123).  transformers >= 5 builds the Thinker MoE block with FUSED experts
(`experts.gate_up_proj` [E, 2I, H], `experts.down_proj` [E, H, I]) and a TopKRouter gate
(`gate.weight`, `gate.top_k`, `gate.norm_topk_prob`), so no per-expert module exists for
the triplets to land on, and the reference's loader drops them.  This module reads the
triplets straight from the checkpoint and stacks them per layer:

    ckpt = ShardedTensors("/path/to/model")            # lazy: model.safetensors.index.json
    for prefix in moe_prefixes(ckpt):                   # e.g. "thinker.model.layers.7.mlp"
        st = stack_layer(ckpt, prefix, dtype=torch.float16)
        moe = FusedPackedMoE.from_stacked(st["gate_weight"], st["gu_packed"], st["gu_scale"],
                                          st["dn_packed"], st["dn_scale"], top_k=8,
                                          gu_zeros=st["gu_zeros"], dn_zeros=st["dn_zeros"])

or `fuse_packed_moe_blocks(model, ..., checkpoint=ckpt, prefix="thinker.model.")`, which
also replaces the fused-expert blocks.  Optional zero points come in one of two forms:
  * `weight_zeros` (this build's): [R, ceil(G/8)] int32, nibble j of word m the zero
    point z of group 8m + j, value = (nibble - z) * scale;
  * `weight_zero_point` (compressed-tensors' asymmetric pack-quantized format): the
    signed zero point zp in [-8, 7] per (row, group), either packed as compressed-tensors
    writes it (`pack_to_int32(zp, 4, packed_dim=0)`: zp + 8 in nibble j of word m of
    row block m, [ceil(R/8), G] int32) or unpacked ([R, G]).  Its weights hold
    q = nibble - 8 and dequantise to (q - zp) * scale, which is (nibble - (zp + 8)) *
    scale, so z = zp + 8, converted here to the layout above.
Everything here is host-side tensor plumbing.
"""

from __future__ import annotations

import json
import re
from collections.abc import Mapping
from pathlib import Path

import torch

PROJS = ("gate_proj", "up_proj", "down_proj")
ZERO_KEYS = ("weight_zeros", "weight_zero_point")
_EXPERT = re.compile(r"^(?P<prefix>.+)\.experts\.(?P<i>\d+)\.gate_proj\.weight_packed$")


class ShardedTensors(Mapping):
    """Read-only mapping of tensor name -> tensor over a safetensors checkpoint: a single
    `.safetensors` file, or a directory with `model.safetensors.index.json` (its
    weight_map) or plain `*.safetensors` shards.  Tensors are read on access."""

    def __init__(self, path):
        from safetensors import safe_open
        self._open = safe_open
        p = Path(path)
        self._where: dict[str, Path] = {}
        if p.is_file():
            files = [p]
        elif (p / "model.safetensors.index.json").exists():
            wm = json.loads((p / "model.safetensors.index.json").read_text())["weight_map"]
            self._where = {k: p / v for k, v in wm.items()}
            files = []
        else:
            files = sorted(p.glob("*.safetensors"))
            if not files:
                raise FileNotFoundError(f"no safetensors checkpoint under {p}")
        for f in files:
            with safe_open(str(f), framework="pt") as h:
                for k in h.keys():
                    self._where[k] = f
        self._handles = {}

    def _handle(self, f: Path):
        h = self._handles.get(f)
        if h is None:
            h = self._open(str(f), framework="pt")
            self._handles[f] = h
        return h

    def __getitem__(self, key: str) -> torch.Tensor:
        f = self._where.get(key)
        if f is None:
            raise KeyError(key)
        return self._handle(f).get_tensor(key)

    def __iter__(self):
        return iter(self._where)

    def __len__(self):
        return len(self._where)


def moe_prefixes(tensors: Mapping) -> list[str]:
    """Every `<prefix>` with packed experts `<prefix>.experts.<i>.gate_proj.weight_packed`,
    in layer order (numbers compared as numbers)."""
    found = set()
    for k in tensors:
        m = _EXPERT.match(k)
        if m:
            found.add(m.group("prefix"))
    key = lambda s: [int(t) if t.isdigit() else t for t in re.split(r"(\d+)", s)]  # noqa: E731
    return sorted(found, key=key)


def pack_group_zeros(z: torch.Tensor) -> torch.Tensor:
    """[R, G] zero points in 0..15 -> [R, ceil(G/8)] int32, nibble j of word m = group 8m + j."""
    R, G = z.shape
    Gw = -(-G // 8)
    zz = torch.zeros(R, Gw * 8, dtype=torch.int64)
    zz[:, :G] = z.to(torch.int64) & 0xF
    words = (zz.view(R, Gw, 8) << (4 * torch.arange(8, dtype=torch.int64))).sum(-1)
    return torch.where(words >= 1 << 31, words - (1 << 32), words).to(torch.int32)


def zeros_from_compressed_tensors(zp: torch.Tensor, R: int, G: int) -> torch.Tensor:
    """compressed-tensors' `weight_zero_point` of an R-row linear with G groups -> this
    build's [R, ceil(G/8)] int32 layout.  Packed form: [ceil(R/8), G] int32 (zp + 8 in
    nibble j of word m = row 8m + j); unpacked form: [R, G] signed zero points."""
    zp = zp.to(torch.int64)
    if tuple(zp.shape) == (-(-R // 8), G) and R != -(-R // 8):
        shifts = 4 * torch.arange(8, dtype=torch.int64)
        nib = ((zp & 0xFFFFFFFF).unsqueeze(1) >> shifts.view(1, 8, 1)) & 0xF   # [R/8, 8, G]
        z = nib.reshape(-1, G)[:R]
    elif tuple(zp.shape) == (R, G):
        z = zp + 8
    else:
        raise ValueError(f"weight_zero_point of shape {tuple(zp.shape)} fits neither "
                         f"[{-(-R // 8)}, {G}] (packed) nor [{R}, {G}]")
    if int(z.min()) < 0 or int(z.max()) > 15:
        raise ValueError("weight_zero_point outside the 4-bit range")
    return pack_group_zeros(z)


def linear_zeros(mod):
    """A packed Linear's zero points in this build's [R, ceil(G/8)] int32 layout, on the
    module's device: `weight_zeros` as is, compressed-tensors' `weight_zero_point`
    converted (zeros_from_compressed_tensors), or None for a symmetric module."""
    z = getattr(mod, "weight_zeros", None)
    if z is not None:
        return z
    zp = getattr(mod, "weight_zero_point", None)
    if zp is None:
        return None
    s = mod.weight_scale
    R = int(mod.weight_shape[0]) if getattr(mod, "weight_shape", None) is not None \
        else int(mod.weight_packed.shape[0])
    G = s.shape[1] if s.dim() == 2 else 1
    return zeros_from_compressed_tensors(zp.cpu(), R, G).to(zp.device)


def _zeros(tensors: Mapping, base: str, R: int, G: int):
    if f"{base}.weight_zeros" in tensors:
        return tensors[f"{base}.weight_zeros"].to(torch.int32)
    if f"{base}.weight_zero_point" in tensors:
        return zeros_from_compressed_tensors(tensors[f"{base}.weight_zero_point"], R, G)
    return None


def _stack(tensors: Mapping, prefix: str, proj: str, E: int, dtype):
    packed, scale, zeros, shape = [], [], [], None
    for i in range(E):
        base = f"{prefix}.experts.{i}.{proj}"
        try:
            p, s = tensors[f"{base}.weight_packed"], tensors[f"{base}.weight_scale"]
        except KeyError as e:
            raise KeyError(f"{prefix}: expert {i} has no packed {proj} ({e})") from None
        shp = tuple(int(v) for v in tensors[f"{base}.weight_shape"].tolist()) \
            if f"{base}.weight_shape" in tensors else (p.shape[0], p.shape[1] * 8)
        if shape is None:
            shape = shp
        if shp != shape or p.shape != (shape[0], -(-shape[1] // 8)) or s.shape[0] != shape[0]:
            raise ValueError(f"{base}: packed {tuple(p.shape)}, scale {tuple(s.shape)}, shape "
                             f"{shp} disagree with expert 0's {shape}")
        packed.append(p.to(torch.int32))
        scale.append(s.to(dtype) if dtype is not None else s)
        zeros.append(_zeros(tensors, base, shape[0], s.shape[1]))
    if any(z is None for z in zeros) and not all(z is None for z in zeros):
        raise ValueError(f"{prefix}.{proj}: zero points on some experts only")
    z = None if zeros[0] is None else torch.stack(zeros)
    return torch.stack(packed), torch.stack(scale), z, shape


def stack_layer(tensors: Mapping, prefix: str, dtype=None) -> dict:
    """The stacked experts of one MoE layer (`<prefix>.experts.<i>.*`, `<prefix>.gate.weight`):

    gate_weight [E, H]; gu_packed [E, 2I, H/8] int32 (gate rows, then up rows, as the
    reference concatenates them, fused_packed_moe.py:120-121); gu_scale [E, 2I, H/g];
    dn_packed [E, H, I/8]; dn_scale [E, H, I/g]; gu_zeros / dn_zeros or None; E, H, I.
    Scales (and the gate) are cast to `dtype` when given."""
    E = 0
    while f"{prefix}.experts.{E}.gate_proj.weight_packed" in tensors:
        E += 1
    if E == 0:
        raise KeyError(f"no packed experts under {prefix!r}")
    gp, gs, gz, (I, H) = _stack(tensors, prefix, "gate_proj", E, dtype)
    up, us, uz, ushape = _stack(tensors, prefix, "up_proj", E, dtype)
    dp, ds, dz, dshape = _stack(tensors, prefix, "down_proj", E, dtype)
    if ushape != (I, H) or dshape != (H, I):
        raise ValueError(f"{prefix}: gate {(I, H)}, up {ushape}, down {dshape} do not form an MoE")
    if (gz is None) != (uz is None):
        raise ValueError(f"{prefix}: zero points on gate_proj or up_proj only")
    gw = tensors[f"{prefix}.gate.weight"]
    if tuple(gw.shape) != (E, H):
        raise ValueError(f"{prefix}.gate.weight is {tuple(gw.shape)}, expected {(E, H)}")
    return {
        "gate_weight": gw.to(dtype) if dtype is not None else gw,
        "gu_packed": torch.cat([gp, up], dim=1), "gu_scale": torch.cat([gs, us], dim=1),
        "gu_zeros": None if gz is None else torch.cat([gz, uz], dim=1),
        "dn_packed": dp, "dn_scale": ds, "dn_zeros": dz, "E": E, "H": H, "I": I,
    }


def fused_expert_sites(model, tensors: Mapping, prefix: str = "") -> list:
    """transformers >= 5 fused-expert MoE blocks of `model` whose packed experts are in
    `tensors` under `prefix + <module name>`: [(parent, attr, key prefix, top_k,
    norm_topk_prob)].  Blocks with per-expert modules are left to the reference's path."""
    sites = []
    for name, mod in model.named_modules():
        for attr, child in mod.named_children():
            if not type(child).__name__.endswith("SparseMoeBlock"):
                continue
            ex = getattr(child, "experts", None)
            if ex is None or not hasattr(ex, "gate_up_proj"):
                continue
            qual = f"{name}.{attr}" if name else attr
            key = prefix + qual
            if f"{key}.experts.0.gate_proj.weight_packed" not in tensors:
                continue
            gate = child.gate
            top_k = getattr(child, "top_k", None) or getattr(gate, "top_k")
            norm = getattr(child, "norm_topk_prob", getattr(gate, "norm_topk_prob", True))
            sites.append((mod, attr, key, int(top_k), bool(norm)))
    return sites
