"""Packed-checkpoint plumbing (CPU): per-expert compressed-tensors triplets in sharded
safetensors files -> the stacked layout FusedPackedMoE takes, and detection of the
fused-expert MoE blocks transformers >= 5 builds (no per-expert modules; the reference's
loader, src/duplex/loader.py:31-55, drops their packed tensors)."""

import json
from types import SimpleNamespace as NS

import numpy as np
import pytest
import torch

import oracle as O
from duplex import synth
from duplex.streaming.packed_checkpoint import (ShardedTensors, fused_expert_sites, moe_prefixes,
                                                stack_layer)

PROJS = ("gate_proj", "up_proj", "down_proj")
pack_to_int32 = pytest.importorskip(
    "compressed_tensors.compressors.pack_quantized.helpers").pack_to_int32


def checkpoint_tensors(L, prefix, zero_key="weight_zeros"):
    """The per-expert triplets of one synthetic layer (synth.moe_layer_np) under `prefix`."""
    E, H, I = L["E"], L["H"], L["I"]
    t = {f"{prefix}.gate.weight": torch.from_numpy(L["gate_w"].copy())}
    for i in range(E):
        parts = {"gate_proj": (slice(0, I), "gu", (I, H)), "up_proj": (slice(I, 2 * I), "gu", (I, H)),
                 "down_proj": (slice(0, H), "dn", (H, I))}
        for proj, (rows, src, shape) in parts.items():
            base = f"{prefix}.experts.{i}.{proj}"
            t[f"{base}.weight_packed"] = torch.from_numpy(L[f"{src}_packed"][i, rows].copy())
            t[f"{base}.weight_scale"] = torch.from_numpy(L[f"{src}_scale"][i, rows].copy())
            t[f"{base}.weight_shape"] = torch.tensor(shape, dtype=torch.int64)
            if L[f"{src}_zeros"] is not None:
                zw = L[f"{src}_zeros"][i, rows].copy()        # this build's [R, ceil(G/8)]
                if zero_key == "weight_zeros":
                    t[f"{base}.weight_zeros"] = torch.from_numpy(zw)
                else:                                         # compressed-tensors' forms
                    G = L[f"{src}_scale"].shape[-1]
                    zp = torch.from_numpy(O.unpack_zeros(zw, G).astype(np.int8) - 8)
                    if zero_key == "weight_zero_point":
                        zp = pack_to_int32(zp, 4, packed_dim=0)
                    t[f"{base}.weight_zero_point"] = zp
    return t


def write_checkpoint(path, tensors, n_shards=2):
    from safetensors.torch import save_file
    keys = sorted(tensors)
    wm = {}
    for s in range(n_shards):
        part = {k: tensors[k].contiguous() for k in keys[s::n_shards]}
        name = f"model-{s + 1:05d}-of-{n_shards:05d}.safetensors"
        save_file(part, str(path / name))
        wm.update({k: name for k in part})
    (path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))


@pytest.mark.parametrize("zero_key", [None, "weight_zeros", "weight_zero_point",
                                      "weight_zero_point_unpacked"])
def test_sharded_checkpoint_stacks_to_the_module_layout(tmp_path, zero_key):
    layers = [synth.moe_layer_np(seed=40 + l, E=4, H=64, I=32, top_k=2, group=32,
                                 zero_points=zero_key is not None) for l in range(2)]
    tens = {}
    for l, L in enumerate(layers):
        tens.update(checkpoint_tensors(L, f"thinker.model.layers.{l}.mlp", zero_key or "weight_zeros"))
    tens["thinker.model.embed_tokens.weight"] = torch.zeros(8, 64)
    write_checkpoint(tmp_path, tens)
    ck = ShardedTensors(tmp_path)
    assert len(ck) == len(tens)
    pre = moe_prefixes(ck)
    assert pre == ["thinker.model.layers.0.mlp", "thinker.model.layers.1.mlp"]
    for L, p in zip(layers, pre):
        st = stack_layer(ck, p)
        assert (st["E"], st["H"], st["I"]) == (4, 64, 32)
        for k in ("gu_packed", "gu_scale", "dn_packed", "dn_scale"):
            assert np.array_equal(st[k].numpy(), L[k]), k
        assert np.array_equal(st["gate_weight"].numpy(), L["gate_w"])
        if zero_key is None:
            assert st["gu_zeros"] is None and st["dn_zeros"] is None
        else:
            assert np.array_equal(st["gu_zeros"].numpy(), L["gu_zeros"])
            assert np.array_equal(st["dn_zeros"].numpy(), L["dn_zeros"])
        assert stack_layer(ck, p, dtype=torch.float32)["gu_scale"].dtype == torch.float32


def test_layer_numbers_sort_as_numbers():
    t = {f"m.layers.{l}.mlp.experts.0.gate_proj.weight_packed": torch.zeros(1) for l in (10, 2, 1)}
    assert moe_prefixes(t) == ["m.layers.1.mlp", "m.layers.2.mlp", "m.layers.10.mlp"]


def test_inconsistent_experts_are_refused():
    L = synth.moe_layer_np(seed=3, E=3, H=64, I=32, top_k=2, group=32, zero_points=False)
    t = checkpoint_tensors(L, "p")
    bad = dict(t)
    bad["p.experts.1.up_proj.weight_packed"] = torch.zeros(16, 8, dtype=torch.int32)
    with pytest.raises(ValueError):
        stack_layer(bad, "p")
    missing = {k: v for k, v in t.items() if not k.startswith("p.experts.2.down_proj")}
    with pytest.raises(KeyError):
        stack_layer(missing, "p")
    with pytest.raises(KeyError):
        stack_layer(t, "q")


def tiny_thinker_moe(E=8, H=64, I=32, top_k=2):
    """A model holding transformers' own fused-expert Thinker MoE block at layers.0.mlp."""
    from transformers.models.qwen3_omni_moe import modeling_qwen3_omni_moe as m
    cfg = NS(num_experts=E, hidden_size=H, moe_intermediate_size=I, hidden_act="silu",
             num_experts_per_tok=top_k, norm_topk_prob=True)
    layer = torch.nn.Module()
    layer.mlp = m.Qwen3OmniMoeThinkerTextSparseMoeBlock(cfg)
    model = torch.nn.Module()
    model.layers = torch.nn.ModuleList([layer])
    return model


def test_fused_expert_blocks_of_transformers_are_found():
    model = tiny_thinker_moe()
    L = synth.moe_layer_np(seed=4, E=8, H=64, I=32, top_k=2, group=32, zero_points=True)
    t = checkpoint_tensors(L, "thinker.model.layers.0.mlp")
    sites = fused_expert_sites(model, t, prefix="thinker.model.")
    assert len(sites) == 1
    parent, attr, key, top_k, norm = sites[0]
    assert parent is model.layers[0] and attr == "mlp"
    assert key == "thinker.model.layers.0.mlp" and top_k == 2 and norm is True
    assert fused_expert_sites(model, t, prefix="") == []   # keys under another prefix


@pytest.mark.parametrize("R,G", [(768, 16), (2048, 6), (13, 9), (1, 3)])
def test_compressed_tensors_zero_points_convert_to_the_group_layout(R, G):
    """compressed-tensors' asymmetric zero points (signed zp, packed over rows by its own
    pack_to_int32 or unpacked) -> this build's z = zp + 8, nibbles along the groups."""
    from duplex.streaming.fused_packed_moe import _stack_zeros
    from duplex.streaming.packed_checkpoint import zeros_from_compressed_tensors
    z = np.random.default_rng(R * 31 + G).integers(0, 16, (R, G))
    want = O.pack_zeros(z)
    zp = torch.from_numpy((z - 8).astype(np.int8))
    assert np.array_equal(zeros_from_compressed_tensors(zp, R, G).numpy(), want)
    if R > 1:
        packed = pack_to_int32(zp, 4, packed_dim=0)
        assert tuple(packed.shape) == (-(-R // 8), G)
        assert np.array_equal(zeros_from_compressed_tensors(packed, R, G).numpy(), want)
    lin = NS(weight_shape=torch.tensor([R, 8 * G]), weight_scale=torch.ones(R, G),
             weight_zero_point=zp)
    assert np.array_equal(_stack_zeros([lin, lin], "cpu").numpy(), np.stack([want, want]))
    with pytest.raises(ValueError):
        zeros_from_compressed_tensors(torch.zeros(R + 1, G + 1, dtype=torch.int32), R, G)


def test_linear_zeros_reads_either_key_and_refuses_mixed_experts():
    from duplex import _lib
    from duplex.streaming.fused_packed_moe import _stack_zeros
    from duplex.streaming.packed_checkpoint import linear_zeros
    R, G = 24, 4
    z = np.random.default_rng(3).integers(0, 16, (R, G))
    ours = torch.from_numpy(O.pack_zeros(z))
    ct = pack_to_int32(torch.from_numpy((z - 8).astype(np.int8)), 4, packed_dim=0)
    base = dict(weight_shape=torch.tensor([R, 8 * G]), weight_scale=torch.ones(R, G))
    a, b, sym = NS(weight_zeros=ours, **base), NS(weight_zero_point=ct, **base), NS(**base)
    assert linear_zeros(a) is ours
    assert torch.equal(linear_zeros(b), ours)
    assert linear_zeros(sym) is None and _stack_zeros([sym, sym], "cpu") is None
    assert torch.equal(_stack_zeros([a, b], "cpu"), torch.stack([ours, ours]))
    with pytest.raises(_lib.DuplexError):
        _stack_zeros([a, sym], "cpu")
