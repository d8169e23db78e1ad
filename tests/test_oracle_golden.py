"""Pin the numpy oracle to the reference: golden vectors produced by running the
reference's own torch code (tests/golden/make_golden.py).  CPU only."""

import numpy as np
import pytest

import oracle as O
from duplex import synth


def load(golden_dir, name):
    return np.load(golden_dir / name)


def test_unpack4_matches_reference(golden_dir):
    g = load(golden_dir, "golden_unpack.npz")
    assert np.array_equal(O.unpack4(g["words"], 190), g["unpack4_190"])
    # compressed-tensors unpack equals the reference's unpack4 (fused_packed_moe.py:57-61)
    assert np.array_equal(g["ct_unpack"], g["unpack4_190"])


def test_pack4_round_trip(golden_dir):
    g = load(golden_dir, "golden_unpack.npz")
    nib = g["ct_unpack"][:, :184] + 8
    assert np.array_equal(O.pack4(nib), g["words"][:, :23])
    assert np.array_equal(O.pack4(g["ct_unpack"][:, :184] + 8), g["ct_pack"][:, :23])
    rng = np.random.default_rng(3)
    n = rng.integers(0, 16, size=(7, 64))
    assert np.array_equal(O.unpack_nibbles(O.pack4(n), 64), n)


@pytest.mark.parametrize("gname", ["g32", "g128"])
@pytest.mark.parametrize("dname,dt", [("f32", "float32"), ("f16", "float16"), ("bf16", "bfloat16")])
def test_dequant_bit_exact(golden_dir, gname, dname, dt):
    d = load(golden_dir, "golden_dequant.npz")
    s = O.round_to(d[f"{gname}_scale_f16"].astype(np.float32), dt)
    w = O.dequant(d[f"{gname}_packed"], s, 256, None, dt)
    assert np.array_equal(np.asarray(w, np.float32), d[f"{gname}_{dname}"])


@pytest.mark.parametrize("dname,dt", [("f32", "float32"), ("f16", "float16"), ("bf16", "bfloat16")])
def test_dequantize_weight_bit_exact(golden_dir, dname, dt):
    g = load(golden_dir, "golden_dequantize_weight.npz")
    w = O.dequantize_weight(g["packed"], g["scale"], (48, 256), dt)
    assert np.array_equal(np.asarray(w, np.float32), g[dname])


def test_dequantize_weight_group_error():
    with pytest.raises(ValueError):
        O.dequantize_weight(np.zeros((4, 32), np.int32), np.ones((4, 2), np.float16), (4, 256))


def test_zero_point_eight_is_reference(golden_dir):
    """nibble - z with z == 8 everywhere reproduces the symmetric reference exactly."""
    d = load(golden_dir, "golden_dequant.npz")
    pk, s = d["g32_packed"], d["g32_scale_f16"]
    z = O.pack_zeros(np.full(pk.shape[:-1] + (s.shape[-1],), 8))
    for dt in ("float32", "float16", "bfloat16"):
        s2 = O.round_to(s.astype(np.float32), dt)
        a = O.dequant(pk, s2, 256, None, dt)
        b = O.dequant(pk, s2, 256, z, dt)
        assert np.array_equal(np.asarray(a, np.float32), np.asarray(b, np.float32))


@pytest.mark.parametrize("g", [64, 128])
@pytest.mark.parametrize("dt", ["float16", "bfloat16", "float32"])
def test_zero_point_dequant_matches_compressed_tensors(golden_dir, g, dt):
    """value = (nibble - z) * scale, bit for bit against compressed-tensors' asymmetric
    group dequantisation (q - zp) * scale with q = nibble - 8, zp = z - 8
    (golden_zero_point_dequant.npz, made by make_zero_point_golden.py)."""
    d = load(golden_dir, "golden_zero_point_dequant.npz")
    s = O.round_to(d[f"g{g}_{dt}_scale"], dt)
    w = O.dequant(d[f"g{g}_packed"], s, 256, d[f"g{g}_zeros"], dt)
    assert np.array_equal(np.asarray(w, np.float32), d[f"g{g}_{dt}_w"])


def test_gemv_matches_reference_gemv(golden_dir):
    g = load(golden_dir, "golden_gemv.npz")
    y = O.dequant_gemv(g["x"], g["packed"], g["scale"], g["sel"])
    np.testing.assert_allclose(y, g["y"], rtol=0, atol=1e-6 * np.abs(g["y"]).max())


@pytest.mark.parametrize("group", [32, 128])
def test_moe_small_matches_reference(golden_dir, group):
    m = load(golden_dir, f"golden_moe_small_g{group}.npz")
    k = int(m["top_k"])
    w, sel, _ = O.router(m["x"], m["gate_w"], k, True, None, "float32")
    assert np.array_equal(sel, m["sel_f32"])
    np.testing.assert_allclose(w, m["w_f32"], rtol=1e-6, atol=1e-7)
    y = O.moe_experts(m["x"], sel, w, m["gu_packed"], m["gu_scale"], m["dn_packed"], m["dn_scale"])
    ymax = np.abs(m["y_f32"]).max()
    assert np.abs(y - m["y_f32"]).max() <= 1e-5 * ymax
    # fp16 module routing (fp16 logits) matches the reference's fp16 module too
    _, sel16, _ = O.router(m["x"], m["gate_w"], k, True, None, "float16")
    assert np.array_equal(sel16, m["sel_f16"])
    # and the reference's own fp16 path stays inside the tolerance this build uses
    assert np.abs(m["y_f16"] - m["y_f32"]).max() <= 2e-3 * ymax


@pytest.mark.parametrize("group", [128, 32])
def test_moe_thinker_geometry_matches_reference(golden_dir, group):
    """Config-0 geometry (128 experts, H 2048, I 768, top-8), symmetric format, seed 0."""
    m = load(golden_dir, f"golden_moe_thinker_g{group}.npz")
    L = synth.moe_layer_np(seed=int(m["seed"]), group=group, zero_points=False, T=1)
    w, sel, _ = O.router(L["x"], L["gate_w"], 8)
    assert np.array_equal(sel, m["sel_f32"])
    y = O.moe_experts(L["x"], sel, w, L["gu_packed"], L["gu_scale"], L["dn_packed"], L["dn_scale"])
    assert np.abs(y - m["y_f32"]).max() <= 1e-5 * np.abs(m["y_f32"]).max()


def test_router_tie_breaks_to_lower_index():
    x = np.ones((1, 8), np.float16)
    W = np.zeros((6, 8), np.float16)
    W[[1, 3, 4]] = 0.5        # three equal logits
    W[5] = 0.25
    w, sel, _ = O.router(x, W, 3)
    assert sel.tolist() == [[1, 3, 4]]
    np.testing.assert_allclose(w.sum(), 1.0, rtol=1e-6)


def test_packed_linear_two_roundings():
    rng = np.random.default_rng(5)
    d = synth.linear_np(rng, 48, 256, 128, True)
    x = rng.standard_normal((3, 256)).astype(np.float16)
    b = (rng.standard_normal(48) * 0.1).astype(np.float16)
    y = O.packed_linear(x, d["packed"], d["scale"], d["zeros"], b, "float16")
    acc = O.dequant_gemv(x[0], d["packed"][None], d["scale"][None], [0], d["zeros"][None])[0]
    ref = (acc.astype(np.float16).astype(np.float32) + b.astype(np.float32)).astype(np.float16)
    assert np.array_equal(y[0], ref)


def test_by_expert_oracle_is_the_per_token_oracle():
    """The expert-batched restatement gives the per-token forward (fp32 summation order
    aside), also when a token lists one expert in two slots."""
    L = synth.moe_layer_np(seed=9, E=8, H=128, I=64, top_k=3, group=32, zero_points=True, T=5)
    rng = np.random.default_rng(9)
    sel = np.stack([rng.choice(8, 3, replace=False) for _ in range(5)]).astype(np.int32)
    sel[2, 1] = sel[2, 0]
    w = rng.random((5, 3)).astype(np.float32)
    args = (L["gu_packed"], L["gu_scale"], L["dn_packed"], L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    a = O.moe_experts(L["x"], sel, w, *args)
    b = O.moe_experts_by_expert(L["x"], sel, w, *args)
    assert np.abs(a - b).max() <= 1e-5 * np.abs(a).max()
