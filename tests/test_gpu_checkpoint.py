"""GPU: a transformers >= 5 fused-expert Thinker MoE block replaced from a packed checkpoint
(fuse_packed_moe_blocks(..., checkpoint=...)) computes the layer of the oracle (the
reference's gather-bmm forward restated, fused_packed_moe.py:191-275) at 2e-3 max|y|."""

import numpy as np
import pytest
import torch

import oracle as O
from duplex import synth
from test_packed_checkpoint import checkpoint_tensors, tiny_thinker_moe

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("zero_key", [None, "weight_zero_point"])
def test_fused_expert_block_from_checkpoint_vs_oracle(cuda, zero_key):
    from duplex.streaming.fused_packed_moe import FusedPackedMoE, fuse_packed_moe_blocks
    E, H, I, k = 16, 256, 128, 4
    L = synth.moe_layer_np(seed=70, E=E, H=H, I=I, top_k=k, group=64,
                           zero_points=zero_key is not None, T=5)
    t = checkpoint_tensors(L, "thinker.model.layers.0.mlp", zero_key or "weight_zeros")
    model = tiny_thinker_moe(E=E, H=H, I=I, top_k=k)
    n = fuse_packed_moe_blocks(model, dtype=torch.float16, device=cuda, verbose=False,
                               checkpoint=t, prefix="thinker.model.")
    assert n == 1 and isinstance(model.layers[0].mlp, FusedPackedMoE)
    x = torch.from_numpy(L["x"]).to(cuda)
    y = model.layers[0].mlp(x.view(1, 5, H)).view(5, H).float().cpu().numpy()
    w, sel, _ = O.router(L["x"], L["gate_w"], k, True, None, "float16")
    ref = O.moe_experts(L["x"], sel, w, L["gu_packed"], L["gu_scale"], L["dn_packed"],
                        L["dn_scale"], L["gu_zeros"], L["dn_zeros"])
    assert np.abs(y - ref).max() <= 2e-3 * np.abs(ref).max()
    assert model.layers[0].mlp.device_errors() == 0
