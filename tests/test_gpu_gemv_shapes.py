"""GPU parity of the dense int4 dequant-GEMV at the config-1 shapes (the Thinker's q,
k / v, o, the fused q|k|v of the clock path, and the lm_head) for B = 1, 2, 4, 8 rows,
group 128 with zero points, through `TritonPackedLinear.forward` (the reference's
`TritonPackedLinear.forward`, src/duplex/streaming/triton_dequant_gemv.py:151-159),
against the oracle's `packed_linear` on the same seeded inputs."""

import numpy as np
import pytest
import torch

import oracle as O
from duplex import synth

pytestmark = pytest.mark.gpu

TOL = 2e-3


@pytest.mark.parametrize("name,R,K", [("q", 4096, 2048), ("kv", 512, 2048), ("o", 2048, 4096),
                                      ("qkv", 5120, 2048), ("lm_head", 151936, 2048)])
def test_config1_shape_vs_oracle(cuda, name, R, K):
    from types import SimpleNamespace as NS
    from duplex.streaming.triton_dequant_gemv import TritonPackedLinear
    rng = np.random.default_rng(R + K)
    lin = synth.linear_np(rng, R, K, 128, True)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    mod = NS(weight_packed=t(lin["packed"]), weight_scale=t(lin["scale"]),
             weight_zeros=t(lin["zeros"]), weight_shape=torch.tensor([R, K]), bias=None)
    m = TritonPackedLinear(mod, cuda)
    x = rng.standard_normal((8, K)).astype(np.float16)
    ref = np.asarray(O.packed_linear(x, lin["packed"], lin["scale"], lin["zeros"], None,
                                     "float16"), np.float32)
    for B in (1, 2, 4, 8):
        got = m(t(x[:B])).float().cpu().numpy()
        r = ref[:B]
        assert got.shape == (B, R)
        assert np.isfinite(got).all()
        assert np.abs(got - r).max() <= TOL * np.abs(r).max(), (name, B)
        # fp32 summation order moves a row by ~1e-5 of max|y|: at most 2 fp16 ulp after rounding
        ulp = np.spacing(np.abs(r).astype(np.float16)).astype(np.float32)
        assert np.all(np.abs(got - r) <= 2 * ulp + 2e-5 * np.abs(r).max()), (name, B)
