"""The no-allocation MoE entry point against the workspace entry point.

Some callers cannot call cudaMalloc for the MoE scratch: a real-time frame loop
(an allocation can synchronise the device and miss the 80 ms frame) or a C host
without a caching allocator.  `duplex_moe_forward_noalloc` serves them from a
static device array.  This file is collected last; it calls the entry point
twice in a row through the C ABI (different shapes, so the second call runs on
the first call's leftovers) and checks each result against `duplex_moe_forward`
on the same inputs, within the layer tolerance the other tests use.
"""

import ctypes

import numpy as np
import pytest
import torch

from duplex import _lib, synth

pytestmark = pytest.mark.gpu

TOL = 2e-3  # max|d| / max|y_ref|, as for every fp16 MoE layer test


def _module(dev, seed, E, H, I, k, group, zp, T):
    from duplex.streaming.fused_packed_moe import FusedPackedMoE
    L = synth.moe_layer_np(seed=seed, E=E, H=H, I=I, top_k=k, group=group, zero_points=zp, T=T)

    def t(a):
        return None if a is None else torch.from_numpy(a).to(dev)

    m = FusedPackedMoE.from_stacked(t(L["gate_w"]), t(L["gu_packed"]), t(L["gu_scale"]),
                                    t(L["dn_packed"]), t(L["dn_scale"]), k,
                                    gu_zeros=t(L["gu_zeros"]), dn_zeros=t(L["dn_zeros"]),
                                    dtype=torch.float16, device=dev)
    return m, t(L["x"])


def _noalloc_call(m, x, out, w, sel):
    g = m.gate
    return _lib.load().duplex_moe_forward_noalloc(
        _lib.ptr(x), _lib.DTYPE_F16, x.shape[0], _lib.ptr(g.weight), _lib.ptr(g.bias),
        m.num_experts, m.hidden, m.inter, m.top_k, 1 if m.norm_topk_prob else 0,
        _lib.ptr(m.gu_tiles.buf), _lib.ptr(m.dn_tiles.buf), m.gu_tiles.scale_code,
        1 if m.has_zeros else 0, m.group, None, _lib.ptr(out), _lib.ptr(w), _lib.ptr(sel),
        _lib.ptr(m.err), 0.0, 0, _lib.stream_of(x))


def _rel(a, b):
    a, b = a.float().cpu().numpy(), b.float().cpu().numpy()
    return np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)


def test_noalloc_matches_workspace_entry_on_two_calls(cuda):
    cases = [
        # Thinker geometry (config 0: 128 experts, hidden 2048, inter 768, top-8,
        # group 128 with zero points), one decode token
        dict(seed=31, E=128, H=2048, I=768, k=8, group=128, zp=True, T=1),
        # a smaller block with three tokens, run right after on the same scratch
        dict(seed=32, E=16, H=256, I=128, k=4, group=32, zp=False, T=3),
    ]
    for c in cases:
        m, x = _module(cuda, c["seed"], c["E"], c["H"], c["I"], c["k"], c["group"], c["zp"],
                       c["T"])
        ref = torch.empty(c["T"], c["H"], dtype=torch.float16, device=cuda)
        m.forward_into(x, ref)                       # workspace entry point
        got = torch.full_like(ref, float("nan"))
        w = torch.empty(c["T"], c["k"], dtype=torch.float32, device=cuda)
        sel = torch.empty(c["T"], c["k"], dtype=torch.int32, device=cuda)
        rc = _noalloc_call(m, x, got, w, sel)
        assert rc == 0, _lib.load().duplex_error_string(rc)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert _rel(got, ref) <= TOL
        w_ref, sel_ref = m.route(x)
        assert torch.equal(sel, sel_ref)
        assert m.device_errors() == 0


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    lib = _lib.load()
    limit = lib.duplex_moe_noalloc_scratch_bytes()
    need = ctypes.c_size_t()
    assert lib.duplex_moe_workspace_bytes(8, 256, 4096, 4096, 8, ctypes.byref(need)) == 0
    assert need.value > limit
    p = ctypes.c_void_p(1 << 20)
    rc = lib.duplex_moe_forward_noalloc(p, 0, 8, p, None, 256, 4096, 4096, 8, 1, p, p, 0, 1, 128,
                                        None, p, None, None, None, 0.0, 0, None)
    assert rc == 7  # DUPLEX_ERR_SCRATCH_LIMIT, before anything is launched
