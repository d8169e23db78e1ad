"""The no-allocation MoE entry point against the workspace entry point.

Some callers cannot call cudaMalloc for the MoE scratch: a real-time frame loop
(an allocation can synchronise the device and miss the 80 ms frame) or a C host
without a caching allocator.  `duplex_moe_forward_noalloc` serves them from a
static device array.  This file is collected last.  It first fills that array
with a large call (8 tokens at Thinker geometry), then calls the entry point twice
in a row through the C ABI (different shapes, each running on the previous call's
leftovers) and checks each output, routing weights and expert ids against
`duplex_moe_forward` on the same inputs.  Both entry points run the same kernels
on the same scratch layout, so the results must be bit-identical.
"""

import ctypes

import pytest
import torch

from duplex import _lib, synth

pytestmark = pytest.mark.gpu

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


def _workspace_call(m, x):
    """duplex_moe_forward (the entry point with a caller workspace) on the same inputs."""
    T, k = x.shape[0], m.top_k
    ref = torch.empty(T, m.hidden, dtype=torch.float16, device=x.device)
    w = torch.empty(T, k, dtype=torch.float32, device=x.device)
    sel = torch.empty(T, k, dtype=torch.int32, device=x.device)
    m.forward_into(x, ref, w_out=w, sel_out=sel)
    return ref, w, sel


def test_noalloc_matches_workspace_entry_on_two_calls(cuda):
    big, xbig = _module(cuda, 30, 128, 2048, 768, 8, 128, True, 8)
    cases = [
        # Thinker geometry (config 0: 128 experts, hidden 2048, inter 768, top-8,
        # group 128 with zero points), one decode token
        dict(seed=31, E=128, H=2048, I=768, k=8, group=128, zp=True, T=1),
        # a smaller block with three tokens, run right after on the same scratch
        dict(seed=32, E=16, H=256, I=128, k=4, group=32, zp=False, T=3),
    ]
    # fill the shared scratch with the leftovers of a larger problem first
    junk = torch.empty(8, 2048, dtype=torch.float16, device=cuda)
    wj = torch.empty(8, 8, dtype=torch.float32, device=cuda)
    sj = torch.empty(8, 8, dtype=torch.int32, device=cuda)
    assert _noalloc_call(big, xbig, junk, wj, sj) == 0
    for c in cases:
        m, x = _module(cuda, c["seed"], c["E"], c["H"], c["I"], c["k"], c["group"], c["zp"],
                       c["T"])
        ref, w_ref, sel_ref = _workspace_call(m, x)
        got = torch.full_like(ref, float("nan"))
        w = torch.full((c["T"], c["k"]), float("nan"), dtype=torch.float32, device=cuda)
        sel = torch.full((c["T"], c["k"]), -1, dtype=torch.int32, device=cuda)
        rc = _noalloc_call(m, x, got, w, sel)
        assert rc == 0, _lib.load().duplex_error_string(rc)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)
        assert torch.equal(w, w_ref)
        assert torch.equal(sel, sel_ref)
        assert m.device_errors() == 0
    assert big.device_errors() == 0


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
