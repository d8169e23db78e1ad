"""Clock-path stack: every int4 linear of Thinker layers [0, n) for one decode step.

The reference's clock path (src/duplex/streaming/clock.py:106-226) runs
Thinker[0:24] with `TritonPackedLinear` for q/k/v/o (`patch_attention_to_triton`,
clock.py:132-134) and `FusedPackedMoE` for the MoE, one token per 80 ms frame.
This module is the same chain of int4 linears with the attention core left out
(a decode token's attention output is replaced by the q projection it would
consume) and the two RMSNorms of a Qwen3 decoder layer kept (weightless), so
the hidden state stays finite through the stack:

    h  -> qkv = W_qkv . rms(h)                 (q 4096 | k 512 | v 512 rows, K 2048)
       -> h1  = h + W_o . qkv[:, :4096]        (K 4096)
       -> h'  = h1 + MoE(rms(h1))              (router + 128-expert top-8 int4 MoE)

By default the whole stack is ONE launch of the persistent clock-path kernel
(`duplex_stack_forward`: one CTA per SM, grid barriers between the phases of a
layer, weights streamed ahead across phases).  `fused=False` runs the same math
as 5 kernels per layer (fused qkv, o, router, gate|up, down) chained with
programmatic dependent launch.  `capture()` records a step in a CUDA graph and
`decode()` is the user-facing call: host -> device copy of the step's tokens,
graph replay, device -> host copy of the result.
"""

from __future__ import annotations

from types import SimpleNamespace as NS

import torch

from duplex import _lib, synth
from duplex.streaming.fused_packed_moe import FusedPackedMoE
from duplex.streaming.triton_dequant_gemv import TritonPackedLinear

RMS_EPS = 1e-6  # Thinker text config rms_norm_eps


def _linear(packed, scale, zeros, out_f, in_f, device):
    mod = NS(weight_packed=packed, weight_scale=scale, weight_zeros=zeros,
             weight_shape=torch.tensor([out_f, in_f]), bias=None)
    lin = TritonPackedLinear(mod, device)
    lin.pdl = True
    return lin


def _groups(K, group):
    return -(-K // group)


def linear_bytes(lin: TritonPackedLinear) -> int:
    """Algorithmic bytes of an int4 linear: nibbles, one 16-bit scale and (if present)
    one 4-bit zero point per (row, group)."""
    R, K, G = lin.out_features, lin.in_features, _groups(lin.in_features, lin.group)
    n = R * K // 2 + R * G * 2
    if lin.tiles.has_zeros:
        n += R * G // 2
    return n


def moe_bytes(moe: FusedPackedMoE, T: int = 1) -> int:
    """Algorithmic HBM bytes of one decode MoE layer at batch T=1: router weights,
    the 8 selected experts' nibbles + scales + zero points, token in and out."""
    E, H, I, k = moe.num_experts, moe.hidden, moe.inter, moe.top_k
    g_gu, g_dn = _groups(H, moe.group), _groups(I, moe.group)
    per = 2 * I * H // 2 + H * I // 2 + (2 * I * g_gu + H * g_dn) * 2
    if moe.has_zeros:
        per += (2 * I * g_gu + H * g_dn) // 2
    return E * H * moe.gate.weight.element_size() + k * per + 2 * T * H * 2


class Persistent:
    """Device-side layer descriptors and workspace of one `duplex_stack_forward` program."""

    def __init__(self, descs, has_attn, moe_residual, T, H, E, I, top_k, norm, qkv_R, q_dim,
                 group, has_zeros, dtype, rms_eps, device):
        arr = (_lib.StackLayer * len(descs))(*descs)
        raw = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
        self.desc = raw.to(device)
        self.n = len(descs)
        n = _lib.ctypes.c_size_t()
        _lib.call("duplex_stack_workspace_bytes", T, H, E, I, top_k, qkv_R, _lib.ctypes.byref(n))
        self.ws = torch.zeros(n.value, dtype=torch.uint8, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.args = (has_attn, moe_residual, T, H, E, I, top_k, norm, qkv_R, q_dim, group,
                     has_zeros, _lib.dtype_code(dtype), float(rms_eps))

    def run(self, x, out, wait_limit_cycles=0, test_flags=0):
        """Enqueue the launch for x [T, H] -> out.  wait_limit_cycles / test_flags are the
        C entry point's (0: waits bounded at about 2 s; bit 0 of test_flags: the first
        grid barrier cannot complete, for the timeout test)."""
        (has_attn, moe_res, T, H, E, I, top_k, norm, qkv_R, q_dim, group, hz, code,
         eps) = self.args
        _lib.call("duplex_stack_forward", _lib.ptr(self.desc), self.n, has_attn, moe_res,
                  _lib.ptr(x), _lib.ptr(out), code, code, hz, T, H, E, I, top_k, norm, qkv_R,
                  q_dim, group, eps, _lib.ptr(self.ws), self.ws.numel(), int(wait_limit_cycles),
                  int(test_flags), _lib.ptr(self.err), _lib.stream_of(x))
        return out

    def device_errors(self) -> int:
        v = int(self.err.item())
        self.err.zero_()
        return v


def gate_records(moe: FusedPackedMoE) -> torch.Tensor:
    """The router's gate matrix as the persistent kernel's gate records (built once,
    kept on the module)."""
    rec = getattr(moe, "_gate_records", None)
    w = moe.gate.weight
    if rec is None or rec[1] != (w.data_ptr(), w._version):
        E, H = w.shape
        n = _lib.ctypes.c_size_t()
        _lib.call("duplex_gate_records_bytes", E, H, _lib.ctypes.byref(n))
        buf = torch.empty(n.value, dtype=torch.uint8, device=w.device)
        src = _lib.aligned(w.detach())
        _lib.call("duplex_repack_gate_records", _lib.ptr(src), _lib.dtype_code(src.dtype), E, H,
                  _lib.ptr(buf), buf.numel(), _lib.stream_of(src))
        rec = (buf, (w.data_ptr(), w._version))
        moe._gate_records = rec
    return rec[0]


def _moe_desc(moe: FusedPackedMoE, qkv=None, o=None):
    if moe.dn_slices is None:
        raise _lib.DuplexError("the persistent stack needs the down K-slices: build the MoE "
                               "with stack=True (group 32, 64 or 128, dims multiples of 128)")
    g = moe.gate
    return _lib.StackLayer(
        qkv_tiles=None if qkv is None else qkv.tiles.buf.data_ptr(),
        o_tiles=None if o is None else o.tiles.buf.data_ptr(),
        gate_w=gate_records(moe).data_ptr(), gate_b=None if g.bias is None else g.bias.data_ptr(),
        gu_tiles=moe.gu_tiles.buf.data_ptr(), dn_tiles=moe.dn_slices.buf.data_ptr())


class MoEChain:
    """n MoE layers chained through the persistent kernel: x -> MoE(rms(x)) (+ x).
    The decode-MoE layer of config 0, repeated over distinct weights."""

    def __init__(self, moes, rms_eps=RMS_EPS, residual=False, T=1):
        m0 = moes[0]
        dev = m0.gu_tiles.buf.device
        self.moes = moes
        self.p = Persistent([_moe_desc(m) for m in moes], 0, 1 if residual else 0, T, m0.hidden,
                            m0.num_experts, m0.inter, m0.top_k, 1 if m0.norm_topk_prob else 0, 0,
                            0, m0.group, 1 if m0.has_zeros else 0, m0.gate.weight.dtype, rms_eps,
                            dev)

    def forward_into(self, x, out):
        return self.p.run(x, out)


class ClockLayer:
    def __init__(self, qkv: TritonPackedLinear, o: TritonPackedLinear, moe: FusedPackedMoE):
        self.qkv, self.o, self.moe = qkv, o, moe


class ClockStack:
    """Thinker layers [0, n) of the clock path on the B200 kernels (batch T <= 8)."""

    def __init__(self, layers, hidden=synth.THINKER_HIDDEN, q_dim=None, T=1, rms_eps=RMS_EPS,
                 device="cuda", dtype=torch.float16, fused=True):
        self.layers = layers
        self.fused = fused
        self._persist = None
        self.hidden, self.T, self.rms_eps = hidden, T, rms_eps
        self.qkv_dim = layers[0].qkv.out_features
        self.q_dim = q_dim or layers[0].o.in_features
        self.device, self.dtype = torch.device(device), dtype
        z = lambda n: torch.zeros(T, n, device=device, dtype=dtype)  # noqa: E731
        self.x_in, self.out = z(hidden), z(hidden)
        self.qkv_buf, self.h1, self.hA, self.hB = z(self.qkv_dim), z(hidden), z(hidden), z(hidden)
        for L in layers:
            L.moe.workspace(T, self.device)
        self.graph = None

    # ------------------------------------------------------------------ construction
    @classmethod
    def synthetic(cls, n_layers=24, seed=0, device="cuda", group=128, zero_points=True,
                  dtype=torch.float16, E=synth.THINKER_EXPERTS, H=synth.THINKER_HIDDEN,
                  I=synth.THINKER_MOE_INTER, top_k=synth.THINKER_ACTIVE,
                  n_q=synth.THINKER_Q_HEADS, n_kv=synth.THINKER_KV_HEADS, head_dim=synth.HEAD_DIM,
                  T=1, fused=True):
        """Seeded synthetic weights with the benchmark distributions, drawn on `device`."""
        gen = torch.Generator(device=device).manual_seed(seed)
        q, kv = n_q * head_dim, n_kv * head_dim
        layers = []
        for _ in range(n_layers):
            a = synth.linear_torch(gen, q + 2 * kv, H, group, zero_points, device, dtype)
            b = synth.linear_torch(gen, H, q, group, zero_points, device, dtype)
            m = synth.moe_layer_torch(gen, E, H, I, group, zero_points, device, dtype)
            qkv = _linear(a["packed"], a["scale"], a["zeros"], q + 2 * kv, H, device)
            o = _linear(b["packed"], b["scale"], b["zeros"], H, q, device)
            moe = FusedPackedMoE.from_stacked(m["gate_w"], m["gu_packed"], m["gu_scale"],
                                              m["dn_packed"], m["dn_scale"], top_k,
                                              gu_zeros=m["gu_zeros"], dn_zeros=m["dn_zeros"],
                                              dtype=dtype, device=device, stack=fused)
            layers.append(ClockLayer(qkv, o, moe))
        return cls(layers, H, q, T, device=device, dtype=dtype, fused=fused)

    @classmethod
    def from_arrays(cls, arrays, top_k, device="cuda", dtype=torch.float16, T=1, group=None,
                    fused=True):
        """From per-layer dicts of numpy/torch arrays (used to check the stack against
        the oracle): keys qkv_packed/qkv_scale/qkv_zeros, o_*, gate_w, gu_*, dn_*."""
        t = lambda a: None if a is None else torch.as_tensor(a).to(device)  # noqa: E731
        layers = []
        for d in arrays:
            H = d["gate_w"].shape[1]
            qkv = _linear(t(d["qkv_packed"]), t(d["qkv_scale"]), t(d.get("qkv_zeros")),
                          d["qkv_packed"].shape[0], H, device)
            o = _linear(t(d["o_packed"]), t(d["o_scale"]), t(d.get("o_zeros")), H,
                        d["o_packed"].shape[1] * 8, device)
            moe = FusedPackedMoE.from_stacked(t(d["gate_w"]), t(d["gu_packed"]), t(d["gu_scale"]),
                                              t(d["dn_packed"]), t(d["dn_scale"]), top_k,
                                              gu_zeros=t(d.get("gu_zeros")),
                                              dn_zeros=t(d.get("dn_zeros")), dtype=dtype,
                                              device=device, stack=True)
            layers.append(ClockLayer(qkv, o, moe))
        H = arrays[0]["gate_w"].shape[1]
        return cls(layers, H, None, T, device=device, dtype=dtype, fused=fused)

    # ------------------------------------------------------------------ execution
    def bytes_per_step(self) -> int:
        n = 0
        for L in self.layers:
            n += linear_bytes(L.qkv) + linear_bytes(L.o) + moe_bytes(L.moe, self.T)
        return n

    def kernels_per_step(self) -> int:
        return 1 if self.fused else 5 * len(self.layers)

    def persistent(self) -> Persistent:
        if self._persist is None:
            m0 = self.layers[0].moe
            self._persist = Persistent(
                [_moe_desc(L.moe, L.qkv, L.o) for L in self.layers], 1, 1, self.T, self.hidden,
                m0.num_experts, m0.inter, m0.top_k, 1 if m0.norm_topk_prob else 0, self.qkv_dim,
                self.q_dim, m0.group, 1 if m0.has_zeros else 0, self.dtype, self.rms_eps,
                self.device)
        return self._persist

    def step_into(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Enqueue one decode step for x [T, H] on the current stream; result in out."""
        if self.fused:
            return self.persistent().run(x, out)
        h_in = x
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            h_out = out if i == n - 1 else (self.hA if i % 2 == 0 else self.hB)
            L.qkv.forward(h_in, out=self.qkv_buf, rms_eps=self.rms_eps)
            L.o.forward(self.qkv_buf[:, : self.q_dim], residual=h_in, out=self.h1,
                        x_row_stride=self.qkv_dim)
            L.moe.forward_into(self.h1, h_out, residual=self.h1, rms_eps=self.rms_eps)
            h_in = h_out
        return out

    def capture(self):
        """Record one step (x_in -> out) in a CUDA graph."""
        self.step_into(self.x_in, self.out)          # warm: workspaces, attributes
        torch.cuda.synchronize(self.device)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.step_into(self.x_in, self.out)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.graph = g
        return g

    def replay(self):
        self.graph.replay()

    def decode(self, x_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        """Public decode call with host buffers: H2D tokens, replay, D2H result.
        Asynchronous on the current stream when the host buffers are pinned."""
        if self.graph is None:
            self.capture()
        self.x_in.copy_(x_host, non_blocking=True)
        self.graph.replay()
        out_host.copy_(self.out, non_blocking=True)
        return out_host

    def device_errors(self) -> int:
        n = sum(L.moe.device_errors() for L in self.layers)
        if self._persist is not None:
            n += self._persist.device_errors()
        return n
