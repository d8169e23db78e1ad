"""Fused int4 MoE on B200: router, gate|up, SiLU*up, down and combine in three kernels.

Drop-in for the reference module of the same name
(src/duplex/streaming/fused_packed_moe.py).  Same public names and contracts:

  unpack4(packed, out_cols)                                 (reference :54-65)
  _stack_packed(linears, dtype, device)                     (reference :68-80)
  FusedPackedMoE(block, dtype, device, host_resident, cpu_compute)   (:83-275)
      .forward(hidden_states) -> same shape and dtype
      ._dequant(packed, scale, cols)                        (:183-189)
  fuse_packed_moe_blocks(model, dtype, device, n_pinned, cpu_compute, verbose) -> int
                                                            (:278-319)

Differences, all deliberate:
  * `host_resident=True` (and `fuse_packed_moe_blocks(n_pinned=...)` for the layers past
    n_pinned) keeps the layer's expert tile records in mapped pinned host memory.  Each
    call stages only the planned experts into device slots with one kernel that reads
    host memory directly (`duplex_moe_forward_staged`).  The reference instead reads the
    selection back to the host and issues one copy per expert and token
    (fused_packed_moe.py:233-253).  Outputs are bit-identical to a resident layer.
    `cpu_compute` is recorded but nothing is computed on the CPU: a host-resident layer
    is staged and computed on the GPU;
  * batches of up to 8 tokens run as ONE pass (tokens that select the same expert
    share its weight stream) instead of a per-token Python loop; larger batches
    (batched decode of many streams, prefill chunks) run the grouped path, up to
    512 tokens per call: tokens sorted by expert, every selected expert's weights
    streamed once per 20 of its tokens;
  * optional 4-bit zero points (`weight_zeros` on the expert linears,
    [R, ceil(G/8)] int32, nibble order along the group axis); absent means the
    reference's symmetric format (value = nibble - 8);
  * activations must be fp16 or bf16 CUDA tensors; there is no CPU path.
"""

from __future__ import annotations

import ctypes
import gc

import torch
import torch.nn as nn

from duplex import _lib
from duplex.streaming.triton_dequant_gemv import (HAVE_TRITON, DownSlices, Int4Tiles,  # noqa: F401
                                                  TcRecords, dequant_gemv)

NUM_BITS = 4
PACK = 32 // NUM_BITS
GROUP = 32
GROUPED_MAX_TOKENS = 512    # tokens per duplex_moe_grouped call


def unpack4(packed: torch.Tensor, out_cols: int) -> torch.Tensor:
    """Unpack int32-packed signed int4 along the last dim -> int32 in [-8, 7]."""
    _lib.require_cuda(packed)
    p = _lib.aligned(packed.to(torch.int32))
    C = p.shape[-1]
    rows = p.numel() // C if C else 0
    out = torch.empty(*p.shape[:-1], out_cols, dtype=torch.int32, device=p.device)
    _lib.call("duplex_unpack4", _lib.ptr(p), rows, C, out_cols, _lib.ptr(out), _lib.stream_of(p))
    return out


def _stack_packed(linears, dtype, device):
    """Stack packed Linears into (packed, scale, out_features, in_features) (ref :68-80)."""
    l0 = linears[0]
    out_f, in_f = (int(v) for v in l0.weight_shape.tolist())
    E = len(linears)
    packed = torch.empty(E, out_f, l0.weight_packed.shape[1], dtype=torch.int32, device=device)
    scale = torch.empty(E, out_f, l0.weight_scale.shape[1], dtype=dtype, device=device)
    for i, lin in enumerate(linears):
        packed[i] = lin.weight_packed.to(device)
        scale[i] = lin.weight_scale.to(device, dtype)
    return packed, scale, out_f, in_f


def _stack_zeros(linears, device):
    """Zero points of the stacked linears in this build's [R, ceil(G/8)] int32 layout:
    `weight_zeros` as is, or compressed-tensors' asymmetric `weight_zero_point` converted
    (packed_checkpoint.zeros_from_compressed_tensors); None for symmetric linears."""
    from duplex.streaming.packed_checkpoint import linear_zeros
    zs = [linear_zeros(lin) for lin in linears]
    if all(z is None for z in zs):
        return None
    if any(z is None for z in zs):
        raise _lib.DuplexError("zero points on some experts only")
    return torch.stack([z.to(device, torch.int32) for z in zs])


class HostRecords:
    """Tile records moved into mapped pinned host memory (duplex_host_alloc): the GPU
    reads them over the host link at `dev_ptr`; no device copy is kept."""

    def __init__(self, dev_buf: torch.Tensor):
        n = dev_buf.numel()
        h, d = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.call("duplex_host_alloc", n, ctypes.byref(h), ctypes.byref(d))
        self.host_ptr, self.dev_ptr, self.nbytes = h.value, d.value, n
        view = torch.frombuffer((ctypes.c_uint8 * n).from_address(h.value), dtype=torch.uint8)
        view.copy_(dev_buf)       # device -> host, synchronous

    def __del__(self):
        if getattr(self, "host_ptr", None):
            try:
                _lib.load().duplex_host_free(self.host_ptr)
            except Exception:     # interpreter shutdown: the process frees it anyway
                pass
            self.host_ptr = None


class FusedPackedMoE(nn.Module):
    """SparseMoeBlock replacement for int4-packed experts, on the B200 kernels."""

    def __init__(self, block: nn.Module = None, dtype=torch.bfloat16, device="cuda",
                 host_resident: bool = False, cpu_compute: bool = False, tc: bool = False,
                 stack: bool = False):
        super().__init__()
        if dtype not in (torch.float16, torch.bfloat16):
            raise _lib.DuplexError("FusedPackedMoE on B200 runs fp16 or bf16 modules")
        if host_resident and (tc or stack):
            raise _lib.DuplexError("host-resident layers run the staged decode path only "
                                   "(no tensor-core records, no clock-path stack)")
        self.host_resident = host_resident      # experts in mapped pinned host memory
        self.cpu_compute = cpu_compute and host_resident   # recorded; computed on the GPU
        self.pdl = True
        self.stack = stack                      # also build the down K-slices (clock-path stack)
        self.tc = tc                            # also build tensor-core records (batched decode,
                                                # a second copy of the experts; opt-in)
        if block is None:                       # filled by from_stacked()
            return
        experts = block.experts
        self.num_experts = len(experts)
        self.top_k = block.top_k
        self.norm_topk_prob = getattr(block, "norm_topk_prob", True)
        self.gate = block.gate.to(device=device, dtype=dtype)
        gp, gs, inter, hidden = _stack_packed([e.gate_proj for e in experts], dtype, device)
        up, us, _, _ = _stack_packed([e.up_proj for e in experts], dtype, device)
        dp, ds, hid_out, inter_in = _stack_packed([e.down_proj for e in experts], dtype, device)
        gz = _stack_zeros([e.gate_proj for e in experts], device)
        uz = _stack_zeros([e.up_proj for e in experts], device)
        dz = _stack_zeros([e.down_proj for e in experts], device)
        gu_p, gu_s = torch.cat([gp, up], dim=1), torch.cat([gs, us], dim=1)
        gu_z = None if gz is None else torch.cat([gz, uz], dim=1)
        del gp, up, gs, us
        self._install(gu_p, gu_s, gu_z, dp, ds, dz, inter, hidden, hid_out, inter_in)

    @classmethod
    def from_stacked(cls, gate_weight, gu_packed, gu_scale, dn_packed, dn_scale, top_k,
                     gu_zeros=None, dn_zeros=None, norm_topk_prob=True, gate_bias=None,
                     dtype=torch.float16, device="cuda", tc=False, stack=False,
                     host_resident=False):
        """Build from raw stacked tensors ([E,2I,H/8], [E,2I,G], [E,H,I/8], [E,H,G'])."""
        m = cls(None, dtype=dtype, device=device, tc=tc, stack=stack, host_resident=host_resident)
        E, H = gate_weight.shape
        m.num_experts, m.top_k, m.norm_topk_prob = E, top_k, norm_topk_prob
        m.gate = nn.Linear(H, E, bias=gate_bias is not None).to(device=device, dtype=dtype)
        with torch.no_grad():
            m.gate.weight.copy_(gate_weight)
            if gate_bias is not None:
                m.gate.bias.copy_(gate_bias)
        I = gu_packed.shape[1] // 2
        m._install(gu_packed.to(device), gu_scale.to(device, dtype),
                   None if gu_zeros is None else gu_zeros.to(device),
                   dn_packed.to(device), dn_scale.to(device, dtype),
                   None if dn_zeros is None else dn_zeros.to(device),
                   I, H, dn_packed.shape[1], dn_packed.shape[2] * PACK)
        return m

    @classmethod
    def from_checkpoint(cls, tensors, prefix, top_k, norm_topk_prob=True, dtype=torch.bfloat16,
                        device="cuda", tc=False, stack=False, host_resident=False):
        """Build from the packed triplets of one MoE layer in a checkpoint mapping (name ->
        tensor, e.g. duplex.streaming.packed_checkpoint.ShardedTensors): `<prefix>.experts.
        <i>.<gate|up|down>_proj.weight_{packed,scale,shape}` and `<prefix>.gate.weight`."""
        from duplex.streaming.packed_checkpoint import stack_layer
        st = stack_layer(tensors, prefix, dtype=dtype)
        return cls.from_stacked(st["gate_weight"], st["gu_packed"], st["gu_scale"], st["dn_packed"],
                                st["dn_scale"], top_k, gu_zeros=st["gu_zeros"],
                                dn_zeros=st["dn_zeros"], norm_topk_prob=norm_topk_prob,
                                dtype=dtype, device=device, tc=tc, stack=stack,
                                host_resident=host_resident)

    def _install(self, gu_p, gu_s, gu_z, dp, ds, dz, inter, hidden, hid_out, inter_in):
        """Repack the stacked experts once into tile records (gate and up blocks paired)."""
        if inter % 16 or hidden % 32 or inter_in % 32 or hid_out % 16:
            raise _lib.DuplexError("expert dims must satisfy inter % 16 == 0 and hidden, "
                                   "inter % 32 == 0 for the B200 kernels")
        G = gu_s.shape[-1]
        self.group = -(-hidden // G)
        if -(-inter_in // ds.shape[-1]) != self.group:
            raise _lib.DuplexError("gate|up and down must use the same group size")
        if (gu_z is None) != (dz is None):
            raise _lib.DuplexError("gate|up and down must both have or both lack zero points")
        self.gu_tiles = Int4Tiles(gu_p, gu_s, gu_z, group=self.group, K=hidden, pair_halves=True)
        self.dn_tiles = Int4Tiles(dp, ds, dz, group=self.group, K=inter_in)
        # the down projection as K-slice records for the persistent clock-path kernel
        # (a second copy of the down weights; opt-in)
        self.dn_slices = None
        if self.stack and DownSlices.supported(gu_p.shape[0], hid_out, inter_in, self.group):
            self.dn_slices = DownSlices(dp, ds, dz, group=self.group)
        # tensor-core records for batched decode (a second copy of the experts, in the
        # layout of the tcgen05 kernels), where the geometry allows them
        E = gu_p.shape[0]
        self.gu_tc = self.dn_tc = None
        if (self.tc and hid_out == hidden and inter_in == inter
                and TcRecords.supported(E, 2 * inter, hidden, self.group, pair_halves=True)
                and TcRecords.supported(E, hidden, inter, self.group)):
            self.gu_tc = TcRecords(gu_p, gu_s, gu_z, group=self.group, K=hidden, pair_halves=True)
            self.dn_tc = TcRecords(dp, ds, dz, group=self.group, K=inter_in)
        self.register_buffer("err", torch.zeros(1, dtype=torch.int32, device=gu_p.device),
                             persistent=False)
        self.inter, self.hidden, self.hid_out, self.inter_in = inter, hidden, hid_out, inter_in
        self.has_zeros = gu_z is not None
        self._ws = {}
        self.gu_host = self.dn_host = None
        if self.host_resident:
            # the records go to mapped pinned host memory; the device copies are dropped
            # (built on the GPU one layer at a time, so the spike is one layer's records)
            self.gu_host = HostRecords(self.gu_tiles.buf)
            self.dn_host = HostRecords(self.dn_tiles.buf)
            self.gu_tiles.buf = self.gu_tiles.buf.new_empty(0)
            self.dn_tiles.buf = self.dn_tiles.buf.new_empty(0)

    @staticmethod
    def _dequant(packed, scale, cols, zeros=None):
        """[..., R, C] int32 + [..., R, G] scale -> [..., R, cols] in scale dtype (ref :183-189),
        one rounding of the exact (nibble - zero) * scale product."""
        _lib.require_cuda(packed, scale, zeros)
        G = scale.shape[-1]
        if cols % G:
            raise _lib.DuplexError(f"cols {cols} not divisible by {G} scale groups")
        p = _lib.aligned(packed.to(torch.int32)[..., : cols // PACK])
        s = _lib.aligned(scale)
        z = None if zeros is None else _lib.aligned(zeros.to(torch.int32))
        out = torch.empty(*p.shape[:-1], cols, dtype=scale.dtype, device=p.device)
        rows = p.numel() // p.shape[-1]
        code = _lib.dtype_code(scale.dtype)
        _lib.call("duplex_dequant", _lib.ptr(p), _lib.ptr(s), code, _lib.ptr(z), rows, cols,
                  cols // G, _lib.ptr(out), code, _lib.stream_of(p))
        return out

    def workspace(self, T: int, device) -> torch.Tensor:
        ws = self._ws.get((T, device))
        if ws is None:
            n = _lib.ctypes.c_size_t()
            _lib.call("duplex_moe_workspace_bytes", T, self.num_experts, self.hidden, self.inter,
                      self.top_k, _lib.ctypes.byref(n))
            ws = torch.zeros(n.value, dtype=torch.uint8, device=device)
            self._ws[(T, device)] = ws
        return ws

    def grouped_supported(self) -> bool:
        """Whether the grouped path takes this layer's geometry (asked of the library:
        group a power of two >= 64, hidden and inter multiples of 64, one unit's working
        set within shared memory; down projection [hidden, inter])."""
        if self.hid_out != self.hidden or self.inter_in != self.inter:
            return False
        n = _lib.ctypes.c_size_t()
        rc = _lib.load().duplex_moe_grouped_workspace_bytes(
            1, self.num_experts, self.hidden, self.inter, self.top_k, self.group,
            1 if self.has_zeros else 0, _lib.ctypes.byref(n))
        return rc == 0

    # Measured on one B200 (Thinker geometry, g128 + zero points, fp16): the tcgen05 engine
    # takes 188 / 219 / 277 us per layer at 64 / 256 / 512 tokens, the mma.sync engine
    # 109 / 199 / 337 us, so the tensor cores pay off above about 320 tokens.
    TC_MIN_TOKENS = 320

    def grouped_engine(self, T: int) -> str:
        """The expert engine the grouped path takes for T tokens: "tc" (tcgen05 kernels on
        the tensor-core records, built with tc=True) above TC_MIN_TOKENS, else "mma"
        (mma.sync kernels on the tile records)."""
        return "tc" if self.gu_tc is not None and T > self.TC_MIN_TOKENS else "mma"

    def grouped_workspace(self, T: int, device, engine: str = "mma") -> torch.Tensor:
        key = ("grouped", engine, T, device)
        ws = self._ws.get(key)
        if ws is None:
            n = _lib.ctypes.c_size_t()
            fn = ("duplex_moe_grouped_tc_workspace_bytes" if engine == "tc"
                  else "duplex_moe_grouped_workspace_bytes")
            _lib.call(fn, T, self.num_experts, self.hidden, self.inter, self.top_k, self.group,
                      1 if self.has_zeros else 0, _lib.ctypes.byref(n))
            ws = torch.empty(n.value, dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    def forward_grouped_into(self, x, out, residual=None, w_out=None, sel_out=None,
                             logits=None, engine=None):
        """x [T<=512, H] -> out [T, H] (+ residual) through the grouped path, no host
        synchronisation.  logits: optional [T, E] fp32 router logits (already rounded to
        the module dtype) used in place of the gate.  engine: "tc", "mma" or None (the
        module's choice, grouped_engine)."""
        T = x.shape[0]
        if self.host_resident:
            raise _lib.DuplexError("a host-resident layer runs the staged path (forward, "
                                   "forward_into or forward_staged_into), 8 tokens per call")
        if T > GROUPED_MAX_TOKENS:
            raise _lib.DuplexError(f"grouped MoE takes at most {GROUPED_MAX_TOKENS} tokens")
        engine = engine or self.grouped_engine(T)
        if engine == "tc":
            if self.gu_tc is None:
                raise _lib.DuplexError("this layer has no tensor-core records (build with tc=True; "
                                       "group 128, hidden and inter multiples of 256)")
            fn, gu, dn, code = "duplex_moe_grouped_tc", self.gu_tc.buf, self.dn_tc.buf, self.gu_tc.scale_code
        else:
            fn, gu, dn, code = "duplex_moe_grouped", self.gu_tiles.buf, self.dn_tiles.buf, self.gu_tiles.scale_code
        ws = self.grouped_workspace(T, x.device, engine)
        g = self.gate
        lg = None if logits is None else _lib.aligned(logits.float())
        _lib.call(
            fn, _lib.ptr(x), _lib.dtype_code(x.dtype), T, _lib.ptr(g.weight),
            _lib.ptr(g.bias), _lib.ptr(lg), self.num_experts, self.hidden, self.inter,
            self.top_k, 1 if self.norm_topk_prob else 0, _lib.ptr(gu), _lib.ptr(dn), code,
            1 if self.has_zeros else 0, self.group, _lib.ptr(residual), _lib.ptr(out),
            _lib.ptr(w_out), _lib.ptr(sel_out), _lib.ptr(ws), ws.numel(), _lib.ptr(self.err),
            _lib.stream_of(x))
        return out

    def forward_into(self, x, out, residual=None, w_out=None, sel_out=None, rms_eps=0.0):
        """x [T<=8, H] -> out [T, H] (+ residual), no host synchronisation.  rms_eps > 0 routes
        and computes on the RMS-normalised x (clock-path stack).  A host-resident layer takes
        the staged path (forward_staged_into)."""
        if self.host_resident:
            return self.forward_staged_into(x, out, residual, w_out, sel_out, rms_eps)
        T = x.shape[0]
        ws = self.workspace(T, x.device)
        g = self.gate
        _lib.call(
            "duplex_moe_forward", _lib.ptr(x), _lib.dtype_code(x.dtype), T, _lib.ptr(g.weight),
            _lib.ptr(g.bias), self.num_experts, self.hidden, self.inter, self.top_k,
            1 if self.norm_topk_prob else 0, _lib.ptr(self.gu_tiles.buf),
            _lib.ptr(self.dn_tiles.buf), self.gu_tiles.scale_code, 1 if self.has_zeros else 0,
            self.group,
            _lib.ptr(residual), _lib.ptr(out), _lib.ptr(w_out), _lib.ptr(sel_out), _lib.ptr(ws),
            ws.numel(), _lib.ptr(self.err), float(rms_eps), 1 if self.pdl else 0,
            _lib.stream_of(x))
        return out

    def stage_buffer(self, T: int, device) -> torch.Tensor:
        """Device slots of a host-resident layer for T tokens (duplex_moe_stage_bytes: the
        staged plan and min(T * top_k, E) experts' records)."""
        key = ("stage", T, device)
        buf = self._ws.get(key)
        if buf is None:
            n = ctypes.c_size_t()
            _lib.call("duplex_moe_stage_bytes", T, self.num_experts, self.hidden, self.inter,
                      self.top_k, self.group, 1 if self.has_zeros else 0, ctypes.byref(n))
            buf = torch.empty(n.value, dtype=torch.uint8, device=device)
            self._ws[key] = buf
        return buf

    def forward_staged_into(self, x, out, residual=None, w_out=None, sel_out=None, rms_eps=0.0):
        """forward_into for a host-resident layer: route, stage the planned experts from
        host memory into device slots, run the expert kernels on them (no host
        synchronisation)."""
        if self.gu_host is None:
            raise _lib.DuplexError("this layer is GPU resident (build with host_resident=True)")
        T = x.shape[0]
        ws = self.workspace(T, x.device)
        stage = self.stage_buffer(T, x.device)
        g = self.gate
        _lib.call(
            "duplex_moe_forward_staged", _lib.ptr(x), _lib.dtype_code(x.dtype), T,
            _lib.ptr(g.weight), _lib.ptr(g.bias), self.num_experts, self.hidden, self.inter,
            self.top_k, 1 if self.norm_topk_prob else 0, self.gu_host.dev_ptr,
            self.dn_host.dev_ptr, self.gu_tiles.scale_code, 1 if self.has_zeros else 0,
            self.group, _lib.ptr(residual), _lib.ptr(out), _lib.ptr(w_out), _lib.ptr(sel_out),
            _lib.ptr(ws), ws.numel(), _lib.ptr(stage), stage.numel(), _lib.ptr(self.err),
            float(rms_eps), 1 if self.pdl else 0, _lib.stream_of(x))
        return out

    def route(self, hidden_states):
        """(w [T, k] fp32, sel [T, k] int32) exactly as the forward routes them."""
        x = _lib.aligned(hidden_states.reshape(-1, self.hidden))
        T = x.shape[0]
        w = torch.empty(T, self.top_k, dtype=torch.float32, device=x.device)
        sel = torch.empty(T, self.top_k, dtype=torch.int32, device=x.device)
        for t0 in range(0, T, 8):
            xs = x[t0:t0 + 8]
            ws = self.workspace(xs.shape[0], x.device)
            g = self.gate
            _lib.call("duplex_moe_route", _lib.ptr(xs), _lib.dtype_code(x.dtype), xs.shape[0],
                      _lib.ptr(g.weight), _lib.ptr(g.bias), self.num_experts, self.hidden,
                      self.top_k, 1 if self.norm_topk_prob else 0, _lib.ptr(w[t0:t0 + 8]),
                      _lib.ptr(sel[t0:t0 + 8]), _lib.ptr(ws), ws.numel(), 0.0, 0,
                      _lib.stream_of(x))
        return w, sel

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        _lib.require_cuda(hidden_states)
        shape = hidden_states.shape
        x = _lib.aligned(hidden_states.reshape(-1, shape[-1]))
        if x.dtype != self.gate.weight.dtype:
            x = x.to(self.gate.weight.dtype)
        T = x.shape[0]
        out = torch.empty(T, self.hid_out, dtype=x.dtype, device=x.device)
        if self.host_resident:
            for t0 in range(0, T, 8):
                self.forward_staged_into(x[t0:t0 + 8], out[t0:t0 + 8])
        elif T > 8 and self.grouped_supported():
            for t0 in range(0, T, GROUPED_MAX_TOKENS):
                self.forward_grouped_into(x[t0:t0 + GROUPED_MAX_TOKENS],
                                          out[t0:t0 + GROUPED_MAX_TOKENS])
        else:
            for t0 in range(0, T, 8):
                self.forward_into(x[t0:t0 + 8], out[t0:t0 + 8])
        return out.to(hidden_states.dtype).view(shape)

    def device_errors(self) -> int:
        """Read (and clear) the device error word: bit 1 = expert id out of range,
        bit 2 = a bounded wait timed out.  Synchronises."""
        v = int(self.err.item())
        self.err.zero_()
        return v


def fuse_packed_moe_blocks(model, dtype=torch.bfloat16, device="cuda",
                           n_pinned: int | None = None, cpu_compute: bool = False,
                           verbose: bool = True, checkpoint=None, prefix: str = "") -> int:
    """Replace every packed SparseMoeBlock with a FusedPackedMoE (reference :278-319).

    With `checkpoint` (a name -> tensor mapping of the packed checkpoint, e.g.
    packed_checkpoint.ShardedTensors) the fused-expert blocks of transformers >= 5, which
    have no per-expert modules to hold the packed triplets, are replaced too: their
    experts are stacked straight from the checkpoint keys `prefix + <block name>.experts.
    <i>.*` (packed_checkpoint.fused_expert_sites).

    n_pinned: the first n_pinned replaced blocks (checkpoint-built ones first) stay GPU
    resident and every later one is host-resident (FusedPackedMoE(host_resident=True)),
    as in the reference; None keeps every block on the GPU."""
    n_fused = 0
    if checkpoint is not None:
        from duplex.streaming.packed_checkpoint import fused_expert_sites
        for parent, attr, key, top_k, norm in fused_expert_sites(model, checkpoint, prefix):
            host = n_pinned is not None and n_fused >= n_pinned
            setattr(parent, attr, FusedPackedMoE.from_checkpoint(
                checkpoint, key, top_k, norm_topk_prob=norm, dtype=dtype, device=device,
                host_resident=host))
            n_fused += 1
            gc.collect()
        if n_fused and torch.cuda.is_available():
            torch.cuda.empty_cache()
    sites = []
    for parent in model.modules():
        for name, child in list(parent.named_children()):
            if type(child).__name__.endswith("SparseMoeBlock") and hasattr(child, "experts"):
                gp = getattr(child.experts[0], "gate_proj", None)
                if gp is not None and hasattr(gp, "weight_packed"):
                    sites.append((parent, name))
    n = 0
    for parent, name in sites:
        child = getattr(parent, name)
        host = n_pinned is not None and n_fused + n >= n_pinned
        setattr(parent, name, FusedPackedMoE(child, dtype, device, host_resident=host,
                                             cpu_compute=cpu_compute))
        child.experts = None
        del child
        gc.collect()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
        n += 1
        if verbose and n % 6 == 0:
            used = torch.cuda.memory_allocated() / 1024**3 if torch.cuda.is_available() else 0
            print(f"    fused {n}/{len(sites)} packed blocks, {used:.2f} GB", flush=True)
    n += n_fused
    if verbose:
        n_host = 0 if n_pinned is None else max(0, n - n_pinned)
        print(f"fused {n} packed MoE blocks ({n - n_host} GPU-resident, {n_host} host-resident; "
              "B200 kernels)")
    return n
