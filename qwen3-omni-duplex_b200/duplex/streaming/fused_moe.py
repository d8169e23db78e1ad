"""Talker MoE on B200: drop-in for the reference module of the same name
(src/duplex/streaming/fused_moe.py).  Same public names and contracts:

  FusedMoE(block, chunk=8, q8=False)          (reference :40-141)
      .forward(hidden_states) -> same shape and dtype
  fuse_moe_blocks(model, q8=False, verbose=True) -> int      (:144-178)

The block's experts are stacked once into gate_up [E, 2I, H] (gate rows, then up rows)
and down [E, H, I]; with `q8` they are stored as per-output-channel symmetric int8 with
scales amax / 127 in the module dtype, the reference's quantisation (:84-97).  The
forward -- router, the selected experts' gate|up, SiLU(gate) * up, down, the weighted sum
over the slots, plus the shared expert gated by sigmoid(shared_expert_gate(x)) (:136-140)
-- is one `duplex_talker_moe_forward` call per 8 tokens (csrc/talker.cu).

Differences, all deliberate:
  * `chunk` is accepted and recorded; the kernels take 8 tokens per call, so no dense
    [T, k, 2I, H] gather is ever materialised;
  * the shared expert's MLP must be the Qwen3 form (gate_proj, up_proj, down_proj,
    SiLU); its weights are read in place from the block's modules;
  * transformers >= 5 fused-expert blocks (`experts.gate_up_proj`, `experts.down_proj`,
    a TopKRouter gate) are accepted as well as per-expert ModuleLists;
  * activations must be fp16 or bf16 CUDA tensors; there is no CPU path.
"""

from __future__ import annotations

import gc

import torch
import torch.nn as nn

from duplex import _lib

TOKENS_PER_CALL = 8


def _stacked(block):
    """(gate_up [E, 2I, H], down [E, H, I]) of a block's experts, either layout."""
    ex = block.experts
    if hasattr(ex, "gate_up_proj"):              # transformers >= 5: already stacked
        return ex.gate_up_proj.detach(), ex.down_proj.detach()
    e0 = ex[0]
    inter, hidden = e0.gate_proj.weight.shape
    E = len(ex)
    gate_up = torch.empty(E, 2 * inter, hidden, dtype=e0.gate_proj.weight.dtype,
                          device=e0.gate_proj.weight.device)
    down = torch.empty(E, hidden, inter, dtype=e0.down_proj.weight.dtype,
                       device=e0.down_proj.weight.device)
    with torch.no_grad():
        for i, e in enumerate(ex):
            gate_up[i, :inter] = e.gate_proj.weight
            gate_up[i, inter:] = e.up_proj.weight
            down[i] = e.down_proj.weight
    return gate_up, down


def quantize_q8(w: torch.Tensor):
    """Per-output-channel symmetric int8 (the reference's q8, fused_moe.py:84-97):
    s = max|w| over the input dim / 127 (at least 1e-8 / 127), q = round(w / s) in
    [-127, 127]; returns (q int8, s in w's dtype, shape [..., R])."""
    s = w.abs().amax(dim=-1, keepdim=True).clamp_min(1e-8) / 127.0
    q = (w / s).round().clamp_(-127, 127).to(torch.int8)
    return q, s.to(w.dtype).squeeze(-1)


class FusedMoE(nn.Module):
    """Drop-in replacement for a (Talker) SparseMoeBlock, on the B200 kernels."""

    def __init__(self, block: nn.Module, chunk: int = 8, q8: bool = False):
        super().__init__()
        self.chunk = chunk
        self.q8 = q8
        gate = block.gate
        self.top_k = int(getattr(block, "top_k", None) or getattr(gate, "top_k"))
        self.norm_topk_prob = bool(getattr(block, "norm_topk_prob",
                                           getattr(gate, "norm_topk_prob", True)))
        self.gate = gate
        self.shared_expert = getattr(block, "shared_expert", None)
        self.shared_expert_gate = getattr(block, "shared_expert_gate", None)
        gate_up, down = _stacked(block)
        self.num_experts, two_i, self.hidden = gate_up.shape
        self.inter = two_i // 2
        if q8:
            gq, gs = quantize_q8(gate_up)
            dq, ds = quantize_q8(down)
            self.register_buffer("gate_up", gq.contiguous(), persistent=False)
            self.register_buffer("down", dq.contiguous(), persistent=False)
            self.register_buffer("gate_up_s", gs.contiguous(), persistent=False)
            self.register_buffer("down_s", ds.contiguous(), persistent=False)
        else:
            self.register_buffer("gate_up", gate_up.contiguous(), persistent=False)
            self.register_buffer("down", down.contiguous(), persistent=False)
            self.gate_up_s = self.down_s = None
        self.register_buffer("err", torch.zeros(1, dtype=torch.int32), persistent=False)
        self._ws = {}

    def _workspace(self, T, device):
        ws = self._ws.get((T, device))
        if ws is None:
            n = _lib.ctypes.c_size_t()
            S = self._shared_dims()[0]
            _lib.call("duplex_talker_moe_workspace_bytes", T, self.num_experts, self.hidden,
                      self.inter, self.top_k, S, _lib.ctypes.byref(n))
            ws = torch.zeros(n.value, dtype=torch.uint8, device=device)  # zero once (counter)
            self._ws[(T, device)] = ws
        return ws

    def _shared_dims(self):
        se = self.shared_expert
        if se is None:
            return 0, None, None, None
        return se.gate_proj.weight.shape[0], se.gate_proj.weight, se.up_proj.weight, se.down_proj.weight

    def forward_into(self, x: torch.Tensor, out: torch.Tensor, w_out=None, sel_out=None) -> None:
        """x, out [T <= 8, H] contiguous CUDA tensors in the module dtype."""
        _lib.require_cuda(x, out)
        T, H = x.shape
        dt = x.dtype
        S, g, u, d = self._shared_dims()
        sgw = None if self.shared_expert_gate is None else self.shared_expert_gate.weight
        ws = self._workspace(T, x.device)
        if self.err.device != x.device:
            self.err = self.err.to(x.device)
        _lib.call("duplex_talker_moe_forward", _lib.ptr(x), _lib.dtype_code(dt), T,
                  _lib.ptr(self.gate.weight), self.num_experts, H, self.inter, self.top_k,
                  1 if self.norm_topk_prob else 0, _lib.ptr(self.gate_up), _lib.ptr(self.down),
                  1 if self.q8 else 0, _lib.ptr(self.gate_up_s), _lib.ptr(self.down_s),
                  _lib.ptr(g), _lib.ptr(u), _lib.ptr(d), S, _lib.ptr(sgw), _lib.ptr(out),
                  _lib.ptr(w_out), _lib.ptr(sel_out), _lib.ptr(ws), ws.numel(), _lib.ptr(self.err),
                  _lib.stream_of(x))

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        shape = hidden_states.shape
        x = _lib.aligned(hidden_states.reshape(-1, shape[-1]).contiguous())
        out = torch.empty_like(x)
        for i in range(0, x.shape[0], TOKENS_PER_CALL):
            self.forward_into(x[i:i + TOKENS_PER_CALL], out[i:i + TOKENS_PER_CALL])
        return out.view(shape)

    def device_errors(self) -> int:
        """The device error word (DUPLEX_DEVERR_* bits) of this module's launches."""
        return int(self.err.item())


def fuse_moe_blocks(model: nn.Module, q8: bool = False, verbose: bool = True) -> int:
    """Replace every unquantised SparseMoeBlock of `model` with a FusedMoE (reference
    :144-178); blocks whose experts hold packed int4 weights are left to
    fuse_packed_moe_blocks."""
    sites = []
    for parent in model.modules():
        for name, child in list(parent.named_children()):
            if not (type(child).__name__.endswith("SparseMoeBlock") and hasattr(child, "experts")):
                continue
            ex = child.experts
            if hasattr(ex, "gate_up_proj"):
                sites.append((parent, name))
                continue
            gp = getattr(ex[0], "gate_proj", None)
            if gp is None or hasattr(gp, "weight_packed") or not hasattr(gp, "weight"):
                continue
            sites.append((parent, name))
    n = 0
    for parent, name in sites:
        child = getattr(parent, name)
        setattr(parent, name, FusedMoE(child, q8=q8))
        child.experts = None
        del child
        gc.collect()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
        n += 1
    if verbose:
        print(f"fused {n} MoE blocks (B200 talker kernels{', int8' if q8 else ''})")
    return n
