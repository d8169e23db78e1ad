"""Expert-parallel Thinker MoE: one layer's 128 experts sharded over the ranks of a
process group (one process per GPU), tokens data-parallel.

The reference runs every expert on one GPU (`src/duplex/streaming/fused_packed_moe.py`);
this is the multi-GPU form of the same layer, `FusedPackedMoE.forward` semantics per
token, for batched decode (many streams per rank).  Per layer on every rank (with
exchange="peer" steps 2-4 run over NVLink peer memory instead: PeerExchange):

  1. route the rank's own tokens over all E experts (router logits, fp32 softmax,
     top-k, renormalise: `duplex_moe_route_grouped`), whose top-k kernel writes each
     token's exchange row (the token, its k expert ids, its k weights);
  2. dispatch: for every rank d, the rows of the tokens that picked one of d's experts,
     compacted into block d of a send buffer (`duplex_ep_dispatch_pack`), then ONE NCCL
     all-to-all: rank d receives, from every rank, the tokens that need its experts;
  3. the rank's experts [rank * E/N, (rank + 1) * E/N) on the received rows, one fp32
     partial sum per row over the slots that hit them (`duplex_moe_experts_grouped`);
  4. combine: ONE NCCL all-to-all sends every partial row back to the token's owner,
     which adds the partials in rank order (+ residual), one rounding to the activation
     type (`duplex_ep_combine`).

With one rank, steps 2 and 4 are the identity and are skipped: the expert stage reads
the routed rows in place.

Each block of the send buffers holds up to T_local rows (a token can need every rank),
so both all-to-alls have a fixed size: no host synchronisation, and a 48-layer step is
one CUDA graph.  The rows of a block past its count carry an expert id of another rank
and weight 0, which the receiving expert stage skips.  The host logic lives in
`ep_forward`, which takes the device steps as callables: the module passes the sm_100a
kernels; the multi-rank CPU tests pass torch / numpy restatements of the same steps.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from duplex import _lib
from duplex.streaming.triton_dequant_gemv import Int4Tiles

PACK = 8


def exchange_row_bytes(H: int, elt: int, top_k: int) -> int:
    """Bytes of one exchange row: the token, its k expert ids, its k weights (16-aligned)."""
    return -(-(H * elt + 8 * top_k) // 16) * 16


class _DeviceArray:
    """A raw device allocation seen by torch (no copy, no ownership)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3}


class PeerExchange:
    """The two exchanges of an expert-parallel layer over NVLink peer memory, in place of
    the NCCL all-to-alls: every rank allocates its receive buffer [N, T_l, row], its
    return buffer [N, T_l, H] fp32 and a flag block with cudaMalloc (duplex_ipc_alloc),
    the CUDA IPC handles go round the process group, and every rank maps the others'
    buffers (duplex_ipc_open: plain peer mappings, no multicast object).  dispatch()
    packs each destination's rows straight into that destination's receive buffer
    (duplex_ep_dispatch_peer: the pack and the exchange are one kernel) and waits for
    every source's epoch in its own flags (duplex_ep_wait, bounded); give_back() puts the
    partial rows into their owners' return buffers and waits the same way.  A sender
    writes a destination's buffer again only after that destination's next signal to it,
    which it sends after it has read the buffer, so one buffer per exchange suffices."""

    def __init__(self, group, T_l: int, row_bytes: int, H: int, E: int, device):
        self.group = group
        self.E = E
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.T_l, self.row_bytes, self.H = T_l, row_bytes, H
        N = self.world
        lib = _lib.load()
        hb = lib.duplex_ipc_handle_bytes()
        sizes = (N * T_l * row_bytes, N * T_l * H * 4, (2 * N + 8) * 4)
        self._own, handles = [], []
        for n in sizes:
            h = _lib.ctypes.create_string_buffer(hb)
            ptr = _lib.ctypes.c_void_p()
            _lib.call("duplex_ipc_alloc", n, _lib.ctypes.byref(ptr), h)
            self._own.append(ptr.value)
            handles.append(h.raw)
        allh = [None] * N
        dist.all_gather_object(allh, handles, group=group)
        self._opened = []
        peers = []
        for r in range(N):
            if r == self.rank:
                peers.append(list(self._own))
                continue
            row = []
            for h in allh[r]:
                ptr = _lib.ctypes.c_void_p()
                _lib.call("duplex_ipc_open", _lib.ctypes.create_string_buffer(h, hb),
                          _lib.ctypes.byref(ptr))
                self._opened.append(ptr.value)
                row.append(ptr.value)
            peers.append(row)
        dev = torch.device(device)
        i64 = lambda v: torch.tensor(v, dtype=torch.int64, device=dev)  # noqa: E731
        self.recv_peers = i64([p[0] for p in peers])
        self.back_peers = i64([p[1] for p in peers])
        self.fdisp_peers = i64([p[2] for p in peers])
        self.fcomb_peers = i64([p[2] + 4 * N for p in peers])
        f = self._own[2]
        self.fdisp, self.fcomb = f, f + 4 * N
        self.disp_counter, self.disp_epoch = f + 8 * N, f + 8 * N + 4
        self.comb_counter, self.comb_epoch = f + 8 * N + 8, f + 8 * N + 12
        self.recv = torch.as_tensor(_DeviceArray(self._own[0], (N, T_l, row_bytes), "|u1"), device=dev)
        self.back = torch.as_tensor(_DeviceArray(self._own[1], (N, T_l, H), "<f4"), device=dev)

    def dispatch(self, rows, top_k: int, ids_offset: int, slot_of, err):
        st = _lib.stream_of(rows)
        _lib.call("duplex_ep_dispatch_peer", _lib.ptr(rows), rows.stride(0), self.T_l, top_k, self.E,
                  self.world, self.rank, ids_offset, _lib.ptr(self.recv_peers), _lib.ptr(slot_of),
                  _lib.ptr(self.fdisp_peers), self.disp_counter, self.disp_epoch, st)
        _lib.call("duplex_ep_wait", self.fdisp, self.disp_epoch, self.world, 0, _lib.ptr(err), st)
        return self.recv

    def give_back(self, partial, err):
        st = _lib.stream_of(partial)
        _lib.call("duplex_ep_put_peer", _lib.ptr(partial), self.T_l * self.H * 4, self.world,
                  self.rank, _lib.ptr(self.back_peers), _lib.ptr(self.fcomb_peers),
                  self.comb_counter, self.comb_epoch, st)
        _lib.call("duplex_ep_wait", self.fcomb, self.comb_epoch, self.world, 0, _lib.ptr(err), st)
        return self.back

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after a device synchronise, and
        before the process group goes)."""
        torch.cuda.synchronize()
        for ptr in self._opened:
            _lib.call("duplex_ipc_close", ptr)
        for ptr in self._own:
            _lib.call("duplex_ipc_free", ptr)
        self._opened, self._own = [], []


def ep_forward(x, route_fn, pack_fn, experts_fn, combine_fn, top_k: int, group=None,
               residual=None, bufs=None, peer=None, err=None):
    """Host side of one expert-parallel layer on this rank.

    x [T_local, H].  route_fn(x, rows) fills rows [T_local, row] uint8 with each token's
    exchange row (the token's H * elt bytes, its k expert ids as int32, its k weights as
    fp32); pack_fn(rows, send, slot_of) fills send [N, T_local, row] and slot_of
    [N, T_local] int32 (dispatch_pack); experts_fn(x_all, sel_all, w_all) -> fp32
    [N * T_local, H], this rank's experts' weighted sum per received row (row-strided
    views of the received rows); combine_fn(back [N, T_local, H] fp32, slot_of,
    residual) -> [T_local, H], the layer output.  bufs: optional dict of preallocated
    buffers (rows, send, slot_of, recv, back), reused across calls of the same shape.
    """
    world = dist.get_world_size(group)
    T_l, H = x.shape
    xbytes = H * x.element_size()
    row = exchange_row_bytes(H, x.element_size(), top_k)
    dev = x.device
    b = bufs if bufs is not None else {}
    if "rows" not in b:
        b["rows"] = torch.empty(T_l, row, dtype=torch.uint8, device=dev)
        b["send"] = torch.empty(world, T_l, row, dtype=torch.uint8, device=dev)
        b["slot_of"] = torch.empty(world, T_l, dtype=torch.int32, device=dev)
        if world > 1:
            b["recv"] = torch.empty(world, T_l, row, dtype=torch.uint8, device=dev)
            b["back"] = torch.empty(world, T_l, H, dtype=torch.float32, device=dev)
    route_fn(x, b["rows"])
    if peer is not None and world > 1:
        # the pack writes into the destinations' receive buffers; the partials go back
        # into the owners' return buffers (NVLink peer stores, flags, bounded waits)
        recv = peer.dispatch(b["rows"], top_k, xbytes, b["slot_of"], err)
        rv = recv.view(world * T_l, row)
        x_all = rv[:, :xbytes].view(x.dtype)
        sel_all = rv[:, xbytes:xbytes + 4 * top_k].view(torch.int32)
        w_all = rv[:, xbytes + 4 * top_k:xbytes + 8 * top_k].view(torch.float32)
        partial = experts_fn(x_all, sel_all, w_all).view(world, T_l, H)
        return combine_fn(peer.give_back(partial, err), b["slot_of"], residual)
    if world == 1:
        # one rank: every token goes to it, in order, so the block IS the routed rows and
        # the all-to-all is the identity -- no pack, no exchange
        if "ident" not in b:
            b["ident"] = torch.arange(T_l, dtype=torch.int32, device=dev).view(1, T_l)
        recv, slot_of = b["rows"], b["ident"]
    else:
        pack_fn(b["rows"], b["send"], b["slot_of"])
        recv, slot_of = b["recv"], b["slot_of"]
        dist.all_to_all_single(recv, b["send"], group=group)
    rv = recv.view(world * T_l, row)
    x_all = rv[:, :xbytes].view(x.dtype)
    sel_all = rv[:, xbytes:xbytes + 4 * top_k].view(torch.int32)
    w_all = rv[:, xbytes + 4 * top_k:xbytes + 8 * top_k].view(torch.float32)
    partial = experts_fn(x_all, sel_all, w_all).view(world, T_l, H)
    back = partial if world == 1 else b["back"]
    if world > 1:
        dist.all_to_all_single(back, partial, group=group)
    return combine_fn(back, slot_of, residual)


class ExpertParallelMoE(nn.Module):
    """One MoE layer whose experts are split evenly over the ranks of `group`.

    Built from the full stacked tensors (`FusedPackedMoE.from_stacked` layout: gate
    [E, H], gate|up packed [E, 2I, H/8] + scales [E, 2I, G] (+ zeros), down packed
    [E, H, I/8] + scales [E, H, G'] (+ zeros)); every rank keeps the router and its own
    E/N experts (repacked once into tile records).  forward(x [T_local, H]) returns the
    layer output for this rank's tokens; N * T_local <= 512 (the received rows).
    """

    def __init__(self, gate_weight, gu_packed, gu_scale, dn_packed, dn_scale, top_k,
                 gu_zeros=None, dn_zeros=None, norm_topk_prob=True, gate_bias=None,
                 dtype=torch.float16, device="cuda", group=None, exchange: str = "nccl"):
        super().__init__()
        if dtype not in (torch.float16, torch.bfloat16):
            raise _lib.DuplexError("ExpertParallelMoE runs fp16 or bf16 modules")
        if exchange not in ("nccl", "peer"):
            raise _lib.DuplexError("exchange is 'nccl' (all-to-alls) or 'peer' (NVLink peer stores)")
        self.exchange = exchange
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        E, H = gate_weight.shape
        if E % self.world:
            raise _lib.DuplexError(f"{E} experts do not split evenly over {self.world} ranks")
        self.num_experts, self.hidden, self.top_k = E, H, top_k
        self.norm_topk_prob = norm_topk_prob
        self.E_local = E // self.world
        self.e_begin = self.rank * self.E_local
        sl = slice(self.e_begin, self.e_begin + self.E_local)
        self.gate = nn.Linear(H, E, bias=gate_bias is not None).to(device=device, dtype=dtype)
        with torch.no_grad():
            self.gate.weight.copy_(gate_weight)
            if gate_bias is not None:
                self.gate.bias.copy_(gate_bias)
        self.inter = gu_packed.shape[1] // 2
        G = gu_scale.shape[-1]
        self.group_size = -(-H // G)
        self.has_zeros = gu_zeros is not None
        self.gu_tiles = Int4Tiles(gu_packed[sl].to(device), gu_scale[sl].to(device, dtype),
                                  None if gu_zeros is None else gu_zeros[sl].to(device),
                                  group=self.group_size, K=H, pair_halves=True)
        self.dn_tiles = Int4Tiles(dn_packed[sl].to(device), dn_scale[sl].to(device, dtype),
                                  None if dn_zeros is None else dn_zeros[sl].to(device),
                                  group=self.group_size, K=dn_packed.shape[2] * PACK)
        self.register_buffer("err", torch.zeros(1, dtype=torch.int32, device=device), persistent=False)
        self._ws = {}

    def _workspace(self, key, nbytes_fn, device):
        ws = self._ws.get(key)
        if ws is None:
            n = _lib.ctypes.c_size_t()
            nbytes_fn(_lib.ctypes.byref(n))
            ws = torch.empty(max(n.value, 16), dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    def _route_ws(self, T, device):
        ws = self._ws.get(("route", T))
        if ws is None:
            ws = torch.empty(T * self.num_experts * 4, dtype=torch.uint8, device=device)
            self._ws[("route", T)] = ws
        return ws

    def route(self, x, pack=None):
        """Route this rank's tokens over all experts: with pack (an [T, row] uint8
        exchange buffer) write the exchange rows there; without, return (w [T, k] fp32,
        sel [T, k] int32)."""
        T = x.shape[0]
        w = sel = None
        if pack is None:
            w = torch.empty(T, self.top_k, dtype=torch.float32, device=x.device)
            sel = torch.empty(T, self.top_k, dtype=torch.int32, device=x.device)
        ws = self._route_ws(T, x.device)
        g = self.gate
        _lib.call("duplex_moe_route_grouped", _lib.ptr(x), _lib.dtype_code(x.dtype), T,
                  _lib.ptr(g.weight), _lib.ptr(g.bias), None, self.num_experts, self.hidden,
                  self.top_k, 1 if self.norm_topk_prob else 0, _lib.ptr(w), _lib.ptr(sel),
                  _lib.ptr(pack), 0 if pack is None else pack.stride(0), _lib.ptr(ws), ws.numel(),
                  _lib.ptr(self.err), _lib.stream_of(x))
        return w, sel

    def local_experts(self, x_all, sel_all, w_all):
        """fp32 [T_all, H]: this rank's experts' weighted sums for the gathered tokens."""
        T = x_all.shape[0]
        out = torch.empty(T, self.hidden, dtype=torch.float32, device=x_all.device)
        ws = self._workspace(("experts", T), lambda p: _lib.call(
            "duplex_moe_experts_grouped_workspace_bytes", T, self.E_local, self.num_experts,
            self.hidden, self.inter, self.top_k, self.group_size, 1 if self.has_zeros else 0, p),
            x_all.device)
        if x_all.stride(1) != 1 or x_all.data_ptr() % 16:
            raise _lib.DuplexError("token rows must be contiguous and 16-byte aligned")
        if sel_all.stride(0) != w_all.stride(0) or sel_all.stride(1) != 1 or w_all.stride(1) != 1:
            raise _lib.DuplexError("expert ids and weights must share one row stride")
        _lib.call("duplex_moe_experts_grouped", _lib.ptr(x_all), _lib.dtype_code(x_all.dtype), T,
                  x_all.stride(0), _lib.ptr(sel_all), _lib.ptr(w_all), sel_all.stride(0), self.top_k,
                  self.e_begin, self.E_local,
                  self.num_experts, self.hidden, self.inter, _lib.ptr(self.gu_tiles.buf),
                  _lib.ptr(self.dn_tiles.buf), self.gu_tiles.scale_code,
                  1 if self.has_zeros else 0, self.group_size, None, _lib.ptr(out),
                  _lib.DTYPE_F32, _lib.ptr(ws), ws.numel(), _lib.ptr(self.err),
                  _lib.stream_of(x_all))
        return out

    def pack(self, rows, send, slot_of):
        """Dispatch: rows of this rank's tokens into the per-rank blocks of `send`."""
        T = rows.shape[0]
        xbytes = self.hidden * self.gate.weight.element_size()
        _lib.call("duplex_ep_dispatch_pack", _lib.ptr(rows), rows.stride(0), T, self.top_k,
                  self.num_experts, self.world, xbytes, _lib.ptr(send), _lib.ptr(slot_of),
                  _lib.stream_of(rows))

    def combine(self, back, slot_of, residual=None, out=None):
        """Layer output of this rank's tokens from the partial rows returned by every rank."""
        N, T, H = back.shape
        dt = self.gate.weight.dtype
        out = out if out is not None else torch.empty(T, H, dtype=dt, device=back.device)
        res = None if residual is None else _lib.aligned(residual.to(dt))
        _lib.call("duplex_ep_combine", _lib.ptr(back), _lib.ptr(slot_of), T, N, H, _lib.ptr(res),
                  _lib.ptr(out), _lib.dtype_code(dt), _lib.stream_of(back))
        return out

    def forward(self, x, residual=None):
        """x [T_local, H] (this rank's tokens) -> [T_local, H]; every rank calls it with
        the same T_local.  Buffers are kept per T_local (no allocation after the first
        call of a shape, so a layer can be captured in a CUDA graph)."""
        _lib.require_cuda(x)
        x = _lib.aligned(x.to(self.gate.weight.dtype))
        T = x.shape[0]
        if T > 512:
            raise _lib.DuplexError("ExpertParallelMoE takes at most 512 tokens per rank")
        bufs = self._ws.setdefault(("ep", T), {})
        peer = None
        if self.exchange == "peer" and self.world > 1:
            peer = self._ws.get(("peer", T))
            if peer is None:   # collective: every rank builds it on its first call of a shape
                row = exchange_row_bytes(self.hidden, x.element_size(), self.top_k)
                peer = PeerExchange(self.group, T, row, self.hidden, self.num_experts, x.device)
                self._ws[("peer", T)] = peer
        return ep_forward(x, lambda xt, rows: self.route(xt, rows), self.pack,
                          self.local_experts, lambda back, slot_of, res: self.combine(back, slot_of, res),
                          self.top_k, self.group, residual, bufs, peer=peer, err=self.err)

    def close(self) -> None:
        """Release the peer exchange buffers (before the process group is destroyed)."""
        for key in [k for k in self._ws if k[0] == "peer"]:
            self._ws.pop(key).close()

    def device_errors(self) -> int:
        v = int(self.err.item())
        self.err.zero_()
        return v
