"""int4 dequant-GEMV, backed by the sm_100a kernels of libduplex_b200.so.

Drop-in for the reference module of the same name
(src/duplex/streaming/triton_dequant_gemv.py).  The module name is kept so
`from duplex.streaming.triton_dequant_gemv import dequant_gemv, ...` keeps working;
there is no Triton in it.  Public names, signatures and return conventions follow
the reference:

  dequant_gemv(x, packed, scale, sel, group=32, block_r=64, nw_blk=8) -> [k, R] fp32
      (reference :85-113; block_r / nw_blk are accepted and ignored, `zeros=` added)
  reference_gemv(x, packed, scale, sel, group=32)          (reference :116-122)
  TritonPackedLinear(mod, device)                           (reference :125-159)
  patch_attention_to_triton(model, device, verbose) -> int  (reference :162-172)

Packing (unchanged at this interface): unpacked column j = i + 8*m is nibble i of
int32 word m; scales per group of `group` columns; optional zero points.  The
kernels read a one-time repack of that layout (`Int4Tiles`, tile records of 16
rows); modules repack at construction, `dequant_gemv` keeps a small cache keyed by
the source tensors and their version counters.
"""

from __future__ import annotations

import collections

import torch

from duplex import _lib

# Kept for import compatibility with the reference (`fused_packed_moe` imports it):
# True when the B200 kernel library is loadable.
try:
    _lib.load()
    HAVE_TRITON = True
except RuntimeError:  # pragma: no cover - reported loudly at call time
    HAVE_TRITON = False
HAVE_KERNELS = HAVE_TRITON


def _kernel_scale(scale: torch.Tensor) -> torch.Tensor:
    """Kernel scale dtype is fp16 or bf16.  fp32 scales (TritonPackedLinear's in the
    reference) are converted only when that is exact, else rejected."""
    if scale.dtype in (torch.float16, torch.bfloat16):
        return scale
    if scale.dtype == torch.float32:
        for dt in (torch.float16, torch.bfloat16):
            s = scale.to(dt)
            if torch.equal(s.float(), scale):
                return s
    raise _lib.DuplexError(f"scale dtype {scale.dtype} is not exactly representable in fp16/bf16")


class Int4Tiles:
    """Tile records of a stacked int4 matrix [E, R, K/8] (+ scales, zero points).

    One record per (expert, 16-row block) holds the block's nibbles in MMA fragment
    order with its group scales and zero points, so one bulk copy feeds a kernel
    stage (layout documented in csrc/tiles.cuh).  `pair_halves` interleaves the row
    blocks of the two halves (gate | up), so a gate block and its up block are one
    contiguous pair of records.
    """

    def __init__(self, packed, scale, zeros=None, group=None, K=None, pair_halves=False):
        _lib.require_cuda(packed, scale, zeros)
        if packed.dim() == 2:
            packed, scale = packed.unsqueeze(0), scale.unsqueeze(0)
            zeros = None if zeros is None else zeros.unsqueeze(0)
        E, R, NW = packed.shape
        K = int(K if K is not None else NW * 8)
        G = scale.shape[-1]
        group = int(group if group is not None else -(-K // G))
        if NW * 8 != K:
            packed = packed[..., : K // 8]
        self.E, self.R, self.K, self.group = E, R, K, group
        self.has_zeros = zeros is not None
        scale = _lib.aligned(_kernel_scale(scale))
        self.scale_dtype = scale.dtype
        n = _lib.ctypes.c_size_t()
        _lib.call("duplex_tile_record_bytes", K, group, 1 if self.has_zeros else 0,
                  _lib.ctypes.byref(n))
        self.record_bytes = n.value
        rb = -(-R // 16)
        self.buf = torch.empty(E * rb * n.value, dtype=torch.uint8, device=packed.device)
        p = _lib.aligned(packed.to(torch.int32))
        z = None if zeros is None else _lib.aligned(zeros.to(torch.int32))
        _lib.call("duplex_repack_tiles", _lib.ptr(p), _lib.ptr(scale), _lib.ptr(z),
                  _lib.dtype_code(scale.dtype), E, R, K, group, 1 if pair_halves else 0,
                  _lib.ptr(self.buf), self.buf.numel(), _lib.stream_of(p))

    @property
    def scale_code(self) -> int:
        return _lib.dtype_code(self.scale_dtype)

    def nbytes(self) -> int:
        return self.buf.numel()


class TcRecords:
    """Tensor-core records of a stacked int4 matrix [E, R, K/8] (+ scales, zero points).

    One record per (expert, 128-row tile, 128-column chunk): the chunk's nibbles in a
    thread-per-row order, its 128 scales and optionally 128 zero points, so one bulk
    copy feeds a ring stage of the tcgen05 expert kernels (layout documented in
    csrc/grouped_tc.cuh).  Scale groups of 128 only.  `pair_halves` (gate | up):
    every tile holds 64 gate rows and the matching 64 up rows.
    """

    def __init__(self, packed, scale, zeros=None, group=None, K=None, pair_halves=False):
        _lib.require_cuda(packed, scale, zeros)
        if packed.dim() == 2:
            packed, scale = packed.unsqueeze(0), scale.unsqueeze(0)
            zeros = None if zeros is None else zeros.unsqueeze(0)
        E, R, NW = packed.shape
        K = int(K if K is not None else NW * 8)
        G = scale.shape[-1]
        group = int(group if group is not None else -(-K // G))
        if NW * 8 != K:
            packed = packed[..., : K // 8]
        self.E, self.R, self.K, self.group = E, R, K, group
        self.has_zeros = zeros is not None
        scale = _lib.aligned(_kernel_scale(scale))
        self.scale_dtype = scale.dtype
        n = _lib.ctypes.c_size_t()
        _lib.call("duplex_tc_records_bytes", E, R, K, group, 1 if self.has_zeros else 0,
                  1 if pair_halves else 0, _lib.ctypes.byref(n))
        self.buf = torch.empty(n.value, dtype=torch.uint8, device=packed.device)
        p = _lib.aligned(packed.to(torch.int32))
        z = None if zeros is None else _lib.aligned(zeros.to(torch.int32))
        _lib.call("duplex_repack_tc_records", _lib.ptr(p), _lib.ptr(scale), _lib.ptr(z),
                  _lib.dtype_code(scale.dtype), E, R, K, group, 1 if pair_halves else 0,
                  _lib.ptr(self.buf), self.buf.numel(), _lib.stream_of(p))

    @staticmethod
    def supported(E, R, K, group, pair_halves=False) -> bool:
        n = _lib.ctypes.c_size_t()
        return _lib.load().duplex_tc_records_bytes(E, R, K, group, 0, 1 if pair_halves else 0,
                                                   _lib.ctypes.byref(n)) == 0

    @property
    def scale_code(self) -> int:
        return _lib.dtype_code(self.scale_dtype)

    def nbytes(self) -> int:
        return self.buf.numel()


class DownSlices:
    """The down projection of a stacked expert set [E, H, I/8] (+ scales [E, H, I/group],
    zero points) as K-slice records for the persistent clock-path kernel: one record per
    (expert, 128-column slice of I, 16 rows of H), tile-record layout with K = 128,
    16-byte padded (duplex_repack_down_slices).  Groups of 32, 64 or 128."""

    def __init__(self, packed, scale, zeros=None, group=None):
        _lib.require_cuda(packed, scale, zeros)
        E, H, NW = packed.shape
        I = NW * 8
        group = int(group if group is not None else -(-I // scale.shape[-1]))
        self.E, self.H, self.I, self.group = E, H, I, group
        self.has_zeros = zeros is not None
        scale = _lib.aligned(_kernel_scale(scale))
        self.scale_dtype = scale.dtype
        n = _lib.ctypes.c_size_t()
        _lib.call("duplex_down_slices_bytes", E, H, I, group, 1 if self.has_zeros else 0,
                  _lib.ctypes.byref(n))
        self.buf = torch.empty(n.value, dtype=torch.uint8, device=packed.device)
        p = _lib.aligned(packed.to(torch.int32))
        z = None if zeros is None else _lib.aligned(zeros.to(torch.int32))
        _lib.call("duplex_repack_down_slices", _lib.ptr(p), _lib.ptr(scale), _lib.ptr(z),
                  _lib.dtype_code(scale.dtype), E, H, I, group, _lib.ptr(self.buf),
                  self.buf.numel(), _lib.stream_of(p))

    @staticmethod
    def supported(E, H, I, group) -> bool:
        n = _lib.ctypes.c_size_t()
        return _lib.load().duplex_down_slices_bytes(E, H, I, group, 0, _lib.ctypes.byref(n)) == 0


_TILE_CACHE: collections.OrderedDict = collections.OrderedDict()
_TILE_CACHE_MAX = 16


def _key(t):
    return None if t is None else (t.data_ptr(), t._version, tuple(t.shape), t.dtype)


def tiles_for(packed, scale, zeros, K, group) -> Int4Tiles:
    """Cached Int4Tiles of (packed, scale, zeros); invalidated by in-place writes."""
    key = (_key(packed), _key(scale), _key(zeros), K, group)
    hit = _TILE_CACHE.get(key)
    if hit is not None:
        _TILE_CACHE.move_to_end(key)
        return hit[0]
    tl = Int4Tiles(packed, scale, zeros, group=group, K=K)
    _TILE_CACHE[key] = (tl, packed, scale, zeros)   # keep sources alive while cached
    if len(_TILE_CACHE) > _TILE_CACHE_MAX:
        _TILE_CACHE.popitem(last=False)
    return tl


def dequant_gemv(x, packed, scale, sel, group=32, block_r=64, nw_blk=8, zeros=None):
    """y[j, r] = sum_c W[sel[j], r, c] * x[j, c],  W dequantised from int4 in registers.

    x       [K] or [k, K]    fp16/bf16 activations; 1-D is shared across experts
    packed  [E, R, K/8] int32
    scale   [E, R, ceil(K/group)]
    sel     [k] expert ids (device tensor, any int dtype)
    zeros   optional [E, R, ceil(G/8)] int32 packed zero points (None: symmetric, z=8)
    returns [k, R] float32
    """
    _lib.require_cuda(x, packed, scale, sel, zeros)
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise _lib.DuplexError(f"activations must be fp16 or bf16, got {x.dtype}")
    E, R, NW = packed.shape
    K = x.shape[-1]
    if NW * 8 < K:
        raise _lib.DuplexError(f"packed has {NW} words per row, fewer than K/8 = {K // 8}")
    tl = tiles_for(packed, scale, zeros, K, group)
    sel32 = _lib.aligned(sel.reshape(-1).to(torch.int32))
    k = sel32.numel()
    x = _lib.aligned(x)
    x_slot = 0 if x.dim() == 1 else K
    if x.dim() == 2 and x.shape[0] != k:
        raise _lib.DuplexError("per-expert x must have one row per selected expert")
    out = torch.empty(k, R, device=x.device, dtype=torch.float32)
    _lib.call("duplex_dq_gemv", _lib.ptr(x), _lib.dtype_code(x.dtype), x_slot, _lib.ptr(tl.buf),
              tl.scale_code, 1 if tl.has_zeros else 0, E, R, K, group, _lib.ptr(sel32), k,
              _lib.ptr(out), None, _lib.stream_of(x))
    return out


def reference_gemv(x, packed, scale, sel, group=32, zeros=None):
    """Same result through a dense dequantised weight (materialised by the dequant
    kernel) and a plain matmul, for correctness checking (reference :116-122)."""
    from duplex.streaming.fused_packed_moe import FusedPackedMoE

    K = x.numel()
    sel = sel.reshape(-1).long()
    w = FusedPackedMoE._dequant(packed[sel], scale[sel].to(torch.float32), K,
                                zeros=None if zeros is None else zeros[sel])
    return torch.matmul(w, x.to(torch.float32).view(-1, 1)).squeeze(-1)


class TritonPackedLinear(torch.nn.Module):
    """A packed int4 Linear whose forward runs the B200 dequant-GEMV.

    Same constructor and forward contract as the reference (:125-159), but the B
    rows of a call go through ONE kernel launch per group of up to 8 rows (the
    MMA's N dimension) instead of one launch per row.  Scales stay in their
    checkpoint dtype (fp16); the reference's fp32 copy holds the same values.
    """

    def __init__(self, mod, device="cuda"):
        super().__init__()
        shape = tuple(int(v) for v in mod.weight_shape.tolist())
        self.out_features, self.in_features = shape
        from duplex.streaming.packed_checkpoint import linear_zeros
        zeros = linear_zeros(mod)
        scale = mod.weight_scale.to(device)
        self.group = -(-self.in_features // scale.shape[-1])
        self.tiles = Int4Tiles(mod.weight_packed.to(device), scale,
                               None if zeros is None else zeros.to(device), group=self.group,
                               K=self.in_features)
        b = getattr(mod, "bias", None)
        self.register_buffer("bias", b.to(device) if b is not None else None, persistent=False)
        self.register_buffer("_sel", torch.zeros(1, dtype=torch.int32, device=device),
                             persistent=False)
        self.pdl = False

    def forward(self, x, residual=None, out=None, rms_eps: float = 0.0, x_row_stride=None):
        """y = x W^T (+ bias).  Extensions used by the clock-path stack: `residual` is added
        in fp32, `rms_eps > 0` RMS-normalises each input row first, `out` receives y."""
        _lib.require_cuda(x)
        lead, K = x.shape[:-1], x.shape[-1]
        if x_row_stride is not None and x.dim() == 2 and x.stride(1) == 1:
            flat, xs = x, x_row_stride      # strided row view (e.g. q out of a fused qkv)
        else:
            flat = _lib.aligned(x.reshape(-1, K))
            xs = K
        N = flat.shape[0]
        y = out if out is not None else torch.empty(N, self.out_features, device=x.device,
                                                    dtype=x.dtype)
        bias = None if self.bias is None else _lib.aligned(self.bias.to(x.dtype))
        res = None if residual is None else _lib.aligned(residual.reshape(-1, self.out_features))
        st = _lib.stream_of(x)
        tl = self.tiles
        for r0 in range(0, N, 8):
            b = min(8, N - r0)
            _lib.call("duplex_packed_linear", _lib.ptr(flat[r0:r0 + b]), _lib.dtype_code(x.dtype),
                      b, xs, _lib.ptr(tl.buf), tl.scale_code, 1 if tl.has_zeros else 0,
                      self.out_features, K, self.group, _lib.ptr(bias),
                      None if res is None else _lib.ptr(res[r0:r0 + b]), self.out_features,
                      _lib.ptr(y[r0:r0 + b]), self.out_features, float(rms_eps),
                      1 if self.pdl else 0, st)
        return y.view(*lead, self.out_features)


def patch_attention_to_triton(model, device="cuda", verbose=True) -> int:
    """Swap packed attention projections onto the B200 kernel (reference :162-172)."""
    n = 0
    for parent in model.modules():
        for name, child in list(parent.named_children()):
            if hasattr(child, "weight_packed") and hasattr(child, "weight_scale"):
                setattr(parent, name, TritonPackedLinear(child, device))
                n += 1
    if verbose:
        print(f"moved {n} packed linears onto the B200 dequant-GEMV kernel")
    return n
