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

Packing (unchanged): unpacked column j = i + 8*m is nibble i of int32 word m;
scales per group of `group` columns; optional zero points (see `duplex._lib`).
"""

from __future__ import annotations

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


def pad_rows(t: torch.Tensor | None, rows_to: int) -> torch.Tensor | None:
    """Pad dim -2 of a stacked [..., R, C] tensor with zeros up to `rows_to`."""
    if t is None or t.shape[-2] == rows_to:
        return t
    pad = list(t.shape)
    pad[-2] = rows_to - t.shape[-2]
    return torch.cat([t, t.new_zeros(pad)], dim=-2)


def prepare_int4(packed, scale, zeros=None):
    """-> (packed, scale, zeros, R, Rs) laid out as the kernels need: rows padded to a
    multiple of 16, contiguous, 16-byte aligned.  One-time cost for modules."""
    R = packed.shape[-2]
    Rs = (R + 15) // 16 * 16
    scale = _kernel_scale(scale)
    packed, scale, zeros = (pad_rows(packed, Rs), pad_rows(scale, Rs), pad_rows(zeros, Rs))
    packed = _lib.aligned(packed.to(torch.int32))
    scale = _lib.aligned(scale)
    zeros = None if zeros is None else _lib.aligned(zeros.to(torch.int32))
    return packed, scale, zeros, R, Rs


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
    packed, scale, zeros, R, Rs = prepare_int4(packed[..., : K // 8], scale, zeros)
    sel32 = _lib.aligned(sel.reshape(-1).to(torch.int32))
    k = sel32.numel()
    x = _lib.aligned(x)
    x_slot = 0 if x.dim() == 1 else K
    if x.dim() == 2 and x.shape[0] != k:
        raise _lib.DuplexError("per-expert x must have one row per selected expert")
    out = torch.empty(k, R, device=x.device, dtype=torch.float32)
    _lib.call("duplex_dq_gemv", _lib.ptr(x), _lib.dtype_code(x.dtype), x_slot, _lib.ptr(packed),
              _lib.ptr(scale), _lib.ptr(zeros), _lib.dtype_code(scale.dtype), E, R, Rs, K, group,
              _lib.ptr(sel32), k, _lib.ptr(out), None, _lib.stream_of(x))
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
        zeros = getattr(mod, "weight_zeros", None)
        packed, scale, zeros, R, Rs = prepare_int4(
            mod.weight_packed.to(device), mod.weight_scale.to(device),
            None if zeros is None else zeros.to(device))
        self.group = -(-self.in_features // scale.shape[-1])
        self.rows_alloc = Rs
        self.register_buffer("packed", packed.unsqueeze(0), persistent=False)
        self.register_buffer("scale", scale.unsqueeze(0), persistent=False)
        self.register_buffer("zeros", None if zeros is None else zeros.unsqueeze(0),
                             persistent=False)
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
        for r0 in range(0, N, 8):
            b = min(8, N - r0)
            xr = flat[r0:r0 + b]
            yr = y[r0:r0 + b]
            _lib.call("duplex_packed_linear", _lib.ptr(xr), _lib.dtype_code(x.dtype), b, xs,
                      _lib.ptr(self.packed), _lib.ptr(self.scale), _lib.ptr(self.zeros),
                      _lib.dtype_code(self.scale.dtype), self.out_features, self.rows_alloc,
                      K, self.group, _lib.ptr(bias),
                      None if res is None else _lib.ptr(res[r0:r0 + b]), self.out_features,
                      _lib.ptr(yr), self.out_features, float(rms_eps), 1 if self.pdl else 0, st)
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
