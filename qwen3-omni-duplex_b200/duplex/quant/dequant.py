"""2-D int4 dequantisation on the GPU (reference src/duplex/quant/dequant.py:40-77).

`dequantize_weight(mod, dtype, device)` reconstructs the dense weight of one packed
Linear (`weight_packed` [out, in/8] int32, `weight_scale` [out, G], `weight_shape`),
bit-identical to the reference: the scale is first cast to `dtype`, then every
element is one rounding of the exact (nibble - 8) * scale product into `dtype`.
An optional `weight_zeros` buffer ([out, ceil(G/8)] int32) replaces the constant 8.
The reference's CPU serving path around it is out of scope.
"""

from __future__ import annotations

import torch

from duplex import _lib

NUM_BITS = 4
GROUP_SIZE = 32


def dequantize_weight(mod, dtype: torch.dtype | None = None, device=None) -> torch.Tensor:
    shape = mod.weight_shape
    shape = tuple(int(x) for x in (shape.tolist() if torch.is_tensor(shape) else shape))
    out_f, in_f = shape
    packed, scale = mod.weight_packed, mod.weight_scale
    zeros = getattr(mod, "weight_zeros", None)
    if device is not None:
        packed, scale = packed.to(device), scale.to(device)
        zeros = None if zeros is None else zeros.to(device)
    _lib.require_cuda(packed, scale, zeros)
    dtype = dtype or scale.dtype
    if scale.ndim == 2 and scale.shape[1] > 1:
        n_groups = scale.shape[1]
        if n_groups * GROUP_SIZE < in_f:
            raise ValueError(f"scale groups {n_groups} x {GROUP_SIZE} < in_features {in_f}")
        group = -(-in_f // n_groups)
        s = _lib.aligned(scale.to(dtype))
    else:
        group = in_f
        s = _lib.aligned(scale.to(dtype).reshape(out_f, 1))
    p = _lib.aligned(packed.to(torch.int32)[:, : -(-in_f // 8)])
    z = None if zeros is None else _lib.aligned(zeros.to(torch.int32))
    Kp = p.shape[1] * 8
    out = torch.empty(out_f, Kp, dtype=dtype, device=p.device)
    code = _lib.dtype_code(dtype)
    _lib.call("duplex_dequant", _lib.ptr(p), _lib.ptr(s), code, _lib.ptr(z), out_f, Kp, group,
              _lib.ptr(out), code, _lib.stream_of(p))
    return out[:, :in_f]
