"""Packed-linear helpers on the B200 kernels: drop-in for the reference module
src/duplex/quant/dequant.py (every public name of it is here, same signatures).

  dequantize_weight(mod, dtype, device)       reference :40-77   -> duplex_dequant
  patch_packed_linears(model, compute_device, verbose) -> int
                                              reference :94-119  -> duplex_packed_linear
  place_unpacked(root, device, verbose) -> dict   (alias place_thinker)
                                              reference :122-163 (pure module placement)
  sanity_check(model, k) -> list[dict]        reference :166-193

`dequantize_weight` reconstructs the dense weight of one packed Linear
(`weight_packed` [out, in/8] int32, `weight_scale` [out, G], `weight_shape`),
bit-identical to the reference: the scale is first cast to `dtype`, then every
element is one rounding of the exact (nibble - 8) * scale product into `dtype`.  An
optional `weight_zeros` buffer ([out, ceil(G/8)] int32) replaces the constant 8, and so
does compressed-tensors' asymmetric `weight_zero_point` (converted on use).

`patch_packed_linears` installs a forward on every packed Linear.  The reference's
forward dequantises the whole weight on every call and runs F.linear; here the
forward runs the int4 dequant-GEMV kernel (weights dequantised in registers, at most
8 rows per launch) on a one-time repack of the module's packed tensors into tile
records, kept on the compute device.  fp32 activations keep the reference's literal
form (dequantise with the kernel, then a matmul).  The kernels take CUDA tensors
only: a forward whose input (or `compute_device`) is not a CUDA device raises.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from duplex import _lib

NUM_BITS = 4
GROUP_SIZE = 32


def _shape(mod):
    s = mod.weight_shape
    return tuple(int(v) for v in (s.tolist() if torch.is_tensor(s) else s))


def dequantize_weight(mod, dtype: torch.dtype | None = None, device=None) -> torch.Tensor:
    out_f, in_f = _shape(mod)
    packed, scale = mod.weight_packed, mod.weight_scale
    from duplex.streaming.packed_checkpoint import linear_zeros
    zeros = linear_zeros(mod)
    if device is not None:
        packed, scale = packed.to(device), scale.to(device)
        zeros = None if zeros is None else zeros.to(device)
    _lib.require_cuda(packed, scale, zeros)
    dtype = dtype or scale.dtype
    if scale.ndim == 2 and scale.shape[1] > 1:
        n_groups = scale.shape[1]
        if n_groups * GROUP_SIZE < in_f:
            raise ValueError(f"scale groups {n_groups} x {GROUP_SIZE} < in_features {in_f}")
        if in_f % n_groups:
            # the reference's view(out_f, n_groups, -1) of the [out, in] unpack fails here
            raise RuntimeError(f"in_features {in_f} does not split into {n_groups} equal groups")
        group = in_f // n_groups
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


def _kernel_linear(mod, device):
    """The module's TritonPackedLinear on `device`, built (repacked) on first use."""
    from duplex.streaming.triton_dequant_gemv import TritonPackedLinear
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    cache = mod.__dict__.setdefault("_duplex_linears", {})
    lin = cache.get(dev)
    if lin is None:
        lin = TritonPackedLinear(mod, dev)
        cache[dev] = lin
    return lin


def _streaming_forward(mod: nn.Module, compute_device=None):
    """Forward of a packed Linear on the B200 kernels: y = x W^T (+ bias) on
    `compute_device` (default: the input's device), in the input's dtype."""

    def forward(x):
        dev = torch.device(compute_device) if compute_device is not None else x.device
        if dev.type != "cuda":
            raise _lib.DuplexError(
                "patched packed Linear: the B200 kernels run on CUDA devices only "
                f"(got {dev}); pass compute_device='cuda'")
        x = x.to(dev)
        if x.dtype in (torch.float16, torch.bfloat16):
            return _kernel_linear(mod, dev)(x)
        w = dequantize_weight(mod, dtype=x.dtype, device=dev)
        b = getattr(mod, "bias", None)
        if b is not None:
            b = b.to(dev, x.dtype)
        return torch.nn.functional.linear(x, w, b)

    return forward


def patch_packed_linears(model: nn.Module, compute_device=None, verbose: bool = True) -> int:
    """Give every module holding `weight_packed` and `weight_scale` the kernel forward
    above.  A wrapper left by compressed-tensors / accelerate (`_old_forward`) is
    removed first, as the reference does.  Returns the number of modules patched."""
    count = 0
    for mod in model.modules():
        if not (hasattr(mod, "weight_packed") and hasattr(mod, "weight_scale")):
            continue
        if "_old_forward" in mod.__dict__:
            del mod.__dict__["_old_forward"]
        mod.forward = _streaming_forward(mod, compute_device)
        count += 1
    if verbose:
        where = compute_device if compute_device is not None else "the input's device"
        print(f"patched {count} packed Linear modules (int4 dequant-GEMV kernel on {where})")
    return count


def place_unpacked(root: nn.Module, device="cuda", verbose: bool = True) -> dict:
    """Move every parameter and buffer of `root` to `device` except those owned by a
    packed module (one with `weight_packed`), which stay where they are.  Returns the
    element counts moved and kept, and the device."""
    keep = set()
    for mod in root.modules():
        if hasattr(mod, "weight_packed"):
            keep.update(id(t) for t in mod.parameters(recurse=False))
            keep.update(id(t) for t in mod.buffers(recurse=False))
    moved = kept = 0
    for mod in root.modules():
        for name, prm in list(mod.named_parameters(recurse=False)):
            if id(prm) in keep:
                kept += prm.numel()
            else:
                setattr(mod, name, nn.Parameter(prm.data.to(device), requires_grad=False))
                moved += prm.numel()
        for name, buf in list(mod.named_buffers(recurse=False)):
            if id(buf) in keep:
                kept += buf.numel()
            else:
                mod.register_buffer(name, buf.to(device), persistent=False)
                moved += buf.numel()
    stats = {"moved_params": moved, "kept_on_host": kept, "device": str(device)}
    if verbose:
        print(f"  placed {moved / 1e6:.0f}M params on {device}, "
              f"{kept / 1e6:.0f}M packed elements left where they were")
    return stats


place_thinker = place_unpacked


def sanity_check(model: nn.Module, k: int = 3) -> list[dict]:
    """Dequantise the first k packed linears (on the GPU) and report, per module, its
    shape against `weight_shape`, mean / std / absmax, and the number of distinct
    values in the first group of row 0 (at most 16 for a correct int4 unpack)."""
    rows = []
    for name, mod in model.named_modules():
        if len(rows) >= k:
            break
        if not (hasattr(mod, "weight_packed") and hasattr(mod, "weight_scale")):
            continue
        dev = mod.weight_packed.device if mod.weight_packed.is_cuda else "cuda"
        w = dequantize_weight(mod, device=dev).float()
        want = _shape(mod)
        rows.append({
            "name": name,
            "shape": tuple(w.shape),
            "expected_shape": want,
            "shape_ok": tuple(w.shape) == want,
            "mean": float(w.mean()),
            "std": float(w.std()),
            "absmax": float(w.abs().max()),
            "n_unique_first_group": int(w[0, :GROUP_SIZE].unique().numel()),
        })
    return rows
