"""Golden vectors for the zero-point (asymmetric int4) dequantisation, made by running
compressed-tensors, the quantisation library of the reference's checkpoints (its
dependency `compressed-tensors>=0.8`, pyproject.toml:9).

The reference itself is symmetric (value = nibble - 8, fused_packed_moe.py:54-65,183-189)
and has no zero points.  This build's AWQ-style format is value = (nibble - z) * scale
per (row, group of g columns).  compressed-tensors' asymmetric group quantisation stores
q = nibble - 8 with a signed zero point zp per (row, group) and dequantises to
(q - zp) * scale, which is the same value with z = zp + 8.  This script feeds seeded
nibbles, zero points and scales (fp16 / bf16 / fp32) to its `dequantize` with
`QuantizationArgs(num_bits=4, type=int, symmetric=False, strategy=group, group_size=g)`,
and writes the inputs (in this build's packed layout) and outputs to
golden_zero_point_dequant.npz, with the library's version.

    python tests/golden/make_zero_point_golden.py
"""

from __future__ import annotations

from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def main() -> None:
    import sys

    import torch
    import compressed_tensors
    from compressed_tensors.quantization import QuantizationArgs
    from compressed_tensors.quantization.lifecycle.forward import dequantize

    sys.path.insert(0, str(REPO))
    import oracle as O   # only for packing the inputs into this build's layout

    rng = np.random.default_rng(2026)
    R, K = 16, 256
    out = {"version": np.array(compressed_tensors.__version__)}
    for g in (64, 128):
        G = K // g
        nib = rng.integers(0, 16, (R, K)).astype(np.int32)
        z = rng.integers(0, 16, (R, G)).astype(np.int32)
        out[f"g{g}_packed"] = O.pack4(nib)
        out[f"g{g}_zeros"] = O.pack_zeros(z)
        args = QuantizationArgs(num_bits=4, type="int", symmetric=False, strategy="group",
                                group_size=g)
        q = torch.from_numpy((nib - 8).astype(np.int8))
        zp = torch.from_numpy((z - 8).astype(np.int8))
        s32 = (np.abs(rng.standard_normal((R, G))) * 0.01).astype(np.float32)
        for name, dt in (("float16", torch.float16), ("bfloat16", torch.bfloat16),
                         ("float32", torch.float32)):
            s = torch.from_numpy(s32).to(dt)
            w = dequantize(q, s, zp, args=args, dtype=dt)
            out[f"g{g}_{name}_scale"] = s.float().numpy()
            out[f"g{g}_{name}_w"] = w.float().numpy()
    np.savez_compressed(HERE / "golden_zero_point_dequant.npz", **out)
    print("wrote", HERE / "golden_zero_point_dequant.npz")


if __name__ == "__main__":
    main()
