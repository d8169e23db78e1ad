"""B200 (sm_100a) drop-in for the int4 dequant-GEMV / fused-MoE hot path of
thecodacus/qwen3-omni-duplex.  Module layout mirrors the reference's `src/duplex`:

  duplex.streaming.fused_packed_moe      FusedPackedMoE, fuse_packed_moe_blocks, unpack4
  duplex.streaming.triton_dequant_gemv   dequant_gemv, TritonPackedLinear, patch_attention_to_triton
  duplex.quant.dequant                   dequantize_weight
  duplex.clock                           graph-captured clock-path stack (Thinker layers 0-23)

All compute goes through libduplex_b200.so (C ABI in include/duplex_b200.h).
"""

__version__ = "0.1.0"
