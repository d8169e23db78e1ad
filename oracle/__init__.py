"""CPU oracle for the int4 dequant-GEMV / fused-MoE hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the algorithm of the reference's torch path
(thecodacus/qwen3-omni-duplex, `src/duplex/streaming/fused_packed_moe.py`,
`src/duplex/streaming/triton_dequant_gemv.py`, `src/duplex/quant/dequant.py`).
It is the checker, never the thing measured or shipped: only `tests/`,
`__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm may
import it.  The product path in `qwen3-omni-duplex_b200/duplex` never imports it.

Parity pin: the functions here are checked against golden vectors produced by
running the reference's own Python code (`tests/golden/make_golden.py`), see
`tests/test_oracle_golden.py`.  The zero-point generalisation (`nib - z` in place
of `nib - 8`) has no counterpart in the reference; it is pinned only through the
identity z == 8  ->  reference behaviour.
"""

from .moe_oracle import *  # noqa: F401,F403
