"""Overlay this build's hot-path modules onto the reference's installed `duplex` package.

The reference (thecodacus/qwen3-omni-duplex, `src/duplex/`) reaches its int4 hot path
through three modules: `duplex.streaming.fused_packed_moe`,
`duplex.streaming.triton_dequant_gemv` and `duplex.quant.dequant`, and its Talker's
MoE through `duplex.streaming.fused_moe`.  `install()` puts this build's `streaming/`
and `quant/` directories FIRST on the reference packages' `__path__`, so those four
names (and `duplex.streaming.ep_moe`, `packed_checkpoint`) resolve to the sm_100a
modules, and appends this build's `duplex/` directory LAST on `duplex.__path__`, so
`duplex._lib`, `duplex.clock`, `duplex.health` and the rest are found while every module
the reference has itself -- `duplex.config`, `duplex.loader`, `duplex.fast_engine`,
`duplex.server`, `duplex.streaming.clock`, `duplex.streaming.talker`, ... -- still
resolves to the reference's file.  No file of the reference is modified or hidden.

    import duplex_b200_overlay
    duplex_b200_overlay.install()        # before the hot-path modules are imported
    from duplex.streaming.clock import ...   # the reference's caller, unchanged

install() raises if one of the replaced modules was already imported from the
reference (its objects would stay bound to the old code).
"""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent / "duplex"
REPLACED = ("duplex.streaming.fused_packed_moe", "duplex.streaming.triton_dequant_gemv",
            "duplex.quant.dequant", "duplex.streaming.fused_moe")


def install() -> dict:
    """Overlay onto the `duplex` package that `import duplex` finds (the reference's).
    Returns {module name: file} of the replaced modules after the overlay.  Idempotent."""
    pkg = importlib.import_module("duplex")
    if Path(pkg.__file__).resolve().parent == HERE:
        return {m: str(HERE / (m.split(".", 1)[1].replace(".", "/") + ".py")) for m in REPLACED}
    for m in REPLACED:
        mod = sys.modules.get(m)
        if mod is not None and Path(mod.__file__).resolve().parent.parent not in (HERE,):
            raise RuntimeError(f"{m} was imported from {mod.__file__} before install(); "
                               "call duplex_b200_overlay.install() first")
    streaming = importlib.import_module("duplex.streaming")
    quant = importlib.import_module("duplex.quant")
    for sub, p in ((streaming, HERE / "streaming"), (quant, HERE / "quant")):
        if str(p) not in sub.__path__:
            sub.__path__.insert(0, str(p))
    if str(HERE) not in pkg.__path__:
        pkg.__path__.append(str(HERE))
    return {m: importlib.import_module(m).__file__ for m in REPLACED}
