"""Record the public Python surface of the reference's hot-path modules.

    python tests/golden/make_api_manifest.py --ref /path/to/qwen3-omni-duplex

Parses (with `ast`, nothing is imported or run) the reference modules that this
build replaces -- src/duplex/streaming/fused_packed_moe.py,
src/duplex/streaming/triton_dequant_gemv.py, src/duplex/quant/dequant.py and the
Talker's src/duplex/streaming/fused_moe.py -- and
writes `reference_api.json` next to this script:

  modules:  {module: {name: {"kind": "function" | "class" | "value",
                             "params": [[name, default-source or null], ...]}}}
            (public top-level names, plus the methods of public classes as
            "Class.method"; `_dequant` and `_stack_packed` are included because
            callers and tests reach them)
  imports:  [[caller file, module, name], ...] every `from duplex.<module> import
            <name>` in the reference's sources that targets one of those modules.

tests/test_dropin_surface.py checks the repo's mirror modules against this file on
any host, and re-derives it from the reference when a checkout is available.
"""

from __future__ import annotations

import argparse
import ast
import json
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
MODULES = {
    "duplex.streaming.fused_packed_moe": "src/duplex/streaming/fused_packed_moe.py",
    "duplex.streaming.triton_dequant_gemv": "src/duplex/streaming/triton_dequant_gemv.py",
    "duplex.quant.dequant": "src/duplex/quant/dequant.py",
    "duplex.streaming.fused_moe": "src/duplex/streaming/fused_moe.py",
}
KEEP_PRIVATE = {"_dequant", "_stack_packed"}


def _params(fn: ast.FunctionDef) -> list:
    a = fn.args
    pos = a.posonlyargs + a.args
    defaults = [None] * (len(pos) - len(a.defaults)) + [ast.unparse(d) for d in a.defaults]
    out = [[p.arg, d] for p, d in zip(pos, defaults)]
    for p, d in zip(a.kwonlyargs, a.kw_defaults):
        out.append([p.arg, None if d is None else ast.unparse(d)])
    return out


def _public(name: str) -> bool:
    return not name.startswith("_") or name in KEEP_PRIVATE


def module_surface(path: Path) -> dict:
    tree = ast.parse(path.read_text())
    out = {}
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and _public(node.name):
            out[node.name] = {"kind": "function", "params": _params(node)}
        elif isinstance(node, ast.ClassDef) and _public(node.name):
            out[node.name] = {"kind": "class", "params": []}
            for sub in node.body:
                if isinstance(sub, ast.FunctionDef) and (_public(sub.name) or sub.name == "__init__"):
                    out[f"{node.name}.{sub.name}"] = {"kind": "function", "params": _params(sub)}
        elif isinstance(node, ast.Assign):
            for t in node.targets:
                if isinstance(t, ast.Name) and _public(t.id):
                    out[t.id] = {"kind": "value", "params": []}
    return out


def caller_imports(ref: Path) -> list:
    found = []
    for f in sorted((ref / "src").rglob("*.py")):
        for node in ast.walk(ast.parse(f.read_text())):
            if isinstance(node, ast.ImportFrom) and node.module in MODULES:
                for alias in node.names:
                    found.append([str(f.relative_to(ref)), node.module, alias.name])
    return found


def build(ref: Path) -> dict:
    return {"modules": {m: module_surface(ref / p) for m, p in MODULES.items()},
            "imports": caller_imports(ref)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("DUPLEX_REFERENCE"),
                    help="checkout of the reference project (or set DUPLEX_REFERENCE)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("give --ref (or DUPLEX_REFERENCE): the reference checkout to parse")
    data = build(Path(a.ref))
    (HERE / "reference_api.json").write_text(json.dumps(data, indent=1, sort_keys=True) + "\n")
    n = sum(len(v) for v in data["modules"].values())
    print(f"wrote reference_api.json: {n} names, {len(data['imports'])} caller imports")


if __name__ == "__main__":
    main()
