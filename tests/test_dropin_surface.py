"""The drop-in modules expose the reference's whole public surface (CPU only).

`tests/golden/reference_api.json` records every public name of the three
reference modules this build replaces (fused_packed_moe, triton_dequant_gemv,
quant.dequant), with parameter lists, and every `from duplex.<module> import
<name>` in the reference's callers (clock.py, fast_engine.py, server.py, speak.py,
probe.py, ...).  Each name must exist here, each function must accept the
reference's parameters in the same order with the same defaults (extra trailing
parameters are allowed), and every caller import must resolve.
"""

import importlib
import inspect
import json
import os
from pathlib import Path

import pytest
import torch

HERE = Path(__file__).resolve().parent
MANIFEST = json.loads((HERE / "golden" / "reference_api.json").read_text())


def _resolve(module, dotted):
    obj = importlib.import_module(module)
    for part in dotted.split("."):
        obj = getattr(obj, part)
    return obj


def _eval_default(src):
    if src is None:
        return inspect.Parameter.empty
    return eval(src, {"torch": torch})  # literal defaults and torch dtypes only


CASES = [(m, n, spec) for m, names in sorted(MANIFEST["modules"].items())
         for n, spec in sorted(names.items())]


@pytest.mark.parametrize("module,name,spec", CASES, ids=[f"{m}:{n}" for m, n, _ in CASES])
def test_reference_name_is_exported(module, name, spec):
    obj = _resolve(module, name)
    if spec["kind"] != "function":
        return
    ours = list(inspect.signature(obj).parameters.values())
    ref = spec["params"]
    assert len(ours) >= len(ref), f"{name}: fewer parameters than the reference"
    for (rname, rdef), p in zip(ref, ours):
        assert p.name == rname, f"{name}: parameter {p.name!r} where the reference has {rname!r}"
        want = _eval_default(rdef)
        if want is not inspect.Parameter.empty:  # a default gained here breaks no caller
            assert p.default == want, f"{name}.{rname}: default {p.default!r} != {want!r}"
    for p in ours[len(ref):]:
        assert p.default is not inspect.Parameter.empty or p.kind == p.VAR_KEYWORD, \
            f"{name}: extra parameter {p.name!r} must be optional"


@pytest.mark.parametrize("caller,module,name", MANIFEST["imports"],
                         ids=[f"{c}:{n}" for c, _, n in MANIFEST["imports"]])
def test_reference_callers_find_their_imports(caller, module, name):
    assert hasattr(importlib.import_module(module), name), f"{caller} imports {module}.{name}"


def test_manifest_matches_reference_checkout():
    ref = os.environ.get("DUPLEX_REFERENCE")
    if not ref or not Path(ref).is_dir():
        pytest.skip("no reference checkout (set DUPLEX_REFERENCE to re-derive the manifest)")
    spec = importlib.util.spec_from_file_location("_mk", HERE / "golden" / "make_api_manifest.py")
    mk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mk)
    assert mk.build(Path(ref)) == MANIFEST


def test_patched_linear_refuses_cpu_compute():
    """No CPU path: a patched packed Linear called on a CPU input raises at call time."""
    from types import SimpleNamespace
    from duplex import _lib
    from duplex.quant.dequant import patch_packed_linears

    class Packed(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.register_buffer("weight_packed", torch.zeros(16, 8, dtype=torch.int32))
            self.register_buffer("weight_scale", torch.ones(16, 2, dtype=torch.float16))
            self.register_buffer("weight_shape", torch.tensor([16, 64]))
            self._old_forward = SimpleNamespace()

    model = torch.nn.Sequential(Packed(), torch.nn.Identity())
    assert patch_packed_linears(model, verbose=False) == 1
    assert "_old_forward" not in model[0].__dict__
    with pytest.raises(_lib.DuplexError):
        model(torch.zeros(1, 64, dtype=torch.float16))


def test_place_unpacked_keeps_packed_tensors():
    from duplex.quant.dequant import place_unpacked, place_thinker

    class Packed(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.register_buffer("weight_packed", torch.zeros(4, 1, dtype=torch.int32))
            self.register_buffer("weight_scale", torch.ones(4, 1))

    root = torch.nn.Sequential(torch.nn.LayerNorm(8), Packed())
    stats = place_unpacked(root, device="meta", verbose=False)
    assert stats == {"moved_params": 16, "kept_on_host": 8, "device": "meta"}
    assert root[0].weight.device.type == "meta" and root[1].weight_packed.device.type == "cpu"
    assert place_thinker is place_unpacked


def test_overlay_onto_the_installed_reference():
    """duplex_b200_overlay.install() on the reference installed in baseline/_ref: the
    three hot-path modules resolve to this build, every other reference module (config,
    loader, streaming.clock, ...) to the reference's own file, and the reference's
    clock path finds the names it imports."""
    import subprocess
    import sys
    root = HERE.parent
    ref, pkg = root / "baseline" / "_ref", root / "qwen3-omni-duplex_b200"
    if not (ref / "duplex" / "streaming" / "clock.py").exists():
        pytest.skip("reference not installed in baseline/_ref")
    code = f"""
import sys, json
sys.path[:0] = [{str(ref)!r}, {str(pkg)!r}]
import duplex
out = dict(init=duplex.__file__)
import duplex_b200_overlay
out["files"] = duplex_b200_overlay.install()
import duplex.config, duplex.loader, duplex._lib
from duplex.streaming.fused_packed_moe import fuse_packed_moe_blocks
from duplex.quant.dequant import patch_packed_linears
from duplex.streaming.triton_dequant_gemv import patch_attention_to_triton
out.update(config=duplex.config.__file__, loader=duplex.loader.__file__, lib=duplex._lib.__file__,
           fpm=sys.modules[fuse_packed_moe_blocks.__module__].__file__)
import duplex.streaming.clock as c
out["clock"] = c.__file__
out["again"] = duplex_b200_overlay.install()
print(json.dumps(out))
"""
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                       cwd=str(root / "tests"))
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    under = lambda f, d: Path(f).resolve().is_relative_to(d.resolve())  # noqa: E731
    assert under(out["init"], ref)
    assert all(under(f, pkg) for f in out["files"].values()) and out["again"] == out["files"]
    assert under(out["fpm"], pkg) and under(out["lib"], pkg)
    assert under(out["config"], ref) and under(out["loader"], ref) and under(out["clock"], ref)
