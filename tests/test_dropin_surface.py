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
