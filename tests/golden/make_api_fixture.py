"""Record the public API of the reference modules this library replaces (run where vflash is importable).

Writes tests/golden/reference_api.json: for each module the public classes and
functions (plus the hooks callers patch) with their parameter names, kinds and
defaults, and for classes the public methods.  tests/test_api_surface.py checks
the drop-in modules against it.

    PYTHONPATH=<vflash>/src python tests/golden/make_api_fixture.py
"""

from __future__ import annotations

import importlib
import inspect
import json
from pathlib import Path

MODULES = ("h3_fp8_linear", "h3_fp8_activation", "h3_nvfp4_linear", "h3_fused_ops")
HOOKS = {"_require_device", "_operators", "_quantize_activation_torch"}


def describe(fn) -> list:
    out = []
    for p in inspect.signature(fn).parameters.values():
        default = None if p.default is inspect.Parameter.empty else repr(p.default)
        out.append([p.name, p.kind.name, default])
    return out


def main() -> None:
    api = {}
    for short in MODULES:
        name = f"vflash.native.{short}"
        module = importlib.import_module(name)
        entries = {}
        for attr, obj in vars(module).items():
            if attr.startswith("_") and attr not in HOOKS:
                continue
            if getattr(obj, "__module__", None) != name:
                continue
            if inspect.isclass(obj):
                methods = {m: describe(f) for m, f in vars(obj).items()
                           if inspect.isfunction(f) and (not m.startswith("_") or m == "__init__")}
                entries[attr] = {"kind": "class", "methods": methods}
            elif inspect.isfunction(obj):
                entries[attr] = {"kind": "function", "params": describe(obj)}
        api[short] = entries
    path = Path(__file__).with_name("reference_api.json")
    path.write_text(json.dumps(api, indent=1, sort_keys=True) + "\n")
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
