"""The drop-in modules expose the reference modules' public API (names and signatures).

The fixture tests/golden/reference_api.json is recorded from vflash itself by
tests/golden/make_api_fixture.py.  Every public class and function (and the
hooks callers patch) must exist here with the same parameters in the same
order, kinds and defaults; additions are allowed only as keyword-only
parameters with defaults after the reference's own.
"""

from __future__ import annotations

import importlib
import inspect
import json
from pathlib import Path

import pytest

FIXTURE = json.loads((Path(__file__).parent / "golden" / "reference_api.json").read_text())


def describe(fn) -> list:
    out = []
    for p in inspect.signature(fn).parameters.values():
        default = None if p.default is inspect.Parameter.empty else repr(p.default)
        out.append([p.name, p.kind.name, default])
    return out


def assert_compatible(ours: list, theirs: list, where: str) -> None:
    assert ours[: len(theirs)] == theirs, f"{where}: {ours} does not start with the reference's {theirs}"
    for name, kind, default in ours[len(theirs):]:
        assert kind == "KEYWORD_ONLY" and default is not None, f"{where}: extra parameter {name} must be keyword-only with a default"


CASES = [(module, name) for module, entries in FIXTURE.items() for name in entries]


@pytest.mark.parametrize("module,name", CASES, ids=[f"{m}.{n}" for m, n in CASES])
def test_reference_api_is_present(module, name):
    ours = importlib.import_module(f"vflash_b200.native.{module}")
    assert hasattr(ours, name), f"{module}.{name} is missing"
    spec = FIXTURE[module][name]
    obj = getattr(ours, name)
    if spec["kind"] == "function":
        assert inspect.isfunction(obj)
        assert_compatible(describe(obj), spec["params"], f"{module}.{name}")
    else:
        assert inspect.isclass(obj)
        for method, params in spec["methods"].items():
            assert hasattr(obj, method), f"{module}.{name}.{method} is missing"
            assert_compatible(describe(getattr(obj, method)), params, f"{module}.{name}.{method}")
