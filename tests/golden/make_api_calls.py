"""Writes reference_api_calls.json: every use the reference's Python makes of
its three native modules (src/aggregator.py and src/worker/*.py), read with
the ast module: for each call, the module, the function, the number of
positional arguments and the keyword names; for each attribute read that is
not a call (OP_* constants and the like), its name. tests/test_dropin_api_cpu.py
checks that this build's modules of the same names accept every one.

Run from the repository root where the reference checkout is available:
    python tests/golden/make_api_calls.py /path/to/reference
"""
from __future__ import annotations

import ast
import json
import sys
from pathlib import Path

sys.dont_write_bytecode = True
OUT = Path(__file__).resolve().parent / "reference_api_calls.json"
# the names the reference binds its modules to
ALIASES = {"ext_agg": "ext_aggregator", "ext_aggregator": "ext_aggregator", "extq": "ext_ipc_queue",
           "ext_ipc_queue": "ext_ipc_queue", "ub": "ext_unified_barrier", "ext_unified_barrier": "ext_unified_barrier"}


def _module_of(node: ast.AST):
    """ext_agg.X / self.ext_agg.X / extq.X / ub.X -> the module's name."""
    if isinstance(node, ast.Name):
        return ALIASES.get(node.id)
    if isinstance(node, ast.Attribute) and isinstance(node.value, ast.Name) and node.value.id == "self":
        return ALIASES.get(node.attr)
    return None


def scan(files):
    calls, attrs = set(), set()
    for f in files:
        tree = ast.parse(Path(f).read_text(), filename=str(f))
        called = set()
        for node in ast.walk(tree):
            if isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute):
                mod = _module_of(node.func.value)
                if mod and not any(isinstance(a, ast.Starred) for a in node.args):
                    kws = tuple(sorted(k.arg for k in node.keywords if k.arg))
                    calls.add((mod, node.func.attr, len(node.args), kws))
                    called.add(id(node.func))
        for node in ast.walk(tree):
            if isinstance(node, ast.Attribute) and id(node) not in called:
                mod = _module_of(node.value)
                if mod:
                    attrs.add((mod, node.attr))
    return calls, attrs


def main(ref_root: str) -> None:
    src = Path(ref_root) / "src"
    files = sorted([src / "aggregator.py", *sorted((src / "worker").glob("*.py"))])
    calls, attrs = scan(files)
    out = {"files": [str(f.relative_to(ref_root)) for f in files],
           "calls": [{"module": m, "name": n, "positional": p, "keywords": list(k)} for m, n, p, k in sorted(calls)],
           "attributes": [{"module": m, "name": n} for m, n in sorted(attrs)]}
    OUT.write_text(json.dumps(out, indent=1) + "\n")
    print(OUT.name, len(out["calls"]), "calls,", len(out["attributes"]), "attributes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../reference")
