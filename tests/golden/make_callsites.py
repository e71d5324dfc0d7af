"""Record how the reference's Python package calls its native module.

    python tests/golden/make_callsites.py <reference checkout>

Parses the reference's ``src/python/mhc/ops.py`` with ``ast`` (nothing is
imported or executed) and writes ``mhc_ascend_callsites.json``: one entry per
``mhc_ascend.<function>(...)`` call with its line, positional argument count
and keyword names.  ``tests/test_shim.py`` checks that the drop-in module
``mhc_ascend_b200.mhc_ascend_shim`` accepts every one of these calls, so the
reference's ops.py can run on it unchanged.  Nothing at test time reads the
reference: the tests only read the JSON.
"""
import ast
import json
import os
import sys


def callsites(ops_path):
    tree = ast.parse(open(ops_path).read())
    out = []
    for node in ast.walk(tree):
        if isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute) and \
                isinstance(node.func.value, ast.Name) and node.func.value.id == "mhc_ascend":
            out.append({"function": node.func.attr, "line": node.lineno,
                        "positional": len(node.args),
                        "keywords": sorted(k.arg for k in node.keywords if k.arg)})
    return sorted(out, key=lambda c: c["line"])


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MHC_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: make_callsites.py <reference checkout>")
    sites = callsites(os.path.join(root, "src", "python", "mhc", "ops.py"))
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mhc_ascend_callsites.json")
    with open(dst, "w") as f:
        json.dump({"source": "src/python/mhc/ops.py", "calls": sites}, f, indent=1)
    print(f"wrote {len(sites)} call sites to {dst}")


if __name__ == "__main__":
    main()
