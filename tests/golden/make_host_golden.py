"""Generate tests/golden/host_helpers.json by running the REFERENCE'S OWN host helpers.

The reference package cannot be imported here (``import tilec`` needs its Rust
extension), so this script reads tilec/ext.py and tilec/language.py from a reference
checkout (argument or $TILEC_REFERENCE), extracts with ``ast`` only the module-level
host code of the matrix_mul path -- ``cdiv`` (language.py:16-18), ``MAX_BLOCK``
(ext.py:10), ``plan`` (ext.py:29-34), ``SPLITS`` / ``JOINS`` / ``BLOCKS`` (ext.py:37-39),
``_blocks`` (ext.py:43-45) and ``mm_configs`` (ext.py:48-51) -- executes it, and records
its results on a grid of arguments.  tests/test_tilec_compat.py compares the B200
build's helpers of the same names against these values.

Usage:  python tests/golden/make_host_golden.py /path/to/tilec-checkout
"""
import ast
import json
import os
import sys

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "host_helpers.json")
WANT_EXT = {"MAX_BLOCK", "plan", "SPLITS", "JOINS", "BLOCKS", "_blocks", "mm_configs"}

# Arguments recorded: plan(N) and plan(N, block); mm_configs(M1, N, M2).
PLAN_N = [0, 1, 2, 3, 4, 5, 15, 16, 17, 63, 64, 65, 255, 256, 257, 1000, 1023, 1024, 1025, 4095, 4096, 4097,
          5000, 8192, 16384, 100000]
PLAN_BLOCKED = [(100, 7), (4096, 256), (5000, 1024), (1, 1), (0, 64)]
MM_ARGS = [(1, 1, 1), (1, 16, 1), (3, 64, 5), (8, 64, 8), (512, 4096, 64), (64, 1024, 64), (1000, 3001, 777),
           (2048, 2048, 2048), (7, 100, 3), (4096, 65536, 2), (2, 2047, 9)]


def _defs(path, names):
    tree = ast.parse(open(path).read(), path)
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            keep.append(node)
        elif isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id in names for t in node.targets):
            keep.append(node)
    return ast.Module(body=keep, type_ignores=[])


def main(ref):
    ns = {}
    exec(compile(_defs(os.path.join(ref, "tilec", "language.py"), {"cdiv"}), "language.py", "exec"), ns)
    exec(compile(_defs(os.path.join(ref, "tilec", "ext.py"), WANT_EXT), "ext.py", "exec"), ns)
    missing = (WANT_EXT | {"cdiv"}) - set(ns)
    if missing:
        raise SystemExit(f"not found in the reference: {sorted(missing)}")
    out = {
        "MAX_BLOCK": ns["MAX_BLOCK"], "SPLITS": list(ns["SPLITS"]), "JOINS": list(ns["JOINS"]),
        "BLOCKS": list(ns["BLOCKS"]),
        "cdiv": [[a, b, ns["cdiv"](a, b)] for a in (0, 1, 5, 4096, 5000) for b in (1, 3, 4096)],
        "plan": [[n, list(ns["plan"](n))] for n in PLAN_N],
        "plan_block": [[n, b, list(ns["plan"](n, b))] for n, b in PLAN_BLOCKED],
        "mm_configs": [[list(a), [list(c) for c in ns["mm_configs"](*a)]] for a in MM_ARGS],
    }
    with open(OUT, "w") as f:
        json.dump(out, f, indent=0)
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TILEC_REFERENCE", "."))
