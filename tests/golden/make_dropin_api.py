"""Record which names the reference's harnesses import from the modules the
drop-ins replace, and the keyword arguments their call sites pass.

Parses (does not run) every ``.py`` file of the cache-barrier reference and
writes ``dropin_api.json`` next to this script:

    {"imports": {module: {name: [files that import it]}},
     "call_keywords": {name: [keyword names passed at call sites]}}

``tests/test_dropin_api.py`` checks the drop-in modules against it on CPU.
Only needed to regenerate the fixture:

    python tests/golden/make_dropin_api.py --ref /path/to/cache-barrier
"""

from __future__ import annotations

import argparse
import ast
import json
import os

# Modules of the reference that the drop-ins stand in for (as the harnesses
# import them: each harness puts its own directory or the kernel directory on
# sys.path, so the names are bare).
MODULES = ("bench_l2_barrier", "w8a8_bmm", "int4_batched_gemm", "int4_batched_gemm_v2", "triton_gemm")


def scan(ref: str):
    imports: dict[str, dict[str, set]] = {m: {} for m in MODULES}
    keywords: dict[str, set] = {}
    for root, _dirs, files in os.walk(ref):
        if "/." in root:
            continue
        for fn in files:
            if not fn.endswith(".py"):
                continue
            path = os.path.join(root, fn)
            rel = os.path.relpath(path, ref)
            try:
                tree = ast.parse(open(path, encoding="utf-8", errors="replace").read())
            except SyntaxError:
                continue
            local = {}
            for node in ast.walk(tree):
                if isinstance(node, ast.ImportFrom) and node.module:
                    mod = node.module.split(".")[-1]
                    if mod in imports:
                        for a in node.names:
                            imports[mod].setdefault(a.name, set()).add(rel)
                            local[a.asname or a.name] = a.name
            for node in ast.walk(tree):
                if isinstance(node, ast.Call):
                    f = node.func
                    if isinstance(f, ast.Subscript):  # kernel[grid](...)
                        f = f.value
                    name = f.id if isinstance(f, ast.Name) else None
                    if name in local:
                        ks = keywords.setdefault(local[name], set())
                        ks.update(k.arg for k in node.keywords if k.arg is not None)
    return imports, keywords


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the cache-barrier reference checkout")
    args = ap.parse_args()
    imports, keywords = scan(args.ref)
    out = {
        "imports": {m: {n: sorted(fs) for n, fs in sorted(d.items())} for m, d in imports.items() if d},
        "call_keywords": {n: sorted(k) for n, k in sorted(keywords.items())},
    }
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "dropin_api.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print("wrote", dst)


if __name__ == "__main__":
    main()
