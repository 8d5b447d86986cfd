"""The manifest's parameter lists of the ops glmkv replaces, read from kern-glm53's generator.

kern binds a program's buffers, states and scalars to an op by position in its ``params`` list
(kern-glm53 scripts/gen.py:310-311), so that list is the drop-in contract. This script reads
``scripts/gen.py`` with ``ast`` (it is not imported or run), finds every ``G.plain`` / ``G.nulled``
call on the ``glm_glue`` module, resolves list variables assigned in the same function
(``norm_params``, ``prep_params``) and the entry variable ``prep`` (both of its values), and writes
``manifest_params.json`` beside this file: op -> {entries, params, nulled, line}.

    python tests/golden/make_manifest_params.py path/to/kern-glm53
    GLMKV_REFERENCE_ROOT=path/to/kern-glm53 python tests/golden/make_manifest_params.py

The CPU test ``tests/test_manifest.py`` checks the C ABI header and the kernels' parameter lists
against the committed JSON, so it runs where the reference tree is absent.
"""
import ast
import json
import os
import pathlib
import sys

HERE = pathlib.Path(__file__).resolve().parent


def literal(node, env):
    if isinstance(node, ast.Name):
        return env[node.id]
    return ast.literal_eval(node)


def collect(tree):
    ops = {}
    for fn in ast.walk(tree):
        if not isinstance(fn, ast.FunctionDef):
            continue
        env = {}
        for st in ast.walk(fn):
            # list literals and the ternary entry name assigned to plain names inside the function
            if isinstance(st, ast.Assign) and len(st.targets) == 1 and isinstance(st.targets[0], ast.Name):
                v = st.value
                if isinstance(v, ast.List):
                    try:
                        env[st.targets[0].id] = ast.literal_eval(v)
                    except ValueError:
                        pass
                elif isinstance(v, ast.IfExp) and all(isinstance(x, ast.Constant) for x in (v.body, v.orelse)):
                    env[st.targets[0].id] = [v.body.value, v.orelse.value]
        for st in ast.walk(fn):
            calls = []
            if isinstance(st, ast.Dict):
                calls = [(k.value, v) for k, v in zip(st.keys, st.values) if isinstance(k, ast.Constant)]
            elif isinstance(st, ast.Assign) and isinstance(st.targets[0], ast.Subscript):
                key = st.targets[0].slice
                if isinstance(key, ast.Constant):
                    calls = [(key.value, st.value)]
            for name, call in calls:
                if not (isinstance(call, ast.Call) and isinstance(call.func, ast.Attribute)
                        and call.func.attr in ("plain", "nulled")):
                    continue
                if not (isinstance(call.args[0], ast.Constant) and call.args[0].value == "glm_glue"):
                    continue
                entry = literal(call.args[1], env)
                entries = entry if isinstance(entry, list) else [entry]
                params = literal(call.args[2], env)
                nulled = sorted(literal(call.args[3], env)) if call.func.attr == "nulled" else []
                ops[name] = {"entries": entries, "params": params, "nulled": nulled, "line": call.lineno}
    return ops


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GLMKV_REFERENCE_ROOT")
    if not root:
        raise SystemExit("give the kern-glm53 checkout as the argument or in GLMKV_REFERENCE_ROOT")
    ref = pathlib.Path(root)
    if not (ref / "scripts" / "gen.py").exists():
        raise SystemExit(f"{ref} has no scripts/gen.py: not a kern-glm53 checkout")
    gen = ref / "scripts" / "gen.py"
    ops = collect(ast.parse(gen.read_text()))
    out = HERE / "manifest_params.json"
    out.write_text(json.dumps({"source": "kern-glm53 scripts/gen.py", "ops": dict(sorted(ops.items()))}, indent=1)
                   + "\n")
    print(f"{len(ops)} glm_glue ops written to {out}")


if __name__ == "__main__":
    main()
