"""The drop-in contract, checked without a GPU: every manifest op glmkv replaces binds to our kernel
entry and to our C launcher by position, with the same pointer / scalar kind, element type and
constness.

The manifest's parameter lists come from ``tests/golden/manifest_params.json``, which
``tests/golden/make_manifest_params.py`` extracts from kern-glm53 ``scripts/gen.py`` with ``ast``.
The kernel parameter lists are read from the CUDA sources, the launcher lists from
``include/glmkv.h`` and the ctypes binding.
"""
import ctypes
import json
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
MANIFEST = json.loads((ROOT / "tests" / "golden" / "manifest_params.json").read_text())["ops"]
KERNELS = ROOT / "kern-glm53_b200" / "csrc" / "glmkv_kernels.cuh"
HEADER = ROOT / "include" / "glmkv.h"

# the manifest ops of the cache path and of the ops built beside it
OURS = ["plan", "mla_prep_full", "mla_prep_shared", "idx_gather", "kv_dequant", "topk_stream", "topk_slots",
        "q_post_full", "q_post_shared", "add_rms_quant", "rms_quant", "head_norm", "quant_o"]

KERNEL_ELEM = {"bf16": "bf16", "u8": "u8", "i32": "int", "i64": "long long", "u32": "unsigned", "f32": "float",
               "state": "u8"}
HEADER_ELEM = {"bf16": "void", "u8": "void", "i32": "int32_t", "i64": "int64_t", "u32": "uint32_t", "f32": "float",
               "state": "void"}


def manifest_kind(p):
    """'in buffer<i32>' -> ('ptr', 'i32', const=True); 'i32' -> ('int', None, None)."""
    if p == "i32":
        return ("int", None, None)
    m = re.fullmatch(r"(in|out|inout) (?:buffer<(\w+)>|(state))", p)
    assert m, p
    return ("ptr", m.group(2) or "state", m.group(1) == "in")


def split_params(text):
    return [" ".join(x.split()) for x in text.split(",") if x.strip()]


def kernel_params():
    """entry name -> its parameter declarations, from the extern "C" __global__ definitions."""
    src = KERNELS.read_text()
    macros = {m.group(1): m.group(2).replace("\\\n", " ")
              for m in re.finditer(r"#define (\w+)\s+((?:.*\\\n)*.*)", src)}
    out = {}
    for m in re.finditer(r'extern "C" __global__ void (?:__launch_bounds__\([^)]*\)\s*)?(\w+)\(([^)]*)\)', src):
        body = m.group(2).strip()
        body = macros.get(body, body)
        out[m.group(1)] = split_params(body)
    return out


def header_params():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return {m.group(1): split_params(m.group(2)) for m in re.finditer(r"^int (glmkv_\w+)\(([^)]*)\);", text, re.M)}


def decl_kind(decl, elem_names):
    """A C declaration -> (kind, element type, const)."""
    d = decl.replace("__restrict__", "").replace("glmkv::", "")
    d = " ".join(d.split())
    if "*" not in d:
        assert re.fullmatch(r"int \w+", d), decl
        return ("int", None, None)
    const = d.startswith("const ")
    base = d[len("const "):] if const else d
    base = base.split("*")[0].strip()
    return ("ptr", base, const)


@pytest.mark.parametrize("op", OURS)
def test_kernel_entry_binds_like_the_reference(op):
    spec = MANIFEST[op]
    kp = kernel_params()
    for entry in spec["entries"]:
        assert entry in kp, f"{entry} is not an extern \"C\" __global__ entry"
        decls = kp[entry]
        assert len(decls) == len(spec["params"]), (entry, decls)
        for i, (p, d) in enumerate(zip(spec["params"], decls)):
            kind, elem, const = manifest_kind(p)
            got = decl_kind(d, KERNEL_ELEM)
            assert got[0] == kind, (entry, i, p, d)
            if kind == "ptr":
                assert got[1] == KERNEL_ELEM[elem], (entry, i, p, d)
                assert got[2] == const, (entry, i, p, d)


@pytest.mark.parametrize("op", OURS)
def test_c_launcher_binds_like_the_reference(op):
    spec = MANIFEST[op]
    hp = header_params()
    from glmkv import _lib
    for entry in spec["entries"]:
        name = "glmkv_" + entry[len("glm_"):]
        decls = hp[name]
        assert decls[-1] == "glmkv_stream_t stream", name
        decls = decls[:-1]
        assert len(decls) == len(spec["params"]), (name, decls)
        argtypes = _lib.SIGNATURES[name]
        assert argtypes[-1] is ctypes.c_void_p and len(argtypes) == len(decls) + 1
        for i, (p, d) in enumerate(zip(spec["params"], decls)):
            kind, elem, const = manifest_kind(p)
            got = decl_kind(d, HEADER_ELEM)
            assert got[0] == kind, (name, i, p, d)
            assert argtypes[i] is (ctypes.c_void_p if kind == "ptr" else ctypes.c_int), (name, i)
            if kind == "ptr":
                assert got[1] == HEADER_ELEM[elem], (name, i, p, d)
                assert got[2] == const, (name, i, p, d)


def test_nulled_arguments_are_optional_in_our_launchers():
    """Every position the manifest passes as literal 0 (G.nulled) is documented as optional."""
    text = HEADER.read_text()
    for op in OURS:
        spec = MANIFEST[op]
        if not spec["nulled"]:
            continue
        for entry in spec["entries"]:
            name = "glmkv_" + entry[len("glm_"):]
            decls = header_params()[name]
            names = [d.split()[-1].lstrip("*") for d in decls]
            # the doc comment right above the declaration names each nulled argument with "NULL"
            block = text[:text.index(f"int {name}(")].rsplit("*/", 1)[0].rsplit("/*", 1)[-1]
            if "Same arguments" in block:  # glmkv_mla_prep_fp8 refers to glmkv_mla_prep
                block = text[:text.index("int glmkv_mla_prep(")].rsplit("*/", 1)[0].rsplit("/*", 1)[-1]
            assert "NULL" in block, name
            for i in spec["nulled"]:
                assert names[i] in block, (name, names[i])


def test_integration_snippets_are_all_parsed():
    """Every `G.b200(...)` launch of INTEGRATION.md's manifest snippets is one that the GPU test of the
    launch shapes (tests/test_gpu_cubin.py) parses, and names a kernel the cubin exports: a snippet the
    parser skipped would escape that check."""
    from test_gpu_cubin import _snippet_shapes

    text = (ROOT / "INTEGRATION.md").read_text()
    calls = re.findall(r'G\.b200\((?:"(glm_\w+)"|(prep))', text)
    want = []
    for entry, prep in calls:
        want += ["glm_mla_prep_fp8", "glm_mla_prep"] if prep else [entry]
    shapes = _snippet_shapes()
    got = [e for e, *_ in shapes if e != "glm_mqa_logits_paged"]  # that one is a `launch(...)`, not G.b200
    assert got == want
    assert any(e == "glm_mqa_logits_paged" for e, *_ in shapes)
    src = KERNELS.read_text() + (ROOT / "kern-glm53_b200" / "csrc" / "glmkv_mqa.cuh").read_text()
    for e, *_ in shapes:
        assert re.search(r'extern "C" __global__ void(?:\s+__launch_bounds__\([^)]*\))?\s+' + e + r"\(", src), e
