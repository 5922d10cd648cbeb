"""Public Python API parity with StateSpectre's own package.

Reads StateSpectre's ``state_spectre/__init__.py`` from the reference build in
``baseline/_ref`` (skipped when absent) as text, with ``ast``, and checks that
``import state_spectre`` here offers every public class, method, property and
function it defines (constructors of the objects the library hands out
excepted), with every parameter it names, positional parameters in
the same order, and a default wherever the reference has one, so code written
against the reference calls this package unchanged.
"""

import ast
import inspect
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_PKG = os.path.join(ROOT, "baseline", "_ref", "state_spectre")


# Objects the library hands out (sessions, handles, records): user code gets
# them from calls and never builds them, so their constructors are internal.
LIBRARY_MADE = {"Off", "OffloadHandle", "PrefetchHandle", "ManagedRecord", "CanonicalHandle"}


def _reference_api(filename: str):
    path = os.path.join(REF_PKG, filename)
    if not os.path.exists(path):
        pytest.skip("reference build not present (python baseline/build_reference.py)")
    with open(path) as f:
        tree = ast.parse(f.read())
    classes, funcs = {}, {}
    for node in tree.body:
        if isinstance(node, ast.ClassDef) and not node.name.startswith("_"):
            classes[node.name] = [n for n in node.body if isinstance(n, ast.FunctionDef)
                                  and (not n.name.startswith("_") or n.name == "__init__")]
        elif isinstance(node, ast.FunctionDef) and not node.name.startswith("_"):
            funcs[node.name] = node
    return classes, funcs


def _params(fn: ast.FunctionDef):
    a = fn.args
    pos = [x.arg for x in a.posonlyargs + a.args]
    with_default = set(pos[len(pos) - len(a.defaults):]) if a.defaults else set()
    kw = [x.arg for x in a.kwonlyargs]
    with_default |= {x.arg for x, d in zip(a.kwonlyargs, a.kw_defaults) if d is not None}
    return pos, kw, with_default


def _check_callable(qual: str, ref_fn: ast.FunctionDef, ours) -> list:
    problems = []
    try:
        sig = inspect.signature(ours)
    except (TypeError, ValueError):
        return problems  # a builtin or C callable: presence is what can be checked
    params = sig.parameters
    has_var_kw = any(p.kind == p.VAR_KEYWORD for p in params.values())
    pos, kw, with_default = _params(ref_fn)
    if pos and pos[0] in ("self", "cls"):
        pos = pos[1:]
    our_pos = [n for n, p in params.items() if p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD)]
    if our_pos and our_pos[0] in ("self", "cls"):
        our_pos = our_pos[1:]
    for i, name in enumerate(pos):
        if name not in params and not has_var_kw:
            problems.append(f"{qual}: parameter {name!r} missing")
        elif name in params and name not in with_default and (i >= len(our_pos) or our_pos[i] != name):
            problems.append(f"{qual}: positional parameter {name!r} not at position {i}")
    for name in kw:
        if name not in params and not has_var_kw:
            problems.append(f"{qual}: keyword parameter {name!r} missing")
    for name in with_default:
        if name in params and params[name].default is inspect.Parameter.empty:
            problems.append(f"{qual}: parameter {name!r} has no default here")
    return problems


@pytest.mark.parametrize("filename,module", [("__init__.py", "state_spectre"),
                                             ("_rollout.py", "state_spectre._rollout"),
                                             ("_wire.py", "state_spectre._wire")])
def test_state_spectre_offers_the_reference_api(filename, module):
    import importlib

    ns = importlib.import_module(module)
    classes, funcs = _reference_api(filename)
    problems = []
    for cname, methods in classes.items():
        ours = getattr(ns, cname, None)
        if ours is None:
            problems.append(f"class {cname} missing")
            continue
        for m in methods:
            if m.name == "__init__" and cname in LIBRARY_MADE:
                continue
            attr = inspect.getattr_static(ours, m.name, None)
            if attr is None:
                problems.append(f"{cname}.{m.name} missing")
                continue
            is_prop = any(isinstance(d, ast.Name) and d.id == "property" for d in m.decorator_list)
            if is_prop or isinstance(attr, property):
                continue
            problems += _check_callable(f"{cname}.{m.name}", m, getattr(ours, m.name))
    for fname, node in funcs.items():
        ours = getattr(ns, fname, None)
        if ours is None:
            problems.append(f"function {fname} missing")
            continue
        problems += _check_callable(fname, node, ours)
    assert not problems, problems


def _load_reference_wire():
    import importlib.util

    path = os.path.join(REF_PKG, "_wire.py")
    if not os.path.exists(path):
        pytest.skip("reference build not present (python baseline/build_reference.py)")
    spec = importlib.util.spec_from_file_location("_ssref_wire_only", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_wire_helpers_produce_and_read_what_the_reference_helpers_do():
    """StateSpectre's pure-Python wire helpers and this package's, side by
    side: the same request bytes for the same arguments (filters included),
    the same dicts from the reference daemon's captured responses, the same
    frames and export headers."""
    import json
    import struct

    from state_spectre import _wire as ours

    ref = _load_reference_wire()
    job = (0, 12345678901234567890, 3, "job/a")
    assert ours.encode_get_latest(*job, 2) == ref.encode_get_latest(*job, 2)
    for flt in (None, {}, {"tp": 3}, {"pp": 1, "tp": 2, "ep": 3, "etp": 4, "expert": -7}):
        assert ours.encode_get_manifest(*job, 2, 9, flt) == ref.encode_get_manifest(*job, 2, 9, flt), flt
    for transport, target in ((1, "127.0.0.1:5555"), (2, "/tmp/x.bin"), (3, "nic0|abcd")):
        assert ours.encode_pull(*job, 2, 9, 77, transport, target) == ref.encode_pull(*job, 2, 9, 77, transport, target)
    assert ours.make_frame(25, b"abc", 1) == ref.make_frame(25, b"abc", 1)
    hdr = struct.pack("<IIQQQQ", ref.EXPORT_MAGIC, 1, 5, 100, 7, 8)
    assert ours.parse_export_header(hdr) == ref.parse_export_header(hdr)
    with open(os.path.join(ROOT, "tests", "golden", "reference_wire.json")) as f:
        records = json.load(f)["records"]
    seen = set()
    for r in records:
        payload = bytes.fromhex(r["response_hex"])
        for op, fn in ((24, "decode_get_latest_resp"), (25, "decode_get_manifest_resp"), (26, "decode_pull_resp")):
            if r["op"] == op:
                assert getattr(ours, fn)(payload) == getattr(ref, fn)(payload), fn
                seen.add(fn)
    assert len(seen) == 3


def test_cpp_agent_interface_offers_the_reference_methods_and_types():
    """StateSpectre's C++ `offload::OffloadAgent` (its header, read as text
    from the reference build): every public method name and every struct the
    header declares is in this repository's `ofld/offload_agent.h`, whose
    OffloadAgent forwards to this agent (`csrc/tests/compat_agent.cpp` is a
    program written against it)."""
    import re

    ref_h = os.path.join(ROOT, "baseline", "_ref", "include", "agent", "agent.h")
    if not os.path.exists(ref_h):
        pytest.skip("reference build not present (python baseline/build_reference.py)")
    with open(ref_h) as f:
        ref = f.read()
    with open(os.path.join(ROOT, "csrc", "include", "ofld", "offload_agent.h")) as f:
        ours = f.read()
    body = ref[ref.index("class OffloadAgent"):]
    body = body[:body.index("\n};")]
    public = body.split("private:")[0]
    methods = set(re.findall(r"^\s+(?:[\w:<>,]+\s+)+?[&*]?(\w+)\s*\(", public, flags=re.M))
    methods -= {"OffloadAgent", "operator"}
    assert {"evict", "restore", "canonical_evict", "canonical_restore", "discard"} <= methods
    missing = sorted(m for m in methods if not re.search(rf"\b{m}\s*\(", ours))
    assert not missing, missing
    structs = set(re.findall(r"^struct\s+(\w+)", ref, flags=re.M))
    assert structs
    missing = sorted(s for s in structs if not re.search(rf"\b{s}\b", ours))
    assert not missing, missing
