"""Every module of the package imports on a CPU-only host, so syntax and
import-time errors show up without a GPU."""

import importlib
import pkgutil

import pytest

import statespectre_b200

MODULES = sorted(m.name for m in pkgutil.walk_packages(statespectre_b200.__path__, "statespectre_b200."))


@pytest.mark.parametrize("name", MODULES)
def test_module_imports(name):
    importlib.import_module(name)


def test_bench_entry_parses():
    import ast
    import pathlib

    root = pathlib.Path(__file__).resolve().parents[1]
    for f in ("bench.py", "__graft_entry__.py"):
        ast.parse((root / f).read_text(), filename=f)
