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


def test_packaging_metadata():
    """``pip install .`` metadata: name, version, both packages, native files as package data."""
    import pathlib
    import subprocess
    import sys

    root = pathlib.Path(__file__).resolve().parents[1]
    out = subprocess.run([sys.executable, "setup.py", "--name", "--version"], cwd=root, capture_output=True,
                         text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert out.stdout.split()[:2] == ["statespectre-b200", statespectre_b200.__version__]
    text = (root / "setup.py").read_text()
    assert '"_C*.so"' in text and '"bin/offloadd"' in text and "state_spectre" in text
