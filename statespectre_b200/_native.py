"""Loader of the native extension (``statespectre_b200._C``).

The extension is built in-tree (``python -m statespectre_b200._build``). A
missing extension is an error, never a silent Python fallback: every data
path of this package runs in native code.
"""

from __future__ import annotations

import importlib
import os

_mod = None


def native():
    global _mod
    if _mod is None:
        try:
            _mod = importlib.import_module("statespectre_b200._C")
        except ImportError as e:  # pragma: no cover - exercised only on unbuilt trees
            raise ImportError(
                "statespectre_b200 native extension is not built; run `python -m statespectre_b200._build` "
                f"({e})") from e
    return _mod


def bin_path(name: str) -> str:
    """Absolute path of a built executable (offloadd, offload-stat, ofld_selftest)."""
    p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "bin", name)
    if not os.path.exists(p):
        raise FileNotFoundError(f"{name} is not built; run `python -m statespectre_b200._build`")
    return p
