"""Packaging: ``pip install .`` (or ``pip install -e .``).

The native parts (the sm_100a kernels, the agent and the in-process daemon
extension, and the ``offloadd`` / ``offload-stat`` / self-test binaries) are
built by the repository's ninja build (``statespectre_b200/_build.py``: nvcc
with ``-gencode arch=compute_100a,code=sm_100a`` and g++) before the Python
packages are collected, and ship as package data next to them. The packages
are ``statespectre_b200`` and its import-compatible alias ``state_spectre``.
"""

import importlib.util
import os

from setuptools import Distribution, find_packages, setup
from setuptools.command.build_py import build_py

ROOT = os.path.dirname(os.path.abspath(__file__))


def _version() -> str:
    with open(os.path.join(ROOT, "statespectre_b200", "__init__.py")) as f:
        for line in f:
            if line.startswith("__version__"):
                return line.split("=")[1].strip().strip('"')
    return "0.0.0"


class BuildNative(build_py):
    """Runs the ninja build in the source tree, then copies the packages."""

    def run(self):
        # load _build.py by path: importing the package would load the extension
        spec = importlib.util.spec_from_file_location("_ssb_build", os.path.join(ROOT, "statespectre_b200", "_build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
        super().run()


class BinaryDistribution(Distribution):
    """The packages carry a compiled extension: a platform wheel."""

    def has_ext_modules(self):
        return True


setup(
    name="statespectre-b200",
    version=_version(),
    description="GPU tensor-offload and model-state runtime for NVIDIA B200 (sm_100a)",
    packages=find_packages(include=["statespectre_b200", "statespectre_b200.*", "state_spectre",
                                    "state_spectre.*"]),
    package_data={"statespectre_b200": ["_C*.so", "bin/offloadd", "bin/offload-stat", "bin/ofld_selftest"]},
    include_package_data=False,
    python_requires=">=3.10",
    install_requires=["torch", "numpy"],
    cmdclass={"build_py": BuildNative},
    distclass=BinaryDistribution,
    zip_safe=False,
)
