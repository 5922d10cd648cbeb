"""Build the unmodified StateSpectre reference into ``baseline/_ref`` for the
same-box comparison arm of ``bench.py --impl reference``.

StateSpectre needs libnuma and liburing at build time (its CMakeLists.txt:36-37
``find_library(... REQUIRED)``, and ``libraries=[..., "numa", ...]`` in
python_api/setup.py:55). Hosts without them get the small static shims in
``baseline/shim`` (sysfs + raw syscalls, only the calls StateSpectre makes).
Nothing in the reference's source is changed: the shims are passed in as
include and library paths.

Steps (each logged to ``baseline/_ref/build.log``):
  1. compile ``baseline/shim/*.c`` into ``_ref/shim/lib/lib{numa,uring}.a`` (-fPIC);
  2. copy the reference tree to a scratch directory (its Python build writes
     into the source tree, and the original is read-only);
  3. CMake-configure that copy with NUMA_LIB / URING_LIB pointing at the shims
     and build ``offloadd``, ``offload_stat`` and ``offload_bench`` into ``_ref/bin``;
  4. ``pip install --no-index --no-build-isolation --target baseline/_ref`` of
     the copy's ``python_api`` (its own setup.py and torch CppExtension), with
     CFLAGS/LDFLAGS naming the shims.

Run: ``python baseline/build_reference.py [--src <reference tree>]``.
The result is git-ignored; it is rebuilt on demand by bench.py when missing.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
SHIM = os.path.join(HERE, "shim")
DEFAULT_SRC = "/root/reference"


def _run(cmd, log, env=None, cwd=None):
    log.write("$ " + " ".join(cmd) + "\n")
    log.flush()
    r = subprocess.run(cmd, stdout=log, stderr=subprocess.STDOUT, env=env, cwd=cwd)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}; see {log.name}")


def build_shims(log) -> str:
    lib = os.path.join(OUT, "shim", "lib")
    os.makedirs(lib, exist_ok=True)
    inc = os.path.join(SHIM, "include")
    for name, src in (("numa", "numa_shim.c"), ("uring", "uring_shim.c")):
        obj = os.path.join(lib, name + ".o")
        _run(["gcc", "-O2", "-fPIC", "-Wall", f"-I{inc}", "-c", os.path.join(SHIM, src), "-o", obj], log)
        ar = os.path.join(lib, f"lib{name}.a")
        if os.path.exists(ar):
            os.unlink(ar)
        _run(["ar", "rcs", ar, obj], log)
    return lib


def build(src: str = DEFAULT_SRC, jobs: int = 0) -> dict:
    if not os.path.isdir(src):
        raise RuntimeError(f"reference tree not found at {src}")
    os.makedirs(OUT, exist_ok=True)
    log_path = os.path.join(OUT, "build.log")
    with open(log_path, "w") as log:
        lib = build_shims(log)
        inc = os.path.join(SHIM, "include")
        scratch = tempfile.mkdtemp(prefix="ssref-")
        tree = os.path.join(scratch, "src")
        shutil.copytree(src, tree, symlinks=True)
        bdir = os.path.join(scratch, "build")
        cmake = shutil.which("cmake") or os.path.join(os.path.dirname(sys.executable), "cmake")
        _run([cmake, "-S", tree, "-B", bdir, "-DCMAKE_BUILD_TYPE=Release",
              f"-DNUMA_LIB={lib}/libnuma.a", f"-DURING_LIB={lib}/liburing.a",
              f"-DCMAKE_CXX_FLAGS=-I{inc}"], log)
        j = str(jobs or os.cpu_count() or 4)
        _run([cmake, "--build", bdir, "-j", j, "--target", "offloadd", "offload_stat", "offload_bench"], log)
        bindir = os.path.join(OUT, "bin")
        os.makedirs(bindir, exist_ok=True)
        for exe in ("offloadd", "offload-stat", "offload_bench"):
            shutil.copy2(os.path.join(bdir, exe), os.path.join(bindir, exe))
        # the reference's C++ agent interface, read as text by the API parity test
        incdir = os.path.join(OUT, "include", "agent")
        os.makedirs(incdir, exist_ok=True)
        shutil.copy2(os.path.join(tree, "src", "agent", "agent.h"), os.path.join(incdir, "agent.h"))
        env = dict(os.environ)
        env["CFLAGS"] = (env.get("CFLAGS", "") + f" -I{inc}").strip()
        env["CPPFLAGS"] = (env.get("CPPFLAGS", "") + f" -I{inc}").strip()
        env["LDFLAGS"] = (env.get("LDFLAGS", "") + f" -L{lib}").strip()
        env["MAX_JOBS"] = j
        _run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
              "--find-links", "/opt/wheelhouse", "--upgrade", "--target", OUT, os.path.join(tree, "python_api")],
             log, env=env)
        shutil.rmtree(scratch, ignore_errors=True)
    ext = [f for f in os.listdir(os.path.join(OUT, "state_spectre")) if f.startswith("_state_spectre")]
    return {"out": OUT, "bin": os.path.join(OUT, "bin"), "extension": ext, "log": log_path,
            "python": sysconfig.get_python_version()}


def built() -> bool:
    pkg = os.path.join(OUT, "state_spectre")
    return (os.path.exists(os.path.join(OUT, "bin", "offloadd")) and os.path.isdir(pkg)
            and any(f.startswith("_state_spectre") and f.endswith(".so") for f in os.listdir(pkg)))


def main() -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--src", default=DEFAULT_SRC)
    p.add_argument("--jobs", type=int, default=0)
    a = p.parse_args()
    print(build(a.src, a.jobs))
    return 0


if __name__ == "__main__":
    sys.exit(main())
