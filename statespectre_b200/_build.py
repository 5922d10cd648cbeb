"""Native build of statespectre_b200 (ninja, in-tree outputs).

Produces, next to the sources so they travel with the repository:
  statespectre_b200/_C<EXT_SUFFIX>   Python extension: agent, in-process daemon,
                                      sm_100a kernels, host hash oracle
  statespectre_b200/bin/offloadd      the node daemon
  statespectre_b200/bin/offload-stat  metrics CLI
  statespectre_b200/bin/ofld_selftest C++ unit tests (codec, config, layout, allocator)

and, on request (``build(sanitizers=True)`` or ``--sanitizers``), host-code
sanitizer builds of the daemon and the self-test: ``offloadd_asan`` /
``ofld_selftest_asan`` (AddressSanitizer + UndefinedBehaviorSanitizer) and
``offloadd_tsan`` (ThreadSanitizer). The daemon is CUDA-free, so these cover
its whole control plane.

CUDA sources compile with ``-gencode arch=compute_100a,code=sm_100a -lineinfo``.
Run ``python -m statespectre_b200._build`` (or ``__graft_entry__.build()``).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "statespectre_b200")
CSRC = os.path.join(ROOT, "csrc")
BUILD = os.path.join(ROOT, "_build")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")

COMMON = ["common/codec.cpp", "common/transport.cpp", "common/metrics.cpp", "common/numa.cpp"]
DAEMON = ["daemon/config.cpp", "daemon/daemon.cpp", "daemon/slots.cpp", "daemon/tiers.cpp",
          "daemon/nvme.cpp", "daemon/canonical.cpp", "daemon/rollout.cpp", "daemon/persist.cpp"]
AGENT = ["agent/agent.cpp"]
KERNELS = ["kernels/offload_kernels.cu", "kernels/weight_sync.cu", "kernels/hash_noalloc.cu"]
KERNEL_HOST = ["kernels/timing.cpp"]
FABRIC = ["fabric/fabric.cpp", "fabric/vmm.cpp"]
MODULE = ["python/module.cpp", "python/fabric_bind.cpp"]

ARCH = "-gencode arch=compute_100a,code=sm_100a"
SANITIZERS = {
    "asan": "-fsanitize=address,undefined -fno-sanitize-recover=undefined -fno-omit-frame-pointer -g -O1",
    "tsan": "-fsanitize=thread -g -O1",
}


def _ext_suffix() -> str:
    return sysconfig.get_config_var("EXT_SUFFIX") or ".so"


def _pybind_include() -> str:
    import pybind11  # noqa: PLC0415

    return pybind11.get_include()


def _exists(rel: str) -> bool:
    return os.path.exists(os.path.join(CSRC, rel))


def _obj(rel: str) -> str:
    return os.path.join(BUILD, rel.replace("/", "_").rsplit(".", 1)[0] + ".o")


def write_ninja() -> str:
    py_inc = sysconfig.get_paths()["include"]
    inc = f"-I{CSRC}/include -I{CSRC} -I{CUDA_HOME}/include"
    cxx = ("-std=c++17 -O3 -fPIC -Wall -Wextra -Wno-unused-parameter -Wno-stringop-overflow "
           "-fvisibility=hidden -D_GLIBCXX_USE_CXX11_ABI=1")
    nv = (f"{ARCH} -lineinfo -O3 -std=c++17 -Xcompiler -fPIC -Xcompiler -fvisibility=hidden "
          "--expt-relaxed-constexpr -D_GLIBCXX_USE_CXX11_ABI=1")
    lines = [
        "ninja_required_version = 1.5",
        f"cxxflags = {cxx} {inc}",
        f"pyflags = -I{py_inc} -I{_pybind_include()}",
        f"nvflags = {nv} {inc}",
        f"cudalib = -L{CUDA_HOME}/lib64 -lcudart_static -ldl -lrt -lpthread",
        "rule cxx",
        "  command = g++ $cxxflags $extra -MMD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = CXX $out",
        "rule nvcc",
        "  command = nvcc $nvflags $extra -MD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = NVCC $out",
        "rule link_exe",
        "  command = g++ -o $out $in $libs -pthread",
        "  description = LINK $out",
        "rule link_so",
        "  command = g++ -shared -o $out $in $libs -pthread -Wl,--exclude-libs,ALL",
        "  description = LINK $out",
        "rule nvlink_dev",
        f"  command = nvcc {ARCH} -dlink -Xcompiler -fPIC $in -o $out",
        "  description = DLINK $out",
    ]
    objs = {}
    for rel in COMMON + DAEMON + AGENT + FABRIC + KERNEL_HOST + ["daemon/main.cpp", "tools/offload_stat.cpp", "tests/selftest.cpp",
                                                                "tests/compat_agent.cpp"]:
        if not _exists(rel):
            continue
        o = _obj(rel)
        objs[rel] = o
        lines.append(f"build {o}: cxx {os.path.join(CSRC, rel)}")
    for rel in MODULE:
        if not _exists(rel):
            continue
        o = _obj(rel)
        objs[rel] = o
        lines.append(f"build {o}: cxx {os.path.join(CSRC, rel)}")
        lines.append("  extra = $pyflags")
    for rel in KERNELS:
        if not _exists(rel):
            continue
        o = _obj(rel)
        objs[rel] = o
        lines.append(f"build {o}: nvcc {os.path.join(CSRC, rel)}")

    def pick(lst):
        return " ".join(objs[r] for r in lst if r in objs)

    bindir = os.path.join(PKG, "bin")
    os.makedirs(bindir, exist_ok=True)
    lines.append(f"build {bindir}/offloadd: link_exe {objs['daemon/main.cpp']} {pick(DAEMON)} {pick(COMMON)}")
    lines.append("  libs = ")
    if "tools/offload_stat.cpp" in objs:
        lines.append(f"build {bindir}/offload-stat: link_exe {objs['tools/offload_stat.cpp']} {pick(COMMON)}")
        lines.append("  libs = ")
    if "tests/selftest.cpp" in objs:
        lines.append(f"build {bindir}/ofld_selftest: link_exe {objs['tests/selftest.cpp']} {pick(DAEMON)} {pick(COMMON)}")
        lines.append("  libs = ")
    defaults = [f"{bindir}/offloadd"] + [f"{bindir}/{t}" for t in ("offload-stat", "ofld_selftest")
                                           if f"build {bindir}/{t}:" in "\n".join(lines)]
    # sanitizer variants of the CUDA-free host programs (built only when named)
    for tag, flags in SANITIZERS.items():
        lines.append(f"rule cxx_{tag}")
        lines.append(f"  command = g++ $cxxflags {flags} -MMD -MF $out.d -c $in -o $out")
        lines.append("  depfile = $out.d")
        lines.append("  deps = gcc")
        lines.append(f"  description = CXX[{tag}] $out")
        lines.append(f"rule link_{tag}")
        lines.append(f"  command = g++ {flags} -o $out $in -pthread")
        lines.append(f"  description = LINK[{tag}] $out")
        sobj = {}
        for rel in COMMON + DAEMON + ["daemon/main.cpp", "tests/selftest.cpp"]:
            if not _exists(rel):
                continue
            o = os.path.join(BUILD, tag, rel.replace("/", "_").rsplit(".", 1)[0] + ".o")
            sobj[rel] = o
            lines.append(f"build {o}: cxx_{tag} {os.path.join(CSRC, rel)}")
        core = " ".join(sobj[r] for r in COMMON + DAEMON if r in sobj)
        lines.append(f"build {bindir}/offloadd_{tag}: link_{tag} {sobj['daemon/main.cpp']} {core}")
        if tag == "asan" and "tests/selftest.cpp" in sobj:
            lines.append(f"build {bindir}/ofld_selftest_{tag}: link_{tag} {sobj['tests/selftest.cpp']} {core}")
    kern = pick(KERNELS)
    dlink = os.path.join(BUILD, "kernels_dlink.o")
    lines.append(f"build {dlink}: nvlink_dev {kern}")
    ext = os.path.join(PKG, "_C" + _ext_suffix())
    lines.append(f"build {ext}: link_so {pick(MODULE)} {pick(AGENT)} {pick(FABRIC)} {pick(DAEMON)} "
                 f"{pick(COMMON)} {pick(KERNEL_HOST)} {kern} {dlink}")
    lines.append("  libs = $cudalib")
    if "tests/compat_agent.cpp" in objs:  # StateSpectre's C++ agent interface, built against this agent
        compat = f"{bindir}/ofld_compat_agent"
        lines.append(f"build {compat}: link_exe {objs['tests/compat_agent.cpp']} {pick(AGENT)} {pick(FABRIC)} "
                     f"{pick(COMMON)} {pick(KERNEL_HOST)} {kern} {dlink}")
        lines.append("  libs = $cudalib")
        defaults.append(compat)
    lines.append("default " + " ".join(defaults + [ext]))
    os.makedirs(BUILD, exist_ok=True)
    path = os.path.join(BUILD, "build.ninja")
    with open(path, "w") as f:
        f.write("\n".join(lines) + "\n")
    return path


def sanitizer_targets() -> list:
    bindir = os.path.join(PKG, "bin")
    return [os.path.join(bindir, t) for t in ("offloadd_asan", "ofld_selftest_asan", "offloadd_tsan")]


def build(verbose: bool = False, jobs: int | None = None, sanitizers: bool = False) -> None:
    """Compile every native target in-tree (plus the sanitizer builds with
    ``sanitizers``). Raises CalledProcessError on failure."""
    if shutil.which("nvcc") is None and os.path.exists(os.path.join(CUDA_HOME, "bin", "nvcc")):
        os.environ["PATH"] = os.path.join(CUDA_HOME, "bin") + os.pathsep + os.environ.get("PATH", "")
    path = write_ninja()
    cmd = ["ninja", "-f", path]
    if jobs:
        cmd += ["-j", str(jobs)]
    if verbose:
        cmd.append("-v")
    subprocess.run(cmd, check=True, cwd=ROOT)
    if sanitizers:
        subprocess.run(cmd + sanitizer_targets(), check=True, cwd=ROOT)


def built() -> bool:
    return os.path.exists(os.path.join(PKG, "_C" + _ext_suffix())) and \
        os.path.exists(os.path.join(PKG, "bin", "offloadd"))


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, sanitizers="--sanitizers" in sys.argv)
