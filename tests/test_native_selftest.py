"""The native self-test binary (codec, framing, config, layout, ring, hash, zbf16)."""

import os
import subprocess

from statespectre_b200._build import PKG


def test_ofld_selftest_passes():
    exe = os.path.join(PKG, "bin", "ofld_selftest")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert " 0 failed" in r.stdout


def test_statespectre_cpp_agent_interface(tmp_path):
    """A program written against offload::OffloadAgent (StateSpectre's C++
    agent API) builds against this runtime and passes against a live daemon."""
    import subprocess

    from statespectre_b200 import launch_daemon
    from statespectre_b200._native import bin_path

    sock = str(tmp_path / "d.sock")
    with launch_daemon(sock, arena_mb=64, drain_on_complete=False):
        r = subprocess.run([bin_path("ofld_compat_agent"), sock], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "compat agent: ok" in r.stdout
