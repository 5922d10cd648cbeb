"""The native self-test binary (codec, framing, config, layout, ring, hash, zbf16)."""

import os
import subprocess

from statespectre_b200._build import PKG


def test_ofld_selftest_passes():
    exe = os.path.join(PKG, "bin", "ofld_selftest")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert " 0 failed" in r.stdout
