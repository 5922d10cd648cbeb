"""Wire interoperability with the reference's own client code.

StateSpectre's rollout wire module and RolloutWeightClient are pure Python
(python_api/state_spectre/_wire.py, _rollout.py). This test loads those two
files from the reference build in ``baseline/_ref`` (built by
baseline/build_reference.py; skipped when absent) under a private package
name, points them at this repository's offloadd over TCP, and pulls a sealed
version: discovery, manifest, per-object PullTensor with the daemon
connecting back, OFEX framing. Every pulled byte must equal the evicted
tensor, and the next version's manifest, carried forward here for its
unchanged objects, must show their content hashes unchanged when decoded by
the reference's codec.
"""

import importlib.util
import os
import socket
import sys
import types

import pytest
import torch

from statespectre_b200 import ModelRole, in_process_daemon, offload_context

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_PKG = os.environ.get("OFLD_REFERENCE_PY", os.path.join(ROOT, "baseline", "_ref", "state_spectre"))
ROLL = ModelRole.POLICY_ROLLOUT


def _load_reference_client():
    wire_py, rollout_py = os.path.join(REF_PKG, "_wire.py"), os.path.join(REF_PKG, "_rollout.py")
    if not (os.path.exists(wire_py) and os.path.exists(rollout_py)):
        pytest.skip("reference build not present (python baseline/build_reference.py)")
    name = "_ssref_pure"
    pkg = types.ModuleType(name)
    pkg.__path__ = [REF_PKG]
    # the reference's ModelRole lives in its torch-extension __init__; the
    # client only calls ModelRole.parse, whose values are the wire enum
    pkg.ModelRole = ModelRole
    sys.modules[name] = pkg
    mods = {}
    for sub, path in (("_wire", wire_py), ("_rollout", rollout_py)):
        spec = importlib.util.spec_from_file_location(f"{name}.{sub}", path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[f"{name}.{sub}"] = mod
        spec.loader.exec_module(mod)
        setattr(pkg, sub, mod)
        mods[sub] = mod
    return mods["_rollout"].RolloutWeightClient, mods["_wire"]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_reference_rollout_client_pulls_from_this_daemon(sock_path):
    RefClient, ref_wire = _load_reference_client()
    port = _free_port()
    d = in_process_daemon(socket=sock_path, arena_mb=128, drain_on_complete=False, tcp_port=port)
    try:
        tensors = {f"model.layers.{i}.mlp.w": torch.randn(257 + 31 * i, 65) for i in range(4)}
        tensors["model.norm.weight"] = torch.randn(17)
        with offload_context(daemon_addr=sock_path, device="cpu", rank=0, job_name="interop") as off:
            for name, t in tensors.items():
                off.canonical_evict(t.clone(), off.canonical_key(model_role=ROLL, model_version=1, param_name=name,
                                                                 tensor=t))
            off.promote_rollout_version(1)
            c = RefClient(f"tcp://127.0.0.1:{port}", off.job_id, off.launch_epoch, recv_host="127.0.0.1")
            assert c.get_latest_sealed_version() == 1
            man = c.get_manifest(1)
            assert len(man["tensors"]) == len(tensors)
            for e in man["tensors"]:
                payload = c.pull_tensor(e, 1)
                assert payload == tensors[e["key"]["param_fqn_debug"]].numpy().tobytes()
            # version 2: one tensor changes, the rest is carried forward with its content hash
            changed = "model.layers.2.mlp.w"
            tensors[changed] = tensors[changed] + 1
            k = off.canonical_key(model_role=ROLL, model_version=2, param_name=changed, tensor=tensors[changed])
            off.canonical_evict(tensors[changed].clone(), k)
            off.carry_forward_version(ROLL, 1, 2, [off.canonical_key(model_role=ROLL, model_version=2,
                                                                      param_name=n, tensor=t).param_id
                                                   for n, t in tensors.items() if n != changed])
            off.promote_rollout_version(2)
            res = c.sync_latest()
            assert res["version"] == 2
            # the reference client caches by object id, and version 2's
            # objects are new ids: it pulls all of them again
            assert len(res["pulled"]) == len(tensors)
            # the manifest, decoded by the reference's codec, carries the
            # unchanged objects' content hashes unchanged
            man2 = c.get_manifest(2, {"tp": 0})
            assert man2["ok"] and man2["model_version"] == 2 and man2["state"] == 2
            h1 = {e["key"]["param_fqn_debug"]: (e["content_hash_lo"], e["content_hash_hi"]) for e in man["tensors"]}
            h2 = {e["key"]["param_fqn_debug"]: (e["content_hash_lo"], e["content_hash_hi"]) for e in man2["tensors"]}
            assert {n for n in h1 if h1[n] != h2[n]} == {changed}
            for e in man2["tensors"]:
                assert c.pull_tensor(e, 2) == tensors[e["key"]["param_fqn_debug"]].numpy().tobytes()
            assert ref_wire.EXPORT_HEADER_SIZE == 40
    finally:
        d.stop()


def test_this_agent_records_and_pulls_through_the_reference_daemon(tmp_path):
    """The other direction: a host-mode session of this repository against
    StateSpectre's own offloadd (baseline/_ref/bin/offloadd; skipped when not
    built). The session's start-up probe for forwarded agent options
    (opcode 48, which that daemon logs as unknown and leaves unanswered) gives
    up after its reply timeout; registration, the control region, canonical
    evicts, the seal and a TCP pull then work byte for byte."""
    import subprocess
    import time

    from statespectre_b200 import RolloutWeightClient

    binary = os.path.join(ROOT, "baseline", "_ref", "bin", "offloadd")
    if not os.path.exists(binary):
        pytest.skip("reference build not present (python baseline/build_reference.py)")
    sock = str(tmp_path / "d.sock")
    port = _free_port()
    cfg = tmp_path / "offloadd.yaml"
    cfg.write_text("\n".join([
        "daemon:", f"  socket_path: {sock}", f"  control_shm_name: /ofld_interop_{os.getpid()}",
        "  heartbeat_timeout_ms: 60000", "arenas:", "  allocation_granularity_mb: 2", "  per_numa:",
        "    - numa_node: 0", "      size_gb: 2", "      overflow_gb: 1", "      gpu_windows:",
        "        - gpu: 0", "          size_gb: 1",
        "drain_policy:", "  target_tier: pageable", "  drain_on_d2h_complete: false", "nvme:", "  enabled: false"])
        + "\n")
    log = open(tmp_path / "ref.log", "w")
    proc = subprocess.Popen([binary, "--config", str(cfg), "--socket", sock, "--tcp-port", str(port)],
                            stdout=log, stderr=log)
    try:
        deadline = time.time() + 30
        while not os.path.exists(sock) and time.time() < deadline and proc.poll() is None:
            time.sleep(0.05)
        assert os.path.exists(sock), (tmp_path / "ref.log").read_text()
        tensors = {f"layers.{i}.w": torch.randn(1000 + 77 * i, 33) for i in range(3)}
        t0 = time.time()
        with offload_context(daemon_addr=sock, device="cpu", rank=0, job_name="interop-rev") as off:
            assert time.time() - t0 < 20  # the options probe did not hang the session
            for n, t in tensors.items():
                h = off.canonical_evict(t.clone(), off.canonical_key(model_role=ROLL, model_version=1, param_name=n,
                                                                     tensor=t))
                assert h.action_name == "NEED_D2H_CREATE"
            assert off.promote_rollout_version(1)["tensor_count"] == len(tensors)
            cl = RolloutWeightClient(f"tcp://127.0.0.1:{port}", off.job_id, off.launch_epoch, recv_host="127.0.0.1")
            man = cl.get_manifest(1)
            for e in man["tensors"]:
                assert cl.pull_tensor(e, 1) == tensors[e["key"]["param_fqn_debug"]].numpy().tobytes()
            cl.close()
            # v1 tensors: the session speaks only StateSpectre's opcodes (batches
            # one call per item, discard by lease release)
            xs = [torch.randn(5000 + 17 * i) for i in range(4)]
            for x in xs:
                h = off.copy(x, wait=True)
                assert torch.equal(h.restore(), x)
                h.discard()
            hs = off.evict_batch(xs)
            outs = off.restore_batch(hs)
            assert all(torch.equal(o, x) for o, x in zip(outs, xs))
            off.discard_batch(hs)
            t1 = time.time()
            with pytest.raises(RuntimeError, match="v1-only"):
                off.carry_forward_version(ROLL, 1, 2, [1])
            assert time.time() - t1 < 5
    finally:
        proc.terminate()
        try:
            proc.wait(timeout=30)
        except subprocess.TimeoutExpired:
            proc.kill()
        log.close()


def test_offload_stat_prometheus_matches_the_reference_tool(tmp_path):
    """Dashboards built on StateSpectre's `offload-stat --prometheus` keep
    working: against StateSpectre's own daemon, every HELP and TYPE line and
    every sample the reference's tool prints, this repository's tool prints
    too (its per-job series, which need an opcode that daemon lacks, are left
    out within 2 s instead of hanging)."""
    import subprocess
    import time

    from statespectre_b200._native import bin_path

    ref_bin = os.path.join(ROOT, "baseline", "_ref", "bin")
    if not os.path.exists(os.path.join(ref_bin, "offload-stat")):
        pytest.skip("reference build not present (python baseline/build_reference.py)")
    sock = str(tmp_path / "d.sock")
    cfg = tmp_path / "offloadd.yaml"
    cfg.write_text("\n".join([
        "daemon:", f"  socket_path: {sock}", f"  control_shm_name: /ofld_stat_{os.getpid()}",
        "arenas:", "  allocation_granularity_mb: 2", "  per_numa:", "    - numa_node: 0", "      size_gb: 1",
        "      overflow_gb: 0", "      gpu_windows:", "        - gpu: 0", "          size_gb: 1",
        "nvme:", "  enabled: false"]) + "\n")
    log = open(tmp_path / "ref.log", "w")
    proc = subprocess.Popen([os.path.join(ref_bin, "offloadd"), "--config", str(cfg), "--socket", sock],
                            stdout=log, stderr=log)
    try:
        deadline = time.time() + 30
        while not os.path.exists(sock) and time.time() < deadline and proc.poll() is None:
            time.sleep(0.05)
        ref = subprocess.run([os.path.join(ref_bin, "offload-stat"), "--socket", sock, "--prometheus"],
                             capture_output=True, text=True, timeout=30, check=True).stdout.splitlines()
        ours = subprocess.run([bin_path("offload-stat"), "--socket", sock, "--prometheus"],
                              capture_output=True, text=True, timeout=30, check=True).stdout.splitlines()
        assert len(ref) > 100
        mine = set(ours)
        missing = [line for line in ref if line not in mine]
        assert not missing, missing[:10]
    finally:
        proc.terminate()
        try:
            proc.wait(timeout=30)
        except subprocess.TimeoutExpired:
            proc.kill()
        log.close()


BASE_CFG = """daemon:
  socket_path: SOCK
arenas:
  allocation_granularity_mb: 2
  per_numa:
    - numa_node: 0
      size_gb: 1
      overflow_gb: 0
      gpu_windows:
        - gpu: 0
          size_gb: 1
nvme:
  enabled: false
"""


@pytest.mark.parametrize("case,edit", [
    ("valid", lambda c: c),
    ("tab indentation", lambda c: c.replace("  socket_path", "\tsocket_path")),
    ("windows beyond the arena", lambda c: c.replace("          size_gb: 1", "          size_gb: 5")),
    ("unknown drain tier", lambda c: c + "drain_policy:\n  target_tier: floppy\n"),
    ("size that is not a number", lambda c: c.replace("      size_gb: 1\n      overflow", "      size_gb: lots\n"
                                                                                         "      overflow")),
    ("unknown section", lambda c: c + "bogus_section:\n  x: 1\n"),
    ("v2 sections", lambda c: c + "canonical_store:\n  dedup_default_mode: hash_verified\nmanifest:\n"
                                  "  retain_sealed_versions: 3\nquotas:\n  default:\n    max_pinned_bytes: 1GiB\n"),
])
def test_config_files_are_accepted_and_refused_alike(tmp_path, case, edit):
    """A config file StateSpectre's offloadd starts with, this offloadd starts
    with; one it refuses at start-up, this one refuses too."""
    import subprocess

    from statespectre_b200._native import bin_path

    ref = os.path.join(ROOT, "baseline", "_ref", "bin", "offloadd")
    if not os.path.exists(ref):
        pytest.skip("reference build not present (python baseline/build_reference.py)")
    outcome = []
    for i, binary in enumerate((ref, bin_path("offloadd"))):
        sock = str(tmp_path / f"d{i}.sock")
        cfg = tmp_path / f"c{i}.yaml"
        cfg.write_text(edit(BASE_CFG).replace("SOCK", sock))
        try:
            r = subprocess.run([binary, "--config", str(cfg), "--socket", sock], capture_output=True, text=True,
                               timeout=3)
            outcome.append(("exited", r.returncode))
        except subprocess.TimeoutExpired:
            outcome.append(("serving", None))
    assert outcome[0] == outcome[1], (case, outcome)
