import os
import sys
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")
    config.addinivalue_line("markers", "multigpu: needs 2 or more GPUs")
    config.addinivalue_line("markers", "slow: long-running")
    from statespectre_b200 import _build

    if not _build.built():
        _build.build()


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA GPU")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture
def sock_path():
    d = tempfile.mkdtemp(prefix="ofld-test-")
    return os.path.join(d, "offloadd.sock")


@pytest.fixture
def daemon(sock_path):
    """In-process daemon with a small arena, data kept pinned (no drain)."""
    from statespectre_b200 import in_process_daemon

    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=False)
    yield d
    d.stop()


@pytest.fixture
def host_session(daemon, sock_path):
    from statespectre_b200 import offload_context

    s = offload_context(daemon_addr=sock_path, device="cpu", rank=0)
    yield s.off
    s.close()


@pytest.fixture(autouse=True)
def _seeded():
    """Every test starts from the same torch RNG state (reproducible data)."""
    import torch

    torch.manual_seed(0)
    yield
