"""The content hash against an independent implementation of its written
definition (tests/ssh128_numpy.py): the host implementation the daemon and
agent use on CPU, and (GPU) the sm_100a kernels that compute it in the
copy pass."""

import numpy as np
import pytest

from ssh128_numpy import chunk_digests, object_hash
from statespectre_b200._native import native

SIZES = [0, 1, 15, 16, 17, 4095, 4096, 65535, 65536, 65537, 3 * 65536 + 12345, (1 << 20) + 7]


@pytest.mark.parametrize("n", SIZES)
def test_host_implementation_matches_numpy_oracle(n):
    rng = np.random.default_rng(n)
    data = rng.integers(0, 256, n, dtype=np.uint8)
    assert native().ssh_digests(data) == chunk_digests(data.tobytes())
    assert native().ssh_hash(data) == object_hash(data.tobytes())


def test_structured_inputs():
    for data in (np.zeros(70000, np.uint8), np.full(65536 * 2, 0xFF, np.uint8),
                 np.arange(200000, dtype=np.uint32).view(np.uint8)):
        assert native().ssh_hash(data) == object_hash(data.tobytes())
    # one flipped bit changes exactly its chunk's digest
    a = np.random.default_rng(1).integers(0, 256, 5 * 65536, dtype=np.uint8)
    b = a.copy()
    b[2 * 65536 + 999] ^= 4
    da, db = chunk_digests(a.tobytes()), chunk_digests(b.tobytes())
    assert [i for i in range(5) if da[i] != db[i]] == [2]


@pytest.mark.gpu
@pytest.mark.parametrize("n", [17, 65536 * 4 + 48, (8 << 20) + 4096])
def test_kernels_match_numpy_oracle(n):
    import torch

    C = native()
    x = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    host = torch.empty(n + 16, dtype=torch.uint8, pin_memory=True)
    nd = (n + 65535) // 65536
    d1, d2 = (torch.zeros(nd, dtype=torch.int64, device="cuda") for _ in range(2))
    s = torch.cuda.current_stream().cuda_stream
    C.k_evict_hash(x.data_ptr(), host.data_ptr(), n, d1.data_ptr(), s, 0)  # K1: digests in the copy pass
    C.k_hash_device(x.data_ptr(), n, d2.data_ptr(), s, 0)
    torch.cuda.synchronize()
    want = chunk_digests(x.cpu().numpy().tobytes())
    for d in (d1, d2):
        assert [int(v) & 0xFFFFFFFFFFFFFFFF for v in d.cpu().tolist()] == want
