"""The libnuma / liburing shims that let the reference build on this image
(``baseline/shim``): a C program against the shim headers writes a file with
``io_uring_prep_writev`` through the ring, reads it back with ``readv``, and
checks the NUMA queries against sysfs."""

import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "baseline", "shim")

PROGRAM = r"""
#include <fcntl.h>
#include <liburing.h>
#include <numa.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

int main(int argc, char **argv) {
    if (numa_available() < 0) { printf("numa unavailable\n"); }
    printf("max_node %d\n", numa_max_node());
    struct bitmask *m = numa_allocate_cpumask();
    int any = 0;
    if (numa_node_to_cpus(0, m) == 0)
        for (int c = 0; c < numa_num_configured_cpus(); ++c) any |= numa_bitmask_isbitset(m, c);
    numa_free_cpumask(m);
    printf("node0_cpus %d\n", any);

    struct io_uring ring;
    int rc = io_uring_queue_init(8, &ring, 0);
    if (rc < 0) { printf("uring_unavailable %d\n", rc); return 0; }
    int fd = open(argv[1], O_RDWR | O_CREAT | O_TRUNC, 0600);
    enum { N = 6, B = 8192 };
    static char src[N][B], dst[N][B];
    struct iovec iw[N], ir[N];
    for (int i = 0; i < N; ++i) {
        for (int j = 0; j < B; ++j) src[i][j] = (char)(i * 31 + j * 7);
        iw[i].iov_base = src[i]; iw[i].iov_len = B;
        ir[i].iov_base = dst[i]; ir[i].iov_len = B;
    }
    /* writes: all N in flight, completions in any order */
    for (int i = 0; i < N; ++i) {
        struct io_uring_sqe *sqe = io_uring_get_sqe(&ring);
        if (!sqe) { printf("no sqe\n"); return 1; }
        io_uring_prep_writev(sqe, fd, &iw[i], 1, (unsigned long long)i * B);
        io_uring_sqe_set_data(sqe, (void *)(long)(i + 1));
    }
    if (io_uring_submit(&ring) != N) { printf("submit\n"); return 1; }
    int seen = 0;
    for (int i = 0; i < N; ++i) {
        struct io_uring_cqe *cqe;
        if (io_uring_wait_cqe(&ring, &cqe) < 0) { printf("wait\n"); return 1; }
        long ud = (long)io_uring_cqe_get_data(cqe);
        if (cqe->res != B || ud < 1 || ud > N) { printf("bad cqe %d %ld\n", cqe->res, ud); return 1; }
        seen |= 1 << (ud - 1);
        io_uring_cqe_seen(&ring, cqe);
    }
    if (seen != (1 << N) - 1) { printf("missing\n"); return 1; }
    /* reads: one at a time, more requests than ring entries over the loop */
    for (int round = 0; round < 3; ++round)
        for (int i = 0; i < N; ++i) {
            struct io_uring_sqe *sqe = io_uring_get_sqe(&ring);
            memset(dst[i], 0, B);
            io_uring_prep_readv(sqe, fd, &ir[i], 1, (unsigned long long)i * B);
            io_uring_sqe_set_data(sqe, (void *)(long)i);
            if (io_uring_submit(&ring) < 0) { printf("submit r\n"); return 1; }
            struct io_uring_cqe *cqe;
            if (io_uring_wait_cqe(&ring, &cqe) < 0 || cqe->res != B) { printf("read\n"); return 1; }
            io_uring_cqe_seen(&ring, cqe);
            if (memcmp(src[i], dst[i], B) != 0) { printf("mismatch %d\n", i); return 1; }
        }
    io_uring_queue_exit(&ring);
    close(fd);
    printf("uring_ok\n");
    return 0;
}
"""


def _sysfs_max_node():
    base = "/sys/devices/system/node"
    try:
        nodes = [int(d[4:]) for d in os.listdir(base) if d.startswith("node") and d[4:].isdigit()]
    except OSError:
        return 0
    return max(nodes) if nodes else 0


def test_shims_against_the_kernel(tmp_path):
    prog = tmp_path / "t.c"
    prog.write_text(PROGRAM)
    exe = tmp_path / "t"
    inc = os.path.join(SHIM, "include")
    r = subprocess.run(["gcc", "-O1", "-Wall", f"-I{inc}", str(prog), os.path.join(SHIM, "numa_shim.c"),
                        os.path.join(SHIM, "uring_shim.c"), "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe), str(tmp_path / "data.bin")], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    out = dict(line.split(" ", 1) for line in r.stdout.strip().splitlines() if " " in line)
    assert int(out["max_node"]) == _sysfs_max_node()
    assert out["node0_cpus"] == "1"
    if "uring_unavailable" in out:
        pytest.skip(f"io_uring_setup refused here ({out['uring_unavailable']})")
    assert r.stdout.strip().endswith("uring_ok")
