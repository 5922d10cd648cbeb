/* liburing subset over the raw io_uring system calls (see include/liburing.h). */
#define _GNU_SOURCE
#include <liburing.h>

#include <errno.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

static unsigned load_acquire(const unsigned *p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
static void store_release(unsigned *p, unsigned v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }

int io_uring_queue_init(unsigned entries, struct io_uring *ring, unsigned flags) {
    struct io_uring_params p;
    memset(&p, 0, sizeof(p));
    memset(ring, 0, sizeof(*ring));
    p.flags = flags;
    int fd = (int)syscall(__NR_io_uring_setup, entries, &p);
    if (fd < 0) return -errno;
    ring->fd = fd;
    ring->sq_entries = p.sq_entries;
    ring->cq_entries = p.cq_entries;
    ring->sq_map_len = p.sq_off.array + p.sq_entries * sizeof(unsigned);
    ring->cq_map_len = p.cq_off.cqes + p.cq_entries * sizeof(struct io_uring_cqe);
    int single = (p.features & IORING_FEAT_SINGLE_MMAP) != 0;
    if (single && ring->cq_map_len > ring->sq_map_len) ring->sq_map_len = ring->cq_map_len;
    ring->sq_map = mmap(NULL, ring->sq_map_len, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_POPULATE, fd,
                        IORING_OFF_SQ_RING);
    if (ring->sq_map == MAP_FAILED) goto fail;
    if (single) {
        ring->cq_map = ring->sq_map;
    } else {
        ring->cq_map = mmap(NULL, ring->cq_map_len, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_POPULATE, fd,
                            IORING_OFF_CQ_RING);
        if (ring->cq_map == MAP_FAILED) goto fail;
    }
    ring->sqes_len = p.sq_entries * sizeof(struct io_uring_sqe);
    ring->sqes = (struct io_uring_sqe *)mmap(NULL, ring->sqes_len, PROT_READ | PROT_WRITE,
                                             MAP_SHARED | MAP_POPULATE, fd, IORING_OFF_SQES);
    if (ring->sqes == MAP_FAILED) goto fail;
    {
        char *s = (char *)ring->sq_map, *c = (char *)ring->cq_map;
        ring->sq_head = (unsigned *)(s + p.sq_off.head);
        ring->sq_tail = (unsigned *)(s + p.sq_off.tail);
        ring->sq_mask = (unsigned *)(s + p.sq_off.ring_mask);
        ring->sq_array = (unsigned *)(s + p.sq_off.array);
        ring->cq_head = (unsigned *)(c + p.cq_off.head);
        ring->cq_tail = (unsigned *)(c + p.cq_off.tail);
        ring->cq_mask = (unsigned *)(c + p.cq_off.ring_mask);
        ring->cqes = (struct io_uring_cqe *)(c + p.cq_off.cqes);
    }
    ring->sqe_head = ring->sqe_tail = *ring->sq_tail;
    return 0;
fail: {
    int e = errno;
    io_uring_queue_exit(ring);
    return -e;
}
}

void io_uring_queue_exit(struct io_uring *ring) {
    if (ring->sqes && ring->sqes != MAP_FAILED) munmap(ring->sqes, ring->sqes_len);
    if (ring->cq_map && ring->cq_map != MAP_FAILED && ring->cq_map != ring->sq_map)
        munmap(ring->cq_map, ring->cq_map_len);
    if (ring->sq_map && ring->sq_map != MAP_FAILED) munmap(ring->sq_map, ring->sq_map_len);
    if (ring->fd > 0) close(ring->fd);
    memset(ring, 0, sizeof(*ring));
    ring->fd = -1;
}

struct io_uring_sqe *io_uring_get_sqe(struct io_uring *ring) {
    unsigned head = load_acquire(ring->sq_head);
    if (ring->sqe_tail - head >= ring->sq_entries) return NULL;
    struct io_uring_sqe *sqe = &ring->sqes[ring->sqe_tail & *ring->sq_mask];
    ring->sqe_tail++;
    return sqe;
}

int io_uring_submit(struct io_uring *ring) {
    unsigned tail = *ring->sq_tail;
    unsigned n = ring->sqe_tail - ring->sqe_head;
    for (unsigned i = 0; i < n; ++i) {
        ring->sq_array[tail & *ring->sq_mask] = ring->sqe_head & *ring->sq_mask;
        ++tail;
        ++ring->sqe_head;
    }
    store_release(ring->sq_tail, tail);
    /* also submit entries published earlier that the kernel has not consumed */
    unsigned pending = tail - load_acquire(ring->sq_head);
    if (pending == 0) return (int)n;
    for (;;) {
        long r = syscall(__NR_io_uring_enter, ring->fd, pending, 0u, 0u, NULL, 0);
        if (r >= 0) return (int)r;
        if (errno != EINTR) return -errno;
    }
}

int io_uring_wait_cqe(struct io_uring *ring, struct io_uring_cqe **cqe_ptr) {
    for (;;) {
        unsigned head = *ring->cq_head;
        if (head != load_acquire(ring->cq_tail)) {
            *cqe_ptr = &ring->cqes[head & *ring->cq_mask];
            return 0;
        }
        long r = syscall(__NR_io_uring_enter, ring->fd, 0u, 1u, IORING_ENTER_GETEVENTS, NULL, 0);
        if (r < 0 && errno != EINTR) return -errno;
    }
}

void io_uring_cqe_seen(struct io_uring *ring, struct io_uring_cqe *cqe) {
    (void)cqe;
    store_release(ring->cq_head, *ring->cq_head + 1);
}
