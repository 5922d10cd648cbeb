/* Minimal liburing-compatible interface for building StateSpectre (the
 * reference implementation) on hosts without liburing.
 *
 * Declares only what StateSpectre's src/daemon/daemon.cpp:2070-2242 calls:
 * one submission/completion ring pair, readv/writev preparation, user data,
 * submit, blocking wait and completion retirement. The ring lives in the
 * caller's struct io_uring; uring_shim.c drives it with the raw
 * io_uring_setup / io_uring_enter system calls. A build aid for the same-box
 * comparison, not part of the statespectre_b200 runtime. */
#ifndef OFLD_SHIM_LIBURING_H
#define OFLD_SHIM_LIBURING_H

#include <linux/io_uring.h>
#include <stdint.h>
#include <string.h>
#include <sys/uio.h>

#ifdef __cplusplus
extern "C" {
#endif

struct io_uring {
    int fd;
    unsigned sq_entries, cq_entries;
    /* submission ring (kernel-shared words) */
    unsigned *sq_head, *sq_tail, *sq_mask, *sq_array;
    struct io_uring_sqe *sqes;
    unsigned sqe_head, sqe_tail; /* handed out to the caller / not yet published */
    /* completion ring */
    unsigned *cq_head, *cq_tail, *cq_mask;
    struct io_uring_cqe *cqes;
    /* mappings */
    void *sq_map, *cq_map;
    size_t sq_map_len, cq_map_len, sqes_len;
};

/* 0 on success, -errno on failure. */
int io_uring_queue_init(unsigned entries, struct io_uring *ring, unsigned flags);
void io_uring_queue_exit(struct io_uring *ring);
/* NULL when every submission entry is in use. */
struct io_uring_sqe *io_uring_get_sqe(struct io_uring *ring);
/* Number of entries submitted, or -errno. */
int io_uring_submit(struct io_uring *ring);
/* 0 with *cqe_ptr set to the oldest completion (waiting for one), or -errno. */
int io_uring_wait_cqe(struct io_uring *ring, struct io_uring_cqe **cqe_ptr);
void io_uring_cqe_seen(struct io_uring *ring, struct io_uring_cqe *cqe);

static inline void io_uring_shim_prep_rw(int op, struct io_uring_sqe *sqe, int fd, const void *addr, unsigned len,
                                         uint64_t offset) {
    memset(sqe, 0, sizeof(*sqe));
    sqe->opcode = (uint8_t)op;
    sqe->fd = fd;
    sqe->off = offset;
    sqe->addr = (uint64_t)(uintptr_t)addr;
    sqe->len = len;
}

static inline void io_uring_prep_writev(struct io_uring_sqe *sqe, int fd, const struct iovec *iovecs,
                                        unsigned nr_vecs, uint64_t offset) {
    io_uring_shim_prep_rw(IORING_OP_WRITEV, sqe, fd, iovecs, nr_vecs, offset);
}

static inline void io_uring_prep_readv(struct io_uring_sqe *sqe, int fd, const struct iovec *iovecs,
                                       unsigned nr_vecs, uint64_t offset) {
    io_uring_shim_prep_rw(IORING_OP_READV, sqe, fd, iovecs, nr_vecs, offset);
}

static inline void io_uring_sqe_set_data(struct io_uring_sqe *sqe, void *data) {
    sqe->user_data = (uint64_t)(uintptr_t)data;
}

static inline void *io_uring_cqe_get_data(const struct io_uring_cqe *cqe) {
    return (void *)(uintptr_t)cqe->user_data;
}

#ifdef __cplusplus
}
#endif

#endif
