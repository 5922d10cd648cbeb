// NVMe cold tier: objects striped over `stripe_count` files (one directory per
// drive via nvme.stripe_dirs), written and read in block_mb blocks through
// either io_uring (raw io_uring_setup/io_uring_enter syscalls; this image has
// no liburing) with queue_depth blocks in flight, or a pool of nvme.workers
// threads issuing pwrite/pread. O_DIRECT is used when configured and falls back
// to buffered IO on filesystems that refuse it (tmpfs). Reclaimed extents are
// returned to the filesystem with FALLOC_FL_PUNCH_HOLE.
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include <errno.h>
#include <fcntl.h>
#include <linux/falloc.h>
#include <linux/io_uring.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "daemon.h"
#include "ofld/log.h"
#include "ofld/metrics.h"

namespace ofld {

namespace {
constexpr const char* TAG = "nvme";
constexpr uint64_t kAlign = 4096;

void mkdir_p(const std::string& path) {
    std::string cur;
    for (size_t i = 0; i <= path.size(); ++i) {
        if (i == path.size() || path[i] == '/') {
            if (!cur.empty() && ::mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST)
                LOG_WARN(TAG, "mkdir %s: %s", cur.c_str(), std::strerror(errno));
        }
        if (i < path.size()) cur.push_back(path[i]);
    }
}

int open_file(const std::string& path, bool write, bool direct) {
    int flags = (write ? (O_WRONLY | O_CREAT) : O_RDONLY) | O_CLOEXEC;
    int fd = direct ? ::open(path.c_str(), flags | O_DIRECT, 0644) : -1;
    if (fd < 0) fd = ::open(path.c_str(), flags, 0644);  // filesystem without O_DIRECT
    return fd;
}

// One block transfer through an aligned bounce buffer.
struct Block {
    int fd;
    uint64_t file_off;  // aligned
    uint64_t io_len;    // aligned length submitted to the kernel
    char* mem;          // caller memory
    uint64_t skip;      // bytes of the bounce to skip before copying (reads)
    uint64_t len;       // bytes copied between bounce and caller memory
};

void* alloc_aligned(uint64_t n) {
    void* p = nullptr;
    return posix_memalign(&p, kAlign, round_up(n, kAlign)) == 0 ? p : nullptr;
}

// Minimal io_uring over raw syscalls: one SQ/CQ pair, READ/WRITE opcodes.
class Uring {
 public:
    bool init(unsigned depth) {
        io_uring_params p{};
        fd_ = int(::syscall(__NR_io_uring_setup, depth, &p));
        if (fd_ < 0) return false;
        sq_sz_ = p.sq_off.array + p.sq_entries * sizeof(unsigned);
        cq_sz_ = p.cq_off.cqes + p.cq_entries * sizeof(io_uring_cqe);
        single_ = (p.features & IORING_FEAT_SINGLE_MMAP) != 0;
        if (single_) sq_sz_ = cq_sz_ = std::max(sq_sz_, cq_sz_);
        sq_ = ::mmap(nullptr, sq_sz_, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_POPULATE, fd_, IORING_OFF_SQ_RING);
        if (sq_ == MAP_FAILED) return fail();
        cq_ = single_ ? sq_
                      : ::mmap(nullptr, cq_sz_, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_POPULATE, fd_,
                               IORING_OFF_CQ_RING);
        if (cq_ == MAP_FAILED) return fail();
        sqes_sz_ = p.sq_entries * sizeof(io_uring_sqe);
        sqes_ = static_cast<io_uring_sqe*>(
            ::mmap(nullptr, sqes_sz_, PROT_READ | PROT_WRITE, MAP_SHARED | MAP_POPULATE, fd_, IORING_OFF_SQES));
        if (sqes_ == MAP_FAILED) return fail();
        char* s = static_cast<char*>(sq_);
        char* c = static_cast<char*>(cq_);
        sq_head_ = reinterpret_cast<unsigned*>(s + p.sq_off.head);
        sq_tail_ = reinterpret_cast<unsigned*>(s + p.sq_off.tail);
        sq_mask_ = *reinterpret_cast<unsigned*>(s + p.sq_off.ring_mask);
        sq_array_ = reinterpret_cast<unsigned*>(s + p.sq_off.array);
        cq_head_ = reinterpret_cast<unsigned*>(c + p.cq_off.head);
        cq_tail_ = reinterpret_cast<unsigned*>(c + p.cq_off.tail);
        cq_mask_ = *reinterpret_cast<unsigned*>(c + p.cq_off.ring_mask);
        cqes_ = reinterpret_cast<io_uring_cqe*>(c + p.cq_off.cqes);
        entries_ = p.sq_entries;
        return true;
    }
    ~Uring() {
        if (sqes_ && sqes_ != MAP_FAILED) ::munmap(sqes_, sqes_sz_);
        if (cq_ && cq_ != MAP_FAILED && !single_) ::munmap(cq_, cq_sz_);
        if (sq_ && sq_ != MAP_FAILED) ::munmap(sq_, sq_sz_);
        if (fd_ >= 0) ::close(fd_);
    }
    unsigned entries() const { return entries_; }
    void queue(bool write, int fd, void* buf, unsigned len, uint64_t off, uint64_t tag) {
        unsigned tail = __atomic_load_n(sq_tail_, __ATOMIC_RELAXED);
        unsigned idx = tail & sq_mask_;
        io_uring_sqe& e = sqes_[idx];
        std::memset(&e, 0, sizeof(e));
        e.opcode = write ? IORING_OP_WRITE : IORING_OP_READ;
        e.fd = fd;
        e.addr = reinterpret_cast<uint64_t>(buf);
        e.len = len;
        e.off = off;
        e.user_data = tag;
        sq_array_[idx] = idx;
        __atomic_store_n(sq_tail_, tail + 1, __ATOMIC_RELEASE);
        ++pending_;
    }
    // Submit queued SQEs and wait for at least one completion.
    bool submit_and_wait() {
        unsigned n = pending_;
        pending_ = 0;
        for (;;) {
            long r = ::syscall(__NR_io_uring_enter, fd_, n, 1u, IORING_ENTER_GETEVENTS, nullptr, 0);
            if (r >= 0) return true;
            if (errno != EINTR) return false;
            n = 0;
        }
    }
    bool pop(uint64_t* tag, int* res) {
        unsigned head = __atomic_load_n(cq_head_, __ATOMIC_RELAXED);
        if (head == __atomic_load_n(cq_tail_, __ATOMIC_ACQUIRE)) return false;
        const io_uring_cqe& c = cqes_[head & cq_mask_];
        *tag = c.user_data;
        *res = c.res;
        __atomic_store_n(cq_head_, head + 1, __ATOMIC_RELEASE);
        return true;
    }

 private:
    bool fail() {
        if (fd_ >= 0) ::close(fd_);
        fd_ = -1;
        return false;
    }
    int fd_ = -1;
    void *sq_ = nullptr, *cq_ = nullptr;
    io_uring_sqe* sqes_ = nullptr;
    size_t sq_sz_ = 0, cq_sz_ = 0, sqes_sz_ = 0;
    bool single_ = false;
    unsigned *sq_head_ = nullptr, *sq_tail_ = nullptr, *sq_array_ = nullptr, sq_mask_ = 0;
    unsigned *cq_head_ = nullptr, *cq_tail_ = nullptr, cq_mask_ = 0;
    io_uring_cqe* cqes_ = nullptr;
    unsigned entries_ = 0, pending_ = 0;
};

bool run_uring(std::vector<Block>& blocks, bool write, unsigned qd, uint64_t max_io) {
    Uring ring;
    if (!ring.init(qd)) return false;
    qd = std::min(qd, ring.entries());
    std::vector<void*> pool(qd, nullptr);
    std::vector<uint32_t> free_bufs;
    for (unsigned i = 0; i < qd; ++i) {
        pool[i] = alloc_aligned(max_io);
        if (!pool[i]) {
            for (void* p : pool) std::free(p);
            return false;
        }
        free_bufs.push_back(i);
    }
    size_t next = 0, done = 0;
    unsigned inflight = 0;
    bool ok = true;
    while (done < blocks.size() && ok) {
        while (inflight < qd && next < blocks.size() && !free_bufs.empty()) {
            uint32_t b = free_bufs.back();
            free_bufs.pop_back();
            Block& blk = blocks[next];
            if (write) {
                std::memcpy(pool[b], blk.mem, blk.len);
                if (blk.io_len > blk.len) std::memset(static_cast<char*>(pool[b]) + blk.len, 0, blk.io_len - blk.len);
            }
            ring.queue(write, blk.fd, pool[b], unsigned(blk.io_len), blk.file_off, (uint64_t(next) << 16) | b);
            ++next;
            ++inflight;
        }
        if (!ring.submit_and_wait()) {
            ok = false;
            break;
        }
        uint64_t tag;
        int res;
        while (ring.pop(&tag, &res)) {
            uint32_t b = uint32_t(tag & 0xFFFF);
            Block& blk = blocks[tag >> 16];
            bool good = write ? (res >= 0 && uint64_t(res) == blk.io_len)
                              : (res >= 0 && uint64_t(res) >= blk.skip + blk.len);
            if (!good) {
                LOG_ERR(TAG, "io_uring %s res=%d want %llu", write ? "write" : "read", res,
                        (unsigned long long)blk.io_len);
                ok = false;
            } else if (!write) {
                std::memcpy(blk.mem, static_cast<char*>(pool[b]) + blk.skip, blk.len);
            }
            free_bufs.push_back(b);
            --inflight;
            ++done;
        }
    }
    // Drain completions still in flight before the buffers go away.
    while (inflight > 0) {
        if (!ring.submit_and_wait()) break;
        uint64_t tag;
        int res;
        while (ring.pop(&tag, &res)) --inflight;
    }
    for (void* p : pool) std::free(p);
    return ok;
}

bool run_threads(std::vector<Block>& blocks, bool write, unsigned workers, uint64_t max_io) {
    std::atomic<size_t> next{0};
    std::atomic<bool> ok{true};
    auto body = [&] {
        void* bounce = alloc_aligned(max_io);
        if (!bounce) {
            ok = false;
            return;
        }
        for (size_t i; ok.load() && (i = next.fetch_add(1)) < blocks.size();) {
            Block& b = blocks[i];
            char* buf = static_cast<char*>(bounce);
            if (write) {
                std::memcpy(buf, b.mem, b.len);
                if (b.io_len > b.len) std::memset(buf + b.len, 0, b.io_len - b.len);
            }
            uint64_t got = 0;
            while (got < b.io_len) {
                ssize_t r = write ? ::pwrite(b.fd, buf + got, b.io_len - got, off_t(b.file_off + got))
                                  : ::pread(b.fd, buf + got, b.io_len - got, off_t(b.file_off + got));
                if (r < 0 && errno == EINTR) continue;
                if (r < 0) {
                    LOG_ERR(TAG, "%s: %s", write ? "pwrite" : "pread", std::strerror(errno));
                    ok = false;
                    break;
                }
                if (r == 0) break;  // EOF inside the final padding
                got += uint64_t(r);
            }
            if (!ok.load()) break;
            if (write && got != b.io_len) ok = false;
            if (!write) {
                if (got < b.skip + b.len) {
                    ok = false;
                    break;
                }
                std::memcpy(b.mem, buf + b.skip, b.len);
            }
        }
        std::free(bounce);
    };
    workers = std::max(1u, std::min<unsigned>(workers, unsigned(blocks.size())));
    std::vector<std::thread> ts;
    for (unsigned i = 1; i < workers; ++i) ts.emplace_back(body);
    body();
    for (auto& t : ts) t.join();
    return ok.load();
}
}  // namespace

std::string Daemon::stripe_path(uint32_t stripe) const {
    const std::string& dir = cfg_.nvme_stripe_dirs.empty()
                                 ? cfg_.nvme_path
                                 : cfg_.nvme_stripe_dirs[stripe % cfg_.nvme_stripe_dirs.size()];
    return dir + "/off_stripe_" + std::to_string(stripe) + ".dat";
}

bool Daemon::nvme_write(const char* src, uint64_t nbytes, std::vector<Extent>* out) {
    const uint64_t block = round_up(std::max<uint64_t>(cfg_.nvme_block_bytes, kAlign), kAlign);
    std::vector<int> fds;
    std::vector<Block> blocks;
    uint64_t per = nbytes / stripes_, consumed = 0;
    bool ok = true;
    for (uint32_t i = 0; i < stripes_ && ok; ++i) {
        uint64_t seg = i + 1 == stripes_ ? nbytes - consumed : per;
        if (seg == 0 && !(i == 0 && nbytes == 0)) continue;
        std::string path = stripe_path(i);
        mkdir_p(path.substr(0, path.rfind('/')));
        int fd = open_file(path, true, cfg_.nvme_direct_io);
        if (fd < 0) {
            LOG_ERR(TAG, "open %s: %s", path.c_str(), std::strerror(errno));
            ok = false;
            break;
        }
        fds.push_back(fd);
        uint64_t base = stripe_cursor_[i].fetch_add(round_up(std::max<uint64_t>(seg, 1), kAlign));
        out->push_back(Extent{path, base, seg});
        for (uint64_t off = 0; off < seg; off += block) {
            uint64_t len = std::min(block, seg - off);
            blocks.push_back(Block{fd, base + off, round_up(len, kAlign), const_cast<char*>(src) + consumed + off, 0, len});
        }
        consumed += seg;
    }
    if (ok) {
        bool done = false;
        if (cfg_.nvme_io_engine == "io_uring")
            done = run_uring(blocks, true, std::max(1u, cfg_.nvme_queue_depth), block);
        if (!done) ok = run_threads(blocks, true, std::max(1u, cfg_.nvme_workers), block);
    }
    for (int fd : fds) ::close(fd);
    if (!ok) {
        nvme_release(*out);
        out->clear();
    }
    return ok;
}

bool Daemon::nvme_read(const std::vector<Extent>& ext, char* dst, uint64_t off, uint64_t nbytes) {
    const uint64_t block = round_up(std::max<uint64_t>(cfg_.nvme_block_bytes, kAlign), kAlign);
    std::vector<int> fds;
    std::vector<Block> blocks;
    uint64_t logical = 0;  // logical start of the current extent
    bool ok = true;
    for (const Extent& e : ext) {
        uint64_t lo = std::max(off, logical), hi = std::min(off + nbytes, logical + e.length);
        if (lo < hi) {
            int fd = open_file(e.path, false, cfg_.nvme_direct_io);
            if (fd < 0) {
                LOG_ERR(TAG, "open %s: %s", e.path.c_str(), std::strerror(errno));
                ok = false;
                break;
            }
            fds.push_back(fd);
            // File range [e.offset + (lo - logical), e.offset + (hi - logical)).
            for (uint64_t p = lo; p < hi;) {
                uint64_t file_pos = e.offset + (p - logical);
                uint64_t aligned = file_pos / kAlign * kAlign;
                uint64_t skip = file_pos - aligned;
                uint64_t len = std::min(hi - p, block - skip);
                blocks.push_back(Block{fd, aligned, round_up(skip + len, kAlign), dst + (p - off), skip, len});
                p += len;
            }
        }
        logical += e.length;
    }
    if (ok && logical < off + nbytes) ok = false;  // extents do not cover the range
    if (ok && !blocks.empty()) {
        bool done = false;
        if (cfg_.nvme_io_engine == "io_uring")
            done = run_uring(blocks, false, std::max(1u, cfg_.nvme_queue_depth), block);
        if (!done) ok = run_threads(blocks, false, std::max(1u, cfg_.nvme_workers), block);
    }
    for (int fd : fds) ::close(fd);
    return ok;
}

void Daemon::nvme_release(const std::vector<Extent>& ext) {
    for (const Extent& e : ext) {
        int fd = ::open(e.path.c_str(), O_WRONLY | O_CLOEXEC);
        if (fd < 0) continue;
        if (::fallocate(fd, FALLOC_FL_PUNCH_HOLE | FALLOC_FL_KEEP_SIZE, off_t(e.offset),
                        off_t(round_up(std::max<uint64_t>(e.length, 1), kAlign))) != 0)
            LOG_DEBUG(TAG, "punch hole %s: %s", e.path.c_str(), std::strerror(errno));
        ::close(fd);
    }
}

}  // namespace ofld
