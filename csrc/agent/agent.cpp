// Rank agent implementation. See agent.h.
//
// Transfer protocol per evict (StateSpectre order, reference:
// src/agent/agent.cpp:753-868): reserve a run (RequestOffload), mark it
// submitted, launch the copy, record an event, and on completion report
// D2H-complete (completion ring, else RPC) and run the invalidate callback.
// With fast_submit the reservation and the submitted mark travel in one
// round trip (OFLD_FLAG_SUBMIT_ON_GRANT); restore likewise folds
// MarkH2DSubmitted into the ready prefetch (OFLD_FLAG_SUBMIT_ON_READY).
#include "agent.h"

#include <cuda_runtime.h>
#include <sys/mman.h>
#include <unistd.h>

#include <atomic>
#include <condition_variable>
#include <cstring>
#include <list>
#include <map>
#include <mutex>
#include <stdexcept>
#include <thread>
#include <unordered_map>

#include "../kernels/kernels.h"
#include "../kernels/timing.h"

#include <nvtx3/nvToolsExt.h>
#include "ofld/abi/offload_canonical_abi.hpp"
#include "ofld/chunk_hash.h"
#include "ofld/zbf16.h"
#include "ofld/log.h"
#include "ofld/metrics.h"
#include "ofld/numa.h"
#include "ofld/shm.h"
#include "ofld/transport.h"

namespace ofld {

namespace {
// NVTX range over an agent call (nsys/ncu timelines); no cost without a tool.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
};
}  // namespace

namespace {
constexpr const char* TAG = "agent";

#define CUDA_OK(expr)                                                                                 \
    do {                                                                                              \
        cudaError_t e_ = (expr);                                                                      \
        if (e_ != cudaSuccess)                                                                        \
            throw std::runtime_error(std::string("CUDA error at " #expr ": ") + cudaGetErrorString(e_)); \
    } while (0)

struct TvKey {
    uint64_t tid, ver;
    bool operator<(const TvKey& o) const { return tid != o.tid ? tid < o.tid : ver < o.ver; }
};

// Small host-mapped pinned buffers (chunk digests, mismatch counters) cached
// by power-of-two size class.
class PinnedPool {
 public:
    struct Buf {
        void* host = nullptr;
        void* dev = nullptr;
        size_t cls = 0;
    };
    Buf get(size_t bytes) {
        size_t cls = 64;
        while (cls < bytes) cls <<= 1;
        {
            std::lock_guard<std::mutex> g(mu_);
            auto& v = free_[cls];
            if (!v.empty()) {
                Buf b = v.back();
                v.pop_back();
                return b;
            }
        }
        Buf b;
        b.cls = cls;
        CUDA_OK(cudaHostAlloc(&b.host, cls, cudaHostAllocMapped | cudaHostAllocPortable));
        CUDA_OK(cudaHostGetDevicePointer(&b.dev, b.host, 0));
        return b;
    }
    void put(const Buf& b) {
        if (!b.host) return;
        std::lock_guard<std::mutex> g(mu_);
        free_[b.cls].push_back(b);
    }
    void clear() {
        std::lock_guard<std::mutex> g(mu_);
        for (auto& kv : free_)
            for (Buf& b : kv.second) cudaFreeHost(b.host);
        free_.clear();
    }

 private:
    std::mutex mu_;
    std::map<size_t, std::vector<Buf>> free_;
};

}  // namespace

struct Agent::Impl {
    AgentOptions opt;
    bool gpu = false;
    int numa = 0;
    uint64_t epoch = 0;
    std::unique_ptr<RpcClient> rpc;
    std::atomic<uint64_t> rpc_count{0};

    struct ArenaMap {
        uint64_t id = 0;
        char* base = nullptr;
        uint64_t size = 0;
        char* dev = nullptr;  // device alias after registration
        bool registered = false;
        std::vector<std::pair<char*, uint64_t>> pieces;  // registered ranges
    };
    std::vector<ArenaMap> arenas;
    std::mutex reg_mu;
    char* control = nullptr;
    uint64_t control_size = 0;
    ofld_slot_entry_t* slots = nullptr;
    uint32_t num_slots = 0;
    RingHeader* ring = nullptr;
    std::mutex ring_mu;

    cudaStream_t stream = nullptr;
    cudaStream_t side = nullptr;  // evict digests next to a copy-engine copy; coded restore copies
    cudaStream_t aux = nullptr;   // zf32: digests of the fp32 bytes next to the coding and its copies

    // Coded paths through the copy engine: a ring of device staging buffers
    // of zpiece chunks each (allocated on first use; default 2 x 32 MiB) and
    // their events.
    static constexpr int kZDepthMax = 8;
    uint64_t zpiece = 512;
    int zdepth = 2;
    void* zstage[kZDepthMax] = {};
    // zfull[b]: staging b holds a piece (recorded by its producer); zfree[b]:
    // nothing reads staging b any more (recorded by its consumer). Every
    // writer of b waits zfree[b], whichever operation used it last.
    cudaEvent_t zfull[kZDepthMax] = {}, zfree[kZDepthMax] = {};
    uint64_t zturn = 0;  // next staging buffer of the ring
    cudaEvent_t zstart = nullptr, zdone = nullptr;
    // Decodes run on their own stream at the device's highest priority: a
    // restore issues one short decode per piece, and at equal priority each
    // would queue behind the kernels of a concurrent training step.
    cudaStream_t zdec = nullptr;
    std::mutex zmu;  // coded evicts and restores of this session share the staging

    // Piece boundaries of a coded run: zpiece chunks each, except that a
    // short raw tail never sits alone (a piece must itself be a codable
    // object): the piece before it gives up one chunk.
    static uint64_t zpiece_end(uint64_t c0, uint64_t nch, bool short_tail, uint64_t zpiece) {
        uint64_t c1 = std::min(nch, c0 + zpiece);
        if (short_tail && nch - c1 == 1) c1 -= 1;  // pieces that leave one chunk are full, so > 1
        return c1;
    }

    // Coded evict through the copy engine: K1 codes a piece into staging (HBM,
    // digests from the same pass) on the top-priority stream while the copy
    // engine moves the previous piece's stored bytes (`zmax` per 64 KiB row)
    // into the host run on the side stream.
    void evict_z_ce(const uint8_t* src, char* host, uint64_t nbytes, const uint8_t* ebase, uint64_t* dig,
                    uint32_t zmax, cudaStream_t s) {
        std::lock_guard<std::mutex> g(zmu);
        constexpr uint64_t C = zbf16::kChunk;
        zstage_init();
        const uint64_t nch = (nbytes + C - 1) / C;
        const size_t width = std::min<size_t>((size_t(zmax) + 15) / 16 * 16, C);
        const bool short_tail = nbytes - (nch - 1) * C < zbf16::kRawTail;
        CUDA_OK(cudaEventRecord(zstart, s));  // the source is complete on the caller's stream
        CUDA_OK(cudaStreamWaitEvent(zdec, zstart, 0));
        uint64_t c0 = 0;
        while (c0 < nch) {
            const uint64_t c1 = zpiece_end(c0, nch, short_tail, zpiece);
            const int b = int(zturn++ % uint64_t(zdepth));
            CUDA_OK(cudaStreamWaitEvent(zdec, zfree[b], 0));  // the last reader of staging b is done
            const uint64_t piece = std::min(nbytes, c1 * C) - c0 * C;
            CUDA_OK(kern::evict_z(src + c0 * C, zstage[b], piece, ebase + c0, dig ? dig + c0 : nullptr, zdec,
                                  zstage_ctas));
            CUDA_OK(cudaEventRecord(zfull[b], zdec));
            CUDA_OK(cudaStreamWaitEvent(side, zfull[b], 0));
            CUDA_OK(cudaMemcpy2DAsync(host + c0 * C, C, zstage[b], C, width, c1 - c0, cudaMemcpyDeviceToHost, side));
            CUDA_OK(cudaEventRecord(zfree[b], side));
            c0 = c1;
        }
        CUDA_OK(cudaEventRecord(zdone, side));
        CUDA_OK(cudaStreamWaitEvent(s, zdone, 0));  // the evict completes on the caller's stream
    }

    void zstage_init() {
        if (!zstage[0]) {
            if (opt.stage_piece_chunks > 0) zpiece = std::max<uint64_t>(opt.stage_piece_chunks, 2);
            if (opt.stage_depth > 0) zdepth = std::min(std::max(opt.stage_depth, 2), kZDepthMax);
            for (int b = 0; b < zdepth; ++b) {
                CUDA_OK(cudaMalloc(&zstage[b], zpiece * zbf16::kChunk));
                CUDA_OK(cudaEventCreateWithFlags(&zfull[b], cudaEventDisableTiming));
                CUDA_OK(cudaEventCreateWithFlags(&zfree[b], cudaEventDisableTiming));
            }
            CUDA_OK(cudaEventCreateWithFlags(&zstart, cudaEventDisableTiming));
            CUDA_OK(cudaEventCreateWithFlags(&zdone, cudaEventDisableTiming));
            int lo = 0, hi = 0;
            cudaDeviceGetStreamPriorityRange(&lo, &hi);
            CUDA_OK(cudaStreamCreateWithPriority(&zdec, cudaStreamNonBlocking, hi));
            // coding into / decoding from staging is HBM to HBM: two CTAs per
            // SM (the kernels' occupancy), not the few dozen a PCIe pass needs
            int sms = 148;
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, opt.device);
            zstage_ctas = opt.stage_ctas > 0 ? opt.stage_ctas : 2 * sms;
        }
    }
    int zstage_ctas = 0;

    // Coded restore through the copy engine: each chunk's stored bytes (`zmax`
    // per 64 KiB row, one strided copy per piece) go into staging on the side
    // stream; K2 decodes the piece from HBM on the top-priority stream,
    // overlapping the next piece's copy, and the caller's stream joins at the end.
    void restore_z_ce(const char* host, uint8_t* dst, uint64_t nbytes, uint32_t zmax, cudaStream_t s) {
        std::lock_guard<std::mutex> g(zmu);
        constexpr uint64_t C = zbf16::kChunk;
        zstage_init();
        // the decodes write dst after the work already queued on the caller's stream
        CUDA_OK(cudaEventRecord(zstart, s));
        CUDA_OK(cudaStreamWaitEvent(zdec, zstart, 0));
        const uint64_t nch = (nbytes + C - 1) / C;
        const size_t width = std::min<size_t>((size_t(zmax) + 15) / 16 * 16, C);
        const bool short_tail = nbytes - (nch - 1) * C < zbf16::kRawTail;
        uint64_t c0 = 0;
        while (c0 < nch) {
            const uint64_t c1 = zpiece_end(c0, nch, short_tail, zpiece);
            const int b = int(zturn++ % uint64_t(zdepth));
            CUDA_OK(cudaStreamWaitEvent(side, zfree[b], 0));  // the last reader of staging b is done
            CUDA_OK(cudaMemcpy2DAsync(zstage[b], C, host + c0 * C, C, width, c1 - c0, cudaMemcpyHostToDevice, side));
            CUDA_OK(cudaEventRecord(zfull[b], side));
            CUDA_OK(cudaStreamWaitEvent(zdec, zfull[b], 0));
            const uint64_t piece = std::min(nbytes, c1 * C) - c0 * C;
            CUDA_OK(kern::restore_z(zstage[b], dst + c0 * C, piece, kern::Cast::kNone, nullptr, nullptr, nullptr, zdec,
                                    zstage_ctas));
            CUDA_OK(cudaEventRecord(zfree[b], zdec));
            c0 = c1;
        }
        CUDA_OK(cudaEventRecord(zdone, zdec));
        CUDA_OK(cudaStreamWaitEvent(s, zdone, 0));  // the caller's stream continues after the last decode
    }

    // zf32 through the copy engine: the same ring over 128 KiB rows (half as
    // many rows per piece as chunks, so a piece fills the same staging). A
    // row crosses PCIe as its 64 KiB low plane plus the stored bytes of its
    // coded top halves (`zmax`): one strided copy per piece.
    void evict_zf32_ce(const uint8_t* src, char* host, uint64_t nbytes, const uint8_t* ebase, uint32_t zmax,
                       cudaStream_t s) {
        std::lock_guard<std::mutex> g(zmu);
        constexpr uint64_t R = zf32::kRow;
        zstage_init();
        const uint64_t nrows = zf32::rows(nbytes), per = std::max<uint64_t>(zpiece / 2, 1);
        const size_t width = zf32::kLowPlane + std::min<size_t>((size_t(zmax) + 15) / 16 * 16, zbf16::kChunk);
        CUDA_OK(cudaEventRecord(zstart, s));
        CUDA_OK(cudaStreamWaitEvent(zdec, zstart, 0));
        for (uint64_t r0 = 0; r0 < nrows;) {
            const uint64_t r1 = std::min(nrows, r0 + per);
            const int b = int(zturn++ % uint64_t(zdepth));
            CUDA_OK(cudaStreamWaitEvent(zdec, zfree[b], 0));
            CUDA_OK(kern::evict_zf32(src + r0 * R, zstage[b], (r1 - r0) * R, ebase + r0, zdec, zstage_ctas));
            CUDA_OK(cudaEventRecord(zfull[b], zdec));
            CUDA_OK(cudaStreamWaitEvent(side, zfull[b], 0));
            CUDA_OK(cudaMemcpy2DAsync(host + r0 * R, R, zstage[b], R, width, r1 - r0, cudaMemcpyDeviceToHost, side));
            CUDA_OK(cudaEventRecord(zfree[b], side));
            r0 = r1;
        }
        CUDA_OK(cudaEventRecord(zdone, side));
        CUDA_OK(cudaStreamWaitEvent(s, zdone, 0));
    }

    void restore_zf32_ce(const char* host, uint8_t* dst, uint64_t nbytes, uint32_t zmax, cudaStream_t s) {
        std::lock_guard<std::mutex> g(zmu);
        constexpr uint64_t R = zf32::kRow;
        zstage_init();
        CUDA_OK(cudaEventRecord(zstart, s));
        CUDA_OK(cudaStreamWaitEvent(zdec, zstart, 0));
        const uint64_t nrows = zf32::rows(nbytes), per = std::max<uint64_t>(zpiece / 2, 1);
        const size_t width = zf32::kLowPlane + std::min<size_t>((size_t(zmax) + 15) / 16 * 16, zbf16::kChunk);
        for (uint64_t r0 = 0; r0 < nrows;) {
            const uint64_t r1 = std::min(nrows, r0 + per);
            const int b = int(zturn++ % uint64_t(zdepth));
            CUDA_OK(cudaStreamWaitEvent(side, zfree[b], 0));
            CUDA_OK(cudaMemcpy2DAsync(zstage[b], R, host + r0 * R, R, width, r1 - r0, cudaMemcpyHostToDevice, side));
            CUDA_OK(cudaEventRecord(zfull[b], side));
            CUDA_OK(cudaStreamWaitEvent(zdec, zfull[b], 0));
            CUDA_OK(kern::restore_zf32(zstage[b], dst + r0 * R, (r1 - r0) * R, zdec, zstage_ctas));
            CUDA_OK(cudaEventRecord(zfree[b], zdec));
            r0 = r1;
        }
        CUDA_OK(cudaEventRecord(zdone, zdec));
        CUDA_OK(cudaStreamWaitEvent(s, zdone, 0));
    }
    PinnedPool pool;

    struct Pending {
        bool d2h = true;
        uint64_t lease = 0, tid = 0, ver = 0, nbytes = 0;
        uint32_t slot = 0;
        cudaEvent_t ev = nullptr;
        DoneCallback cb;
        bool keep_pinned = false;
        PinnedPool::Buf dig, mism, exp;  // digests out, mismatch counter, expected digests
        uint64_t ndig = 0;
        PinnedPool::Buf zb;              // zbf16 window bases (one byte per chunk) + pre-pass flag
        PinnedPool::Buf err;             // bulk forms: device status word (0 = the copy completed)
        bool z = false;
        bool f32 = false;                // with z: the run is zf32-coded fp32 (else zbf16)
        const char* host_hash_src = nullptr;  // digests still to compute on the host from this pinned copy
        // Batched launches: every item of the batch shares one event and the
        // job table; the last item to finish releases both.
        std::shared_ptr<void> batch_keep;
    };
    std::mutex inflight_mu;
    std::list<Pending> inflight;

    struct TensorRec {
        bool offloaded = false, restored = false;
        bool failed = false;  // the device reported an incomplete copy (bounded wait expired)
        uint64_t hash_lo = 0, hash_hi = 0, lease = 0;
        uint32_t slot = 0;    // first slot of the run (a v1-only discard releases lease and slot)
        uint32_t zmax = 0;    // zbf16 run: largest stored chunk length (0: unknown)
        std::vector<uint64_t> digests;
    };
    mutable std::mutex tab_mu;
    std::condition_variable tab_cv;
    std::map<TvKey, TensorRec> tensors;

    std::atomic<uint64_t> inflight_d2h{0}, inflight_h2d{0}, evicts{0}, restores{0}, d2h_done{0}, h2d_done{0};
    std::atomic<uint64_t> coded_canonical{0};  // canonical objects that crossed PCIe zbf16-coded
    std::atomic<uint64_t> xfer_errors{0};  // copies a kernel reported incomplete
    std::atomic<uint64_t> d2h_bytes{0}, h2d_bytes{0}, registered_bytes{0}, d2h_ns{0}, h2d_ns{0}, reg_ns{0};
    std::atomic<bool> stop{false}, hb_paused{false};
    std::thread progress_thr, heartbeat_thr;

    // ------------------------------------------------------------------
    explicit Impl(const AgentOptions& o) : opt(o) {
        if (opt.uncoded != "copy_engine" && opt.uncoded != "bulk" && opt.uncoded != "sm")
            throw std::invalid_argument("uncoded must be copy_engine, bulk or sm, not '" + opt.uncoded + "'");
        if (opt.coded_restore != "copy_engine" && opt.coded_restore != "sm")
            throw std::invalid_argument("coded_restore must be copy_engine or sm, not '" + opt.coded_restore + "'");
        if (opt.coded_evict != "copy_engine" && opt.coded_evict != "sm")
            throw std::invalid_argument("coded_evict must be copy_engine or sm, not '" + opt.coded_evict + "'");
        if (opt.v1_only) {  // StateSpectre's daemon keeps no run formats and knows no submit flags
            // and applies ring entries only on its poller's schedule, so a
            // restore could overtake its own evict's completion: report by RPC
            opt.use_ring = false;
            opt.fast_submit = false;
            opt.compress = false;
            opt.compress_canonical = false;
            LOG_WARN(TAG, "v1-only session: StateSpectre opcodes 1-30, no coding, batches per item");
        }
        gpu = opt.device >= 0;
        if (gpu) {
            CUDA_OK(cudaSetDevice(opt.device));
            if (opt.kernel_timing) CUDA_OK(kern::timing_enable(opt.device, 4096));
            if (opt.numa_node < 0) {
                char bus[32] = {0};
                if (cudaDeviceGetPCIBusId(bus, sizeof(bus), opt.device) == cudaSuccess) numa = pci_numa_node(bus);
                if (numa < 0) numa = 0;
            } else {
                numa = opt.numa_node;
            }
        } else {
            numa = opt.numa_node < 0 ? 0 : opt.numa_node;
        }
        rpc.reset(new RpcClient(uds_connect(opt.socket_path)));
        RegisterRankRequest rq;
        rq.rank_id = opt.rank_id;
        rq.local_rank = opt.local_rank;
        rq.world_rank = opt.world_rank;
        rq.gpu_id = gpu ? uint32_t(opt.device) : 0xFFFFu;
        rq.numa_node = uint32_t(numa);
        rq.pid = uint64_t(::getpid());
        rq.capabilities = kCapMultiSession;
        std::vector<int> fds;
        RegisterRankResponse rr = rpc->call<Op::kRegisterRank>(rq, &fds);
        ++rpc_count;
        if (!rr.ok) {
            for (int f : fds) ::close(f);
            throw std::runtime_error("RegisterRank rejected: " + rr.message);
        }
        epoch = rr.rank_epoch;
        try {
            for (const ArenaFd& a : rr.arenas) {
                if (a.fd_index >= fds.size()) throw std::runtime_error("arena fd index out of range");
                void* p = ::mmap(nullptr, a.size, PROT_READ | PROT_WRITE, MAP_SHARED, fds[a.fd_index], 0);
                if (p == MAP_FAILED) throw std::runtime_error(std::string("mmap arena: ") + std::strerror(errno));
                ArenaMap m;
                m.id = a.arena_id;
                m.base = static_cast<char*>(p);
                m.size = a.size;
                arenas.push_back(m);
            }
            if (rr.control_fd_index >= fds.size()) throw std::runtime_error("control fd index out of range");
            control_size = rr.control_size;
            void* c = ::mmap(nullptr, control_size, PROT_READ | PROT_WRITE, MAP_SHARED, fds[rr.control_fd_index], 0);
            if (c == MAP_FAILED) throw std::runtime_error(std::string("mmap control: ") + std::strerror(errno));
            control = static_cast<char*>(c);
        } catch (...) {
            for (int f : fds) ::close(f);
            unmap_all();
            throw;
        }
        for (int f : fds) ::close(f);
        auto* h = header_of(control);
        if (h->magic != OFLD_MAGIC || h->abi_version != OFLD_ABI_VERSION) {
            unmap_all();
            throw std::runtime_error("control region magic/ABI mismatch");
        }
        slots = slots_of(control);
        num_slots = h->num_slots;
        if (opt.use_ring && rr.ring_index != 0xFFFFFFFFu) {
            RingHeader* r = ring_at(control, rr.ring_index);
            if (r && r->owner_rank == opt.rank_id && r->rank_epoch == epoch) ring = r;
        }
        if (gpu) {
            int lo = 0, hi = 0;
            cudaDeviceGetStreamPriorityRange(&lo, &hi);
            int prio = opt.stream_priority < 0 ? hi : 0;
            CUDA_OK(cudaStreamCreateWithPriority(&stream, cudaStreamNonBlocking, prio));
            CUDA_OK(cudaStreamCreateWithPriority(&side, cudaStreamNonBlocking, prio));
            CUDA_OK(cudaStreamCreateWithPriority(&aux, cudaStreamNonBlocking, prio));
        }

        // Heartbeats start before the eager pinning below: registering a
        // 100+ GB arena while other ranks pin theirs can outlast the daemon's
        // heartbeat timeout, which would expire this session.
        progress_thr = std::thread([this] { progress_loop(); });
        heartbeat_thr = std::thread([this] { heartbeat_loop(); });
        if (gpu && opt.eager_register)
            for (ArenaMap& m : arenas) register_arena(m);
        LOG_INFO(TAG, "rank %u epoch %llu %s numa %d, %zu arenas, %u slots, ring %s", opt.rank_id,
                 (unsigned long long)epoch, gpu ? ("gpu " + std::to_string(opt.device)).c_str() : "host-mode", numa,
                 arenas.size(), num_slots, ring ? "on" : "off");
    }

    ~Impl() {
        stop.store(true);
        if (progress_thr.joinable()) progress_thr.join();
        if (heartbeat_thr.joinable()) heartbeat_thr.join();
        try {
            drain_all();
        } catch (...) {
        }
        if (stream) cudaStreamDestroy(stream);
        if (side) cudaStreamDestroy(side);
        if (aux) cudaStreamDestroy(aux);
        for (int b = 0; b < kZDepthMax; ++b) {
            if (zstage[b]) cudaFree(zstage[b]);
            if (zfull[b]) cudaEventDestroy(zfull[b]);
            if (zfree[b]) cudaEventDestroy(zfree[b]);
        }
        if (zstart) cudaEventDestroy(zstart);
        if (zdone) cudaEventDestroy(zdone);
        if (zdec) cudaStreamDestroy(zdec);
        pool.clear();
        unmap_all();
    }

    void unmap_all() {
        std::lock_guard<std::mutex> g(reg_mu);
        for (ArenaMap& m : arenas) {
            for (auto& pc : m.pieces) {
                cudaHostUnregister(pc.first);
                cudaGetLastError();
            }
            m.pieces.clear();
            if (m.base) ::munmap(m.base, m.size);
        }
        arenas.clear();
        if (control) ::munmap(control, control_size);
        control = nullptr;
    }

    template <Op O>
    typename OpTypes<O>::Response call(const typename OpTypes<O>::Request& r) {
        ++rpc_count;
        return rpc->call<O>(r);
    }

    // Arena registration, mapped so kernels address it directly. Pinning is
    // page by page (4 KiB pages: memfd shmem gets no huge pages here), so a
    // large arena takes seconds; when the GPU addresses registered memory by
    // its host pointer, the arena is registered as `registration_threads`
    // pieces concurrently: the device sees one contiguous range either way.
    // Otherwise one whole-range registration (a copy must not span two
    // separately mapped registrations).
    void register_arena(ArenaMap& m) {
        std::lock_guard<std::mutex> g(reg_mu);
        if (m.registered) return;
        uint64_t t0 = mono_ns();
        const unsigned flags = cudaHostRegisterPortable | cudaHostRegisterMapped;
        int same_ptr = 0;
        cudaDeviceGetAttribute(&same_ptr, cudaDevAttrCanUseHostPointerForRegisteredMem, opt.device);
        const uint64_t min_piece = 1ull << 30;
        int nthreads = std::max(1, opt.registration_threads);
        if (!same_ptr || m.size < 2 * min_piece) nthreads = 1;
        nthreads = int(std::min<uint64_t>(uint64_t(nthreads), m.size / min_piece ? m.size / min_piece : 1));
        std::vector<std::pair<char*, uint64_t>> pieces;
        const uint64_t step = (m.size / uint64_t(nthreads) + 0xFFFFF) & ~uint64_t(0xFFFFF);  // 1 MiB aligned
        for (uint64_t off = 0; off < m.size; off += step) pieces.push_back({m.base + off, std::min(step, m.size - off)});
        std::vector<cudaError_t> errs(pieces.size(), cudaSuccess);
        auto reg = [&](size_t i) {
            cudaSetDevice(opt.device);
            errs[i] = cudaHostRegister(pieces[i].first, pieces[i].second, flags);
            if (errs[i] == cudaErrorHostMemoryAlreadyRegistered) {
                cudaGetLastError();
                errs[i] = cudaSuccess;
            }
        };
        if (pieces.size() == 1) {
            reg(0);
        } else {
            std::vector<std::thread> ts;
            for (size_t i = 0; i < pieces.size(); ++i) ts.emplace_back(reg, i);
            for (auto& t : ts) t.join();
        }
        for (size_t i = 0; i < pieces.size(); ++i) {
            if (errs[i] != cudaSuccess) {
                for (size_t j = 0; j < pieces.size(); ++j)
                    if (errs[j] == cudaSuccess) cudaHostUnregister(pieces[j].first);
                cudaGetLastError();
                throw std::runtime_error(std::string("cudaHostRegister(arena): ") + cudaGetErrorString(errs[i]));
            }
        }
        void* dev = nullptr;
        CUDA_OK(cudaHostGetDevicePointer(&dev, m.base, 0));
        if (pieces.size() > 1 && dev != m.base) {  // cannot happen when same_ptr; keep the invariant explicit
            for (auto& pc : pieces) cudaHostUnregister(pc.first);
            throw std::runtime_error("pieced registration without host-pointer addressing");
        }
        m.dev = static_cast<char*>(dev);
        m.pieces = std::move(pieces);
        m.registered = true;
        registered_bytes += m.size;
        const double ms = double(mono_ns() - t0) / 1e6;
        reg_ns += uint64_t(ms * 1e6);
        LOG_INFO(TAG, "registered arena %llu: %llu MiB in %.1f ms (%zu piece%s)", (unsigned long long)m.id,
                 (unsigned long long)(m.size >> 20), ms, m.pieces.size(), m.pieces.size() == 1 ? "" : "s");
    }

    ArenaMap& arena(uint64_t id) {
        for (ArenaMap& m : arenas)
            if (m.id == id) return m;
        throw std::runtime_error("unknown arena id " + std::to_string(id));
    }

    // Host pointer and (GPU mode) device alias of (arena, offset, nbytes).
    void resolve(uint64_t arena_id, uint64_t off, uint64_t nbytes, char** host, char** dev) {
        ArenaMap& m = arena(arena_id);
        if (off + nbytes > m.size) throw std::runtime_error("slot range outside arena");
        *host = m.base + off;
        if (gpu) {
            register_arena(m);
            *dev = m.dev + off;
        } else {
            *dev = nullptr;
        }
    }

    cudaStream_t stream_of(StreamHandle s) const {
        return s == kInternalStream ? stream : reinterpret_cast<cudaStream_t>(s);
    }

    // ---- completions -----------------------------------------------------
    bool ring_push_entry(EventType ev, const Pending& p) {
        if (!ring) return false;
        std::lock_guard<std::mutex> g(ring_mu);
        ofld_completion_entry_t e{};
        e.lease_id = p.lease;
        e.tensor_id = p.tid;
        e.version = p.ver;
        e.slot_id = p.slot;
        e.event_type = uint32_t(ev);
        e.timestamp_ns = real_ns();
        return ring_push(ring, e);
    }

    // A completion goes through the shared ring when it has room; the daemon
    // applies pending ring entries before answering any request that depends
    // on them, so the next request of this rank sees it.
    void report_d2h(const Pending& p) {
        if (!ring_push_entry(EventType::kD2HComplete, p)) {
            TransferMark m;
            m.rank_id = opt.rank_id;
            m.rank_epoch = epoch;
            m.lease_id = p.lease;
            m.tensor_id = p.tid;
            m.version = p.ver;
            m.slot_id = p.slot;
            m.timestamp_ns = real_ns();
            MarkD2HCompleteResponse r = call<Op::kMarkD2HComplete>(m);
            if (!r.ok) LOG_ERR(TAG, "MarkD2HComplete rejected for tensor %llu", (unsigned long long)p.tid);
        }
    }

    void report_h2d(const Pending& p) {
        // keep_pinned cannot travel through the ring; the RPC carries it.
        if (!p.keep_pinned && ring_push_entry(EventType::kH2DComplete, p)) return;
        {
            MarkH2DCompleteRequest m;
            m.rank_id = opt.rank_id;
            m.rank_epoch = epoch;
            m.lease_id = p.lease;
            m.tensor_id = p.tid;
            m.version = p.ver;
            m.slot_id = p.slot;
            m.keep_pinned = p.keep_pinned;
            m.timestamp_ns = real_ns();
            StatusResponse r = call<Op::kMarkH2DComplete>(m);
            if (!r.ok) LOG_ERR(TAG, "MarkH2DComplete rejected for tensor %llu: %s", (unsigned long long)p.tid,
                               r.message.c_str());
        }
    }

    // Retire one completed transfer (copy finished).
    // Device status of a bulk launch (a bounded wait inside the kernel that
    // ran out leaves the copy incomplete); the status buffer returns to the pool.
    uint32_t take_device_status(Pending& p) {
        if (!p.err.host) return 0;
        const uint32_t e = *static_cast<volatile uint32_t*>(p.err.host);
        pool.put(p.err);
        p.err = PinnedPool::Buf{};
        return e;
    }

    void finish(Pending& p) {
        if (const uint32_t derr = take_device_status(p)) {
            LOG_ERR(TAG, "%s of tensor %llu v%llu incomplete: device status %u", p.d2h ? "evict" : "restore",
                    (unsigned long long)p.tid, (unsigned long long)p.ver, derr);
            ++xfer_errors;
            if (p.d2h) {
                // the pinned run holds partial bytes: give it back instead of publishing it
                ReleaseLeaseRequest rl{opt.rank_id, epoch, p.lease, p.slot, "device copy incomplete"};
                (void)call<Op::kReleaseLease>(rl);
                pool.put(p.dig);
                pool.put(p.zb);
                p.zb = PinnedPool::Buf{};
                {
                    std::lock_guard<std::mutex> g(tab_mu);
                    TensorRec& t = tensors[{p.tid, p.ver}];
                    t.offloaded = true;  // waiters wake and see the failure
                    t.failed = true;
                }
                inflight_d2h -= p.nbytes;
                if (p.cb) p.cb();
                if (p.batch_keep) p.batch_keep.reset();
                else if (p.ev) cudaEventDestroy(p.ev);
                p.ev = nullptr;
                tab_cv.notify_all();
                return;
            }
            std::lock_guard<std::mutex> g(tab_mu);
            tensors[{p.tid, p.ver}].failed = true;
        }
        if (p.d2h) {
            uint64_t lo = 0, hi = 0;
            std::vector<uint64_t> dig;
            host_digests(p);
            if (p.dig.host) {
                const uint64_t* d = static_cast<const uint64_t*>(p.dig.host);
                ssh::Object o = ssh::fold_digests(d, p.ndig, p.nbytes);
                lo = o.lo;
                hi = o.hi;
                if (opt.keep_digests) dig.assign(d, d + p.ndig);
                pool.put(p.dig);
            }
            pool.put(p.zb);
            p.zb = PinnedPool::Buf{};
            report_d2h(p);
            {
                std::lock_guard<std::mutex> g(tab_mu);
                TensorRec& t = tensors[{p.tid, p.ver}];
                t.offloaded = true;
                t.restored = false;
                t.hash_lo = lo;
                t.hash_hi = hi;
                t.lease = p.lease;
                t.slot = p.slot;
                t.digests = std::move(dig);
            }
            inflight_d2h -= p.nbytes;
            ++d2h_done;
            d2h_bytes += p.nbytes;
            if (p.cb) p.cb();
        } else {
            report_h2d(p);
            {
                std::lock_guard<std::mutex> g(tab_mu);
                tensors[{p.tid, p.ver}].restored = true;
            }
            inflight_h2d -= p.nbytes;
            ++h2d_done;
            h2d_bytes += p.nbytes;
            pool.put(p.mism);
            pool.put(p.exp);
            pool.put(p.dig);  // zf32 verification: digests of the restored bytes
            if (p.cb) p.cb();
        }
        if (p.batch_keep) p.batch_keep.reset();  // shared event: the keep owns it
        else if (p.ev) cudaEventDestroy(p.ev);
        p.ev = nullptr;
        tab_cv.notify_all();
    }

    // One event and one job table for a batched launch, shared by its items.
    std::shared_ptr<void> make_batch_keep(cudaEvent_t ev, PinnedPool::Buf jobs) {
        struct Keep {
            cudaEvent_t ev;
            PinnedPool::Buf jobs;
            PinnedPool* pool;
            ~Keep() {
                cudaEventDestroy(ev);
                pool->put(jobs);
            }
        };
        return std::shared_ptr<void>(new Keep{ev, jobs, &pool}, [](void* k) { delete static_cast<Keep*>(k); });
    }

    bool batch_kernel_ok(uint64_t ptr, uint64_t nbytes) const {
        return gpu && opt.engine != "copy_engine" && (ptr & 15) == 0 && nbytes % 16 == 0 && nbytes > 0;
    }

    void progress_loop() {
        if (gpu) cudaSetDevice(opt.device);
        pin_thread_to_node(numa);
        const uint64_t poll = opt.progress_poll_us ? opt.progress_poll_us : 50;
        while (!stop.load()) {
            std::list<Pending> done;
            {
                std::lock_guard<std::mutex> g(inflight_mu);
                for (auto it = inflight.begin(); it != inflight.end();) {
                    cudaError_t st = cudaEventQuery(it->ev);
                    if (st == cudaErrorNotReady) {
                        ++it;
                        continue;
                    }
                    if (st != cudaSuccess) LOG_ERR(TAG, "transfer failed: %s", cudaGetErrorString(st));
                    auto nx = std::next(it);
                    done.splice(done.end(), inflight, it);
                    it = nx;
                }
            }
            for (Pending& p : done) {
                try {
                    finish(p);
                } catch (const std::exception& e) {
                    LOG_ERR(TAG, "completion failed: %s", e.what());
                }
            }
            if (done.empty()) sleep_us(poll);
        }
    }

    void drain_all() {
        std::list<Pending> all;
        {
            std::lock_guard<std::mutex> g(inflight_mu);
            all.swap(inflight);
        }
        for (Pending& p : all) {
            if (p.ev) cudaEventSynchronize(p.ev);
            finish(p);
        }
    }

    void heartbeat_loop() {
        const uint64_t period = opt.heartbeat_ms ? opt.heartbeat_ms : 1000;
        uint64_t next = mono_ns() + period * 1000000ull;
        while (!stop.load()) {
            sleep_us(10000);
            if (mono_ns() < next || hb_paused.load()) continue;
            next = mono_ns() + period * 1000000ull;
            HeartbeatRequest hb{opt.rank_id, epoch, real_ns()};
            try {
                StatusResponse r = call<Op::kHeartbeat>(hb);
                if (!r.ok) LOG_ERR(TAG, "heartbeat rejected: %s (session invalidated?)", r.message.c_str());
            } catch (const std::exception& e) {
                LOG_ERR(TAG, "heartbeat failed: %s", e.what());
            }
        }
    }

    // Launch K1 (or the copy-engine A/B path) for one reserved run.
    // zbf16 pre-pass: per-chunk window bases into a mapped buffer; true when
    // every chunk fits coded. Waits for the stream (the decision precedes the
    // reservation, whose flags record the format).
    bool zscan(uint64_t src, uint64_t nbytes, cudaStream_t s, PinnedPool::Buf* out, bool f32 = false) {
        zscan_launch(src, nbytes, s, out, f32);
        stream_wait(s);
        return zscan_result(nbytes, out);
    }
    // The pre-pass in two halves, so a batch launches every item's scan and
    // waits once. f32: the zf32 pre-pass (one window base per 128 KiB row;
    // the layout below is sized by 64 KiB chunks either way).
    void zscan_launch(uint64_t src, uint64_t nbytes, cudaStream_t s, PinnedPool::Buf* out, bool f32 = false) {
        const uint64_t nch = kern::digest_count(nbytes);
        const uint64_t flag_off = (nch + 15) / 16 * 16;
        // [window bases][pad][fail word + 12 pad][kZScanSlots per-CTA stored-length maxima]
        *out = pool.get(flag_off + 16 + 4 * kern::kZScanSlots);
        std::memset(static_cast<char*>(out->host) + flag_off, 0, 16 + 4 * kern::kZScanSlots);
        auto* fail = reinterpret_cast<uint32_t*>(static_cast<char*>(out->dev) + flag_off);
        auto* maxc = reinterpret_cast<uint32_t*>(static_cast<char*>(out->dev) + flag_off + 16);
        if (f32)
            CUDA_OK(kern::zscan_f32(reinterpret_cast<const void*>(src), nbytes, static_cast<uint8_t*>(out->dev), fail,
                                    s, 0, maxc));
        else
            CUDA_OK(kern::zscan(reinterpret_cast<const void*>(src), nbytes, static_cast<uint8_t*>(out->dev), fail, s, 0,
                                maxc));
    }
    // Largest stored chunk length recorded by the pre-pass (valid after zscan_result).
    uint32_t zscan_max(uint64_t nbytes, const PinnedPool::Buf& b) const {
        if (!b.host) return 0;
        const uint64_t flag_off = (kern::digest_count(nbytes) + 15) / 16 * 16;
        const volatile uint32_t* m =
            reinterpret_cast<const volatile uint32_t*>(static_cast<const char*>(b.host) + flag_off + 16);
        uint32_t w = 0;
        for (int i = 0; i < kern::kZScanSlots; ++i) w = std::max<uint32_t>(w, uint32_t(m[i]));
        return w;
    }
    bool zscan_result(uint64_t nbytes, PinnedPool::Buf* out) {
        const uint64_t flag_off = (kern::digest_count(nbytes) + 15) / 16 * 16;
        if (*reinterpret_cast<volatile uint32_t*>(static_cast<char*>(out->host) + flag_off) == 0) return true;
        pool.put(*out);
        *out = PinnedPool::Buf{};
        return false;
    }
    void stream_wait(cudaStream_t s) {
        cudaEvent_t ev;
        CUDA_OK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        CUDA_OK(cudaEventRecord(ev, s));
        CUDA_OK(cudaEventSynchronize(ev));
        cudaEventDestroy(ev);
    }

    // Calls on opcodes StateSpectre's daemon does not have: refuse in v1-only
    // mode (that daemon would leave them unanswered).
    void need_ext(const char* what) const {
        if (opt.v1_only)
            throw std::runtime_error(std::string(what) + " needs this repository's offloadd (the session is v1-only)");
    }

    bool want_z(uint64_t ptr, uint64_t nbytes, uint32_t fmt_hint) const {
        return gpu && fmt_hint == kFmtBf16 && opt.compress && opt.engine != "copy_engine" &&
               nbytes >= opt.compress_min_bytes && zbf16::eligible(nbytes) && (ptr & 15) == 0;
    }
    bool want_zf32(uint64_t ptr, uint64_t nbytes, uint32_t fmt_hint) const {
        return gpu && fmt_hint == kFmtF32 && opt.compress && opt.engine != "copy_engine" &&
               nbytes >= opt.compress_min_bytes && zf32::eligible(nbytes) && (ptr & 15) == 0;
    }

    // Format of the bytes in a granted run (slot entries of the shared table).
    uint64_t run_format(uint32_t slot) const {
        return slots && slot < num_slots
                   ? reinterpret_cast<const volatile uint64_t&>(slots[slot].flags) & OFLD_FLAG_FORMAT_MASK
                   : 0;
    }
    bool run_is_z(uint32_t slot) const { return (run_format(slot) & OFLD_FLAG_FORMAT_ZBF16) != 0; }
    // First slot of the run that starts at (arena, offset): the slot table's
    // placement never changes, so the index is built once (canonical restores
    // learn a run by its arena position only).
    std::mutex slot_index_mu;
    std::unordered_map<uint64_t, uint32_t> slot_index;  // (arena << 48) | offset -> slot
    int64_t slot_at(uint64_t arena_id, uint64_t offset) {
        if (!slots) return -1;
        std::lock_guard<std::mutex> g(slot_index_mu);
        if (slot_index.empty())
            for (uint32_t i = 0; i < num_slots; ++i)
                slot_index[(uint64_t(slots[i].arena_id) << 48) | slots[i].arena_offset] = i;
        auto it = slot_index.find((arena_id << 48) | offset);
        return it == slot_index.end() ? -1 : int64_t(it->second);
    }
    bool run_is_zf32(uint32_t slot) const { return (run_format(slot) & OFLD_FLAG_FORMAT_ZF32) != 0; }

    // Digests of a small evict hashed on the host (host_hash_max_bytes), from
    // its pinned copy, once that copy has completed.
    static void host_digests(Pending& p) {
        if (!p.host_hash_src || !p.dig.host) return;
        ssh::host_chunk_digests(p.host_hash_src, p.nbytes, static_cast<uint64_t*>(p.dig.host));
        p.host_hash_src = nullptr;
    }

    void launch_d2h(Pending& p, uint64_t src, char* dst_host, char* dst_dev, cudaStream_t s, bool hash) {
        if (!gpu) {
            std::memcpy(dst_host, reinterpret_cast<const void*>(src), p.nbytes);
            if (hash) {
                p.ndig = kern::digest_count(p.nbytes);
                p.dig.host = std::malloc(std::max<uint64_t>(p.ndig, 1) * 8);  // host mode: plain memory
                ssh::host_chunk_digests(dst_host, p.nbytes, static_cast<uint64_t*>(p.dig.host));
            }
            return;
        }
        uint64_t* dig_dev = nullptr;
        if (hash) {
            p.ndig = kern::digest_count(p.nbytes);
            p.dig = pool.get(std::max<uint64_t>(p.ndig, 1) * 8);
            dig_dev = static_cast<uint64_t*>(p.dig.dev);
        }
        const uint32_t zmax = p.z ? zscan_max(p.nbytes, p.zb) : 0;
        if (p.z && p.f32) {
            // zf32: the coder computes no digests; they come from the fp32
            // bytes on the aux stream, next to the coding and the copies
            cudaEvent_t fork = nullptr, join = nullptr;
            if (hash) {
                CUDA_OK(cudaEventCreateWithFlags(&fork, cudaEventDisableTiming));
                CUDA_OK(cudaEventCreateWithFlags(&join, cudaEventDisableTiming));
                CUDA_OK(cudaEventRecord(fork, s));
                CUDA_OK(cudaStreamWaitEvent(aux, fork, 0));
                CUDA_OK(kern::hash_device(reinterpret_cast<const void*>(src), p.nbytes, dig_dev, aux, opt.hash_ctas));
                CUDA_OK(cudaEventRecord(join, aux));
            }
            if (opt.coded_evict == "copy_engine" && zmax > 0 && (src & 15) == 0 &&
                (reinterpret_cast<uintptr_t>(dst_host) & 15) == 0)
                evict_zf32_ce(reinterpret_cast<const uint8_t*>(src), dst_host, p.nbytes,
                              static_cast<const uint8_t*>(p.zb.dev), zmax, s);
            else
                CUDA_OK(kern::evict_zf32(reinterpret_cast<const void*>(src), dst_dev, p.nbytes,
                                         static_cast<const uint8_t*>(p.zb.dev), s, opt.evict_ctas));
            if (hash) {
                CUDA_OK(cudaStreamWaitEvent(s, join, 0));
                cudaEventDestroy(fork);
                cudaEventDestroy(join);
            }
        } else if (p.z && opt.coded_evict == "copy_engine" && zmax > 0 && (src & 15) == 0 &&
            (reinterpret_cast<uintptr_t>(dst_host) & 15) == 0) {
            evict_z_ce(reinterpret_cast<const uint8_t*>(src), dst_host, p.nbytes, static_cast<const uint8_t*>(p.zb.dev),
                       dig_dev, zmax, s);
        } else if (p.z) {
            CUDA_OK(kern::evict_z(reinterpret_cast<const void*>(src), dst_dev, p.nbytes,
                                  static_cast<const uint8_t*>(p.zb.dev), dig_dev, s, opt.evict_ctas));
        } else if (opt.engine == "copy_engine" || opt.uncoded == "copy_engine") {
            if (hash && p.nbytes <= opt.host_hash_max_bytes) {
                CUDA_OK(cudaMemcpyAsync(dst_host, reinterpret_cast<const void*>(src), p.nbytes, cudaMemcpyDeviceToHost,
                                        s));
                p.host_hash_src = dst_host;  // digests once the copy is done (host_digests)
            } else if (hash) {
                // the digests read HBM on a side stream while the copy engine
                // crosses PCIe; the caller's stream waits for both
                cudaEvent_t fork = nullptr, join = nullptr;
                CUDA_OK(cudaEventCreateWithFlags(&fork, cudaEventDisableTiming));
                CUDA_OK(cudaEventCreateWithFlags(&join, cudaEventDisableTiming));
                CUDA_OK(cudaEventRecord(fork, s));
                CUDA_OK(cudaStreamWaitEvent(side, fork, 0));
                CUDA_OK(kern::hash_device(reinterpret_cast<const void*>(src), p.nbytes, dig_dev, side, opt.hash_ctas));
                CUDA_OK(cudaEventRecord(join, side));
                CUDA_OK(cudaMemcpyAsync(dst_host, reinterpret_cast<const void*>(src), p.nbytes, cudaMemcpyDeviceToHost,
                                        s));
                CUDA_OK(cudaStreamWaitEvent(s, join, 0));
                cudaEventDestroy(fork);
                cudaEventDestroy(join);
            } else {
                CUDA_OK(cudaMemcpyAsync(dst_host, reinterpret_cast<const void*>(src), p.nbytes, cudaMemcpyDeviceToHost,
                                        s));
            }
        } else if (opt.uncoded == "bulk" && kern::bulk_ok(reinterpret_cast<const void*>(src), dst_dev, p.nbytes)) {
            p.err = pool.get(16);
            *static_cast<volatile uint32_t*>(p.err.host) = 0;
            CUDA_OK(kern::evict_bulk(reinterpret_cast<const void*>(src), dst_dev, p.nbytes, dig_dev,
                                     static_cast<uint32_t*>(p.err.dev), s, opt.evict_ctas));
        } else {
            CUDA_OK(kern::evict_hash(reinterpret_cast<const void*>(src), dst_dev, p.nbytes, dig_dev, s, opt.evict_ctas));
        }
        CUDA_OK(cudaEventCreateWithFlags(&p.ev, cudaEventDisableTiming));
        CUDA_OK(cudaEventRecord(p.ev, s));
    }

    void complete_or_queue(Pending&& p, bool wait) {
        if (!gpu || wait) {
            if (p.ev) CUDA_OK(cudaEventSynchronize(p.ev));
            if (!gpu && p.dig.host) {
                // host-mode digests are malloc'd, not pooled
                const uint64_t* d = static_cast<const uint64_t*>(p.dig.host);
                std::vector<uint64_t> keep(d, d + p.ndig);
                std::free(p.dig.host);
                p.dig = {};
                ssh::Object o = ssh::fold_digests(keep.data(), keep.size(), p.nbytes);
                report_d2h(p);
                {
                    std::lock_guard<std::mutex> g(tab_mu);
                    TensorRec& t = tensors[{p.tid, p.ver}];
                    t.offloaded = true;
                    t.restored = false;
                    t.hash_lo = o.lo;
                    t.hash_hi = o.hi;
                    t.lease = p.lease;
                    t.slot = p.slot;
                    if (opt.keep_digests) t.digests = std::move(keep);
                }
                inflight_d2h -= p.nbytes;
                ++d2h_done;
                d2h_bytes += p.nbytes;
                if (p.cb) p.cb();
                tab_cv.notify_all();
                return;
            }
            finish(p);
            return;
        }
        std::lock_guard<std::mutex> g(inflight_mu);
        inflight.push_back(std::move(p));
    }
};

// ============================================================================
Agent::Agent(const AgentOptions& opt) : d_(new Impl(opt)) {}
Agent::~Agent() = default;

EvictTicket Agent::evict(uint64_t ptr, uint64_t nbytes, StreamHandle stream, bool destructive, uint64_t tensor_id,
                         uint64_t version, const std::string& name, DoneCallback on_done, bool wait,
                         uint32_t fmt_hint) {
    NvtxRange nvtx_("ofld.evict");
    Impl& D = *d_;
    EvictTicket t;
    t.tensor_id = tensor_id;
    t.version = version;
    t.nbytes = nbytes;
    if (nbytes == 0) {
        t.message = "nbytes must be > 0";
        return t;
    }
    RequestOffloadRequest rq;
    rq.rank_id = D.opt.rank_id;
    rq.rank_epoch = D.epoch;
    rq.tensor_id = tensor_id;
    rq.version = version;
    rq.nbytes = nbytes;
    rq.gpu_id = D.gpu ? uint32_t(D.opt.device) : 0;
    rq.numa_node = uint32_t(D.numa);
    rq.alignment = 256;
    rq.flags = OFLD_FLAG_ALLOW_OVERFLOW | (destructive ? OFLD_FLAG_DESTRUCTIVE : 0) |
               (D.opt.fast_submit ? OFLD_FLAG_SUBMIT_ON_GRANT : 0);
    rq.debug_name = name;
    PinnedPool::Buf zb;
    bool z = false, f32 = false;
    if (D.want_z(ptr, nbytes, fmt_hint))
        z = D.zscan(ptr, nbytes, D.stream_of(stream), &zb);
    else if (D.want_zf32(ptr, nbytes, fmt_hint))
        z = f32 = D.zscan(ptr, nbytes, D.stream_of(stream), &zb, true);
    if (z) rq.flags |= f32 ? OFLD_FLAG_FORMAT_ZF32 : OFLD_FLAG_FORMAT_ZBF16;
    RequestOffloadResponse g = D.call<Op::kRequestOffload>(rq);
    // Backpressure: every pinned run can be briefly held by transfers in
    // flight (readbacks, restores) with nothing drainable; they release runs
    // shortly, so a blocked reservation is retried for up to blocked_wait_ms.
    const uint64_t blocked_deadline = mono_ns() + D.opt.blocked_wait_ms * 1000000ull;
    uint64_t backoff_us = 200;
    while (g.blocked && mono_ns() < blocked_deadline) {
        sleep_us(backoff_us);
        backoff_us = std::min<uint64_t>(backoff_us * 2, 20000);
        g = D.call<Op::kRequestOffload>(rq);
    }
    if (!g.ok || g.blocked) {
        D.pool.put(zb);
        t.message = g.ok ? "offload blocked (pinned pressure)" : g.message;
        return t;
    }
    ++D.evicts;
    char *host = nullptr, *dev = nullptr;
    D.resolve(g.arena_id, g.arena_offset, nbytes, &host, &dev);
    if (g.state != OFLD_SLOT_D2H_IN_FLIGHT) {
        TransferMark m{D.opt.rank_id, D.epoch, g.lease_id, tensor_id, version, g.slot_id, 0, real_ns()};
        StatusResponse sr = D.call<Op::kMarkD2HSubmitted>(m);
        if (!sr.ok) LOG_WARN(TAG, "MarkD2HSubmitted: %s (continuing)", sr.message.c_str());
    }
    Impl::Pending p;
    p.d2h = true;
    p.lease = g.lease_id;
    p.tid = tensor_id;
    p.ver = version;
    p.slot = g.slot_id;
    p.nbytes = nbytes;
    p.cb = std::move(on_done);
    p.z = z;
    p.f32 = f32;
    p.zb = zb;
    t.coded = z;
    D.inflight_d2h += nbytes;
    {
        std::lock_guard<std::mutex> lg(D.tab_mu);
        Impl::TensorRec& r = D.tensors[{tensor_id, version}];
        r.offloaded = false;
        r.lease = g.lease_id;
        r.slot = g.slot_id;
        r.zmax = z ? D.zscan_max(nbytes, zb) : 0;
    }
    D.launch_d2h(p, ptr, host, dev, D.stream_of(stream), D.opt.hash_on_evict);
    D.complete_or_queue(std::move(p), wait);
    t.ok = true;
    t.message = "ok";
    t.lease_id = g.lease_id;
    t.slot_id = g.slot_id;
    if (wait) {
        std::lock_guard<std::mutex> lg(D.tab_mu);
        auto it = D.tensors.find({tensor_id, version});
        if (it != D.tensors.end() && it->second.failed) {
            t.ok = false;
            t.message = "evict: device copy incomplete (bounded wait expired)";
            return t;
        }
    }
    if (wait) tensor_hash(tensor_id, version, &t.hash_lo, &t.hash_hi);
    return t;
}

// Batched eviction. One zbf16 pre-pass launch covers every eligible item
// and the stream is waited on once; then the batch is reserved and launched
// in groups of about batch_group_bytes, each group one K1 launch, so the
// daemon round trip of group g+1 overlaps the PCIe copy of group g.
// Items the daemon answers as blocked (pinned window full) are retried for
// up to blocked_wait_ms, after the groups already launched have had their
// completions handed on: a pinned run becomes drainable only once its copy
// is published, so the retry never waits on the batch's own reservations.
std::vector<EvictTicket> Agent::evict_batch(const std::vector<BatchItem>& items, StreamHandle stream, bool wait) {
    NvtxRange nvtx_("ofld.evict_batch");
    Impl& D = *d_;
    if (D.opt.v1_only) {  // no batch opcodes: one evict per item
        std::vector<EvictTicket> out;
        out.reserve(items.size());
        for (const BatchItem& it : items)
            out.push_back(evict(it.ptr, it.nbytes, stream, false, it.tensor_id, it.version, "", {}, wait, it.fmt_hint));
        return out;
    }
    std::vector<EvictTicket> out(items.size());
    cudaStream_t s = D.stream_of(stream);
    std::vector<PinnedPool::Buf> zb(items.size());
    std::vector<char> z(items.size(), 0);
    {
        std::vector<kern::XferJob> scan;
        uint64_t scan_chunks = 0;
        for (size_t i = 0; i < items.size(); ++i) {
            if (!D.want_z(items[i].ptr, items[i].nbytes, items[i].fmt_hint)) continue;
            const uint64_t nch = kern::digest_count(items[i].nbytes);
            const uint64_t flag_off = (nch + 15) / 16 * 16;
            zb[i] = D.pool.get(flag_off + 16);
            *reinterpret_cast<volatile uint32_t*>(static_cast<char*>(zb[i].host) + flag_off) = 0;
            kern::XferJob j{};
            j.src = reinterpret_cast<const void*>(items[i].ptr);
            j.dst = zb[i].dev;
            j.nbytes = items[i].nbytes;
            j.chunk_begin = scan_chunks;
            scan_chunks += nch;
            scan.push_back(j);
            z[i] = 1;
        }
        if (!scan.empty()) {
            PinnedPool::Buf tab = D.pool.get(scan.size() * sizeof(kern::XferJob));
            std::memcpy(tab.host, scan.data(), scan.size() * sizeof(kern::XferJob));
            CUDA_OK(kern::zscan_jobs(static_cast<const kern::XferJob*>(tab.dev), int(scan.size()), scan_chunks, s,
                                     D.opt.hash_ctas));
            D.stream_wait(s);
            D.pool.put(tab);
            for (size_t i = 0; i < items.size(); ++i)
                if (z[i]) z[i] = D.zscan_result(items[i].nbytes, &zb[i]);
        }
    }
    std::vector<Impl::Pending> launched;
    cudaEvent_t last_ev = nullptr;
    const uint64_t group_bytes = std::max<uint64_t>(D.opt.batch_group_bytes, 1);
    std::vector<size_t> todo(items.size()), blocked;
    for (size_t i = 0; i < items.size(); ++i) todo[i] = i;
    const uint64_t blocked_deadline = mono_ns() + D.opt.blocked_wait_ms * 1000000ull;
    uint64_t backoff_us = 200;
    for (;;) {
        blocked.clear();
        for (size_t g0 = 0; g0 < todo.size();) {
            size_t g1 = g0;
            uint64_t bytes = 0;
            while (g1 < todo.size() && (g1 == g0 || bytes < group_bytes)) bytes += items[todo[g1++]].nbytes;
            BatchRequestOffloadRequest br;
            br.rank_id = D.opt.rank_id;
            br.rank_epoch = D.epoch;
            for (size_t k = g0; k < g1; ++k) {
                const size_t i = todo[k];
                const BatchItem& it = items[i];
                RequestOffloadRequest rq;
                rq.tensor_id = it.tensor_id;
                rq.version = it.version;
                rq.nbytes = it.nbytes;
                rq.gpu_id = D.gpu ? uint32_t(D.opt.device) : 0;
                rq.numa_node = uint32_t(D.numa);
                rq.alignment = 256;
                rq.flags = OFLD_FLAG_ALLOW_OVERFLOW | OFLD_FLAG_SUBMIT_ON_GRANT | (z[i] ? OFLD_FLAG_FORMAT_ZBF16 : 0);
                br.items.push_back(rq);
            }
            BatchRequestOffloadResponse resp = D.call<Op::kBatchRequestOffload>(br);
            std::vector<kern::XferJob> jobs;  // this group's items on the job kernel, one K1 launch
            const size_t first = launched.size();
            uint64_t total_chunks = 0;
            for (size_t k = g0; k < g1; ++k) {
                const size_t i = todo[k];
                EvictTicket& t = out[i];
                t.tensor_id = items[i].tensor_id;
                t.version = items[i].version;
                t.nbytes = items[i].nbytes;
                if (k - g0 >= resp.grants.size()) {
                    t.message = resp.message.empty() ? "no grant" : resp.message;
                    continue;
                }
                const RequestOffloadResponse& g = resp.grants[k - g0];
                if (!g.ok || g.blocked) {
                    t.message = g.ok ? "offload blocked (pinned pressure)" : g.message;
                    if (g.blocked) blocked.push_back(i);
                    continue;
                }
                char *host = nullptr, *dev = nullptr;
                D.resolve(g.arena_id, g.arena_offset, items[i].nbytes, &host, &dev);
                Impl::Pending p;
                p.z = z[i] != 0;
                p.zb = zb[i];
                zb[i] = PinnedPool::Buf{};
                t.coded = p.z;
                p.lease = g.lease_id;
                p.tid = items[i].tensor_id;
                p.ver = items[i].version;
                p.slot = g.slot_id;
                p.nbytes = items[i].nbytes;
                D.inflight_d2h += p.nbytes;
                ++D.evicts;
                {
                    std::lock_guard<std::mutex> lg(D.tab_mu);
                    D.tensors[{p.tid, p.ver}].offloaded = false;
                }
                // Every item of the group, coded or not, goes into one job-kernel
                // launch: per-item copy-engine copies with their digest kernels
                // beside a training step evicted 4 MiB KV blocks at 30.5 GB/s,
                // the job kernel at 46.7 GB/s (restores: see restore_batch).
                if (D.batch_kernel_ok(items[i].ptr, p.nbytes)) {
                    kern::XferJob j{};
                    j.src = reinterpret_cast<const void*>(items[i].ptr);
                    j.dst = dev;
                    j.nbytes = p.nbytes;
                    j.chunk_begin = total_chunks;
                    j.ebase = p.z ? static_cast<const uint8_t*>(p.zb.dev) : nullptr;
                    if (D.opt.hash_on_evict) {
                        p.ndig = kern::digest_count(p.nbytes);
                        p.dig = D.pool.get(std::max<uint64_t>(p.ndig, 1) * 8);
                        j.digests = static_cast<uint64_t*>(p.dig.dev);
                    }
                    total_chunks += kern::digest_count(p.nbytes);
                    jobs.push_back(j);
                } else {
                    D.launch_d2h(p, items[i].ptr, host, dev, s, D.opt.hash_on_evict);
                    if (p.ev) last_ev = p.ev;
                }
                t.ok = true;
                t.lease_id = g.lease_id;
                t.slot_id = g.slot_id;
                launched.push_back(std::move(p));
            }
            if (!jobs.empty()) {
                PinnedPool::Buf tab = D.pool.get(jobs.size() * sizeof(kern::XferJob));
                std::memcpy(tab.host, jobs.data(), jobs.size() * sizeof(kern::XferJob));
                CUDA_OK(kern::evict_jobs(static_cast<const kern::XferJob*>(tab.dev), int(jobs.size()), total_chunks, s,
                                         D.opt.evict_ctas));
                cudaEvent_t ev;
                CUDA_OK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
                CUDA_OK(cudaEventRecord(ev, s));
                auto keep = D.make_batch_keep(ev, tab);
                for (size_t k = first; k < launched.size(); ++k)
                    if (!launched[k].ev) {
                        launched[k].ev = ev;
                        launched[k].batch_keep = keep;
                    }
                last_ev = ev;
            }
            g0 = g1;
        }
        // The last event recorded covers every launch so far on this stream, so a
        // waiting caller synchronizes once per pass.
        if (wait && D.gpu && last_ev) CUDA_OK(cudaEventSynchronize(last_ev));
        for (Impl::Pending& p : launched) D.complete_or_queue(std::move(p), wait);
        launched.clear();
        last_ev = nullptr;
        if (blocked.empty() || mono_ns() >= blocked_deadline) break;
        sleep_us(backoff_us);
        backoff_us = std::min<uint64_t>(backoff_us * 2, 20000);
        todo.swap(blocked);
    }
    for (PinnedPool::Buf& b : zb) D.pool.put(b);  // items without a grant
    return out;
}

RestoreOutcome Agent::restore(uint64_t tensor_id, uint64_t version, uint64_t ptr, uint64_t nbytes,
                              StreamHandle stream, bool wait, const RestoreOptions& ro) {
    NvtxRange nvtx_("ofld.restore");
    Impl& D = *d_;
    RestoreOutcome out;
    std::vector<uint64_t> expect;
    uint32_t zmax = 0;
    {
        std::lock_guard<std::mutex> g(D.tab_mu);
        auto it = D.tensors.find({tensor_id, version});
        if (it != D.tensors.end()) {
            if (ro.verify) expect = it->second.digests;
            it->second.restored = false;
            zmax = it->second.zmax;
        }
    }
    RequestPrefetchRequest pr;
    pr.rank_id = D.opt.rank_id;
    pr.rank_epoch = D.epoch;
    pr.tensor_id = tensor_id;
    pr.version = version;
    pr.nbytes = nbytes;
    pr.gpu_id = D.gpu ? uint32_t(D.opt.device) : 0;
    pr.numa_node = uint32_t(D.numa);
    pr.flags = D.opt.fast_submit ? OFLD_FLAG_SUBMIT_ON_READY : 0;
    RequestPrefetchResponse r = D.call<Op::kRequestPrefetch>(pr);
    const uint64_t deadline = mono_ns() + 600ull * 1000000000ull;
    while (r.ok && !r.ready) {
        if (mono_ns() > deadline) {
            out.message = "restore: readback timed out";
            return out;
        }
        sleep_us(D.opt.prefetch_poll_us);
        r = D.call<Op::kRequestPrefetch>(pr);
    }
    if (!r.ok) {
        out.message = r.message;
        return out;
    }
    const uint64_t src_bytes = r.nbytes ? r.nbytes : nbytes;
    uint32_t st = r.slot_id < D.num_slots ? D.slots[r.slot_id].state.load(std::memory_order_acquire) : 0;
    bool submitted = r.state == OFLD_SLOT_H2D_IN_FLIGHT;
    if (!(st == OFLD_SLOT_PINNED_VALID || (submitted && st == OFLD_SLOT_H2D_IN_FLIGHT))) {
        out.message = "restore: slot not readable at H2D time";
        return out;
    }
    if (ro.cast == 0 && src_bytes != nbytes) {
        out.message = "restore: destination size " + std::to_string(nbytes) + " != offloaded size " +
                      std::to_string(src_bytes);
        return out;
    }
    char *host = nullptr, *dev = nullptr;
    D.resolve(r.arena_id, r.arena_offset, src_bytes, &host, &dev);
    if (!submitted) {
        TransferMark m{D.opt.rank_id, D.epoch, r.lease_id, tensor_id, r.version, r.slot_id, 0, real_ns()};
        StatusResponse sr = D.call<Op::kMarkH2DSubmitted>(m);
        if (!sr.ok) {
            out.message = "MarkH2DSubmitted: " + sr.message;
            return out;
        }
    }
    ++D.restores;
    Impl::Pending p;
    p.d2h = false;
    p.lease = r.lease_id;
    p.tid = tensor_id;
    p.ver = r.version ? r.version : version;
    p.slot = r.slot_id;
    p.nbytes = src_bytes;
    p.keep_pinned = ro.keep_pinned;
    D.inflight_h2d += src_bytes;
    uint32_t* mism_dev = nullptr;
    const bool z = D.run_is_z(r.slot_id);
    const bool zf = D.run_is_zf32(r.slot_id);
    if (!D.gpu) {
        if (ro.cast != 0) {
            out.message = "casts need a GPU";
            return out;
        }
        if (z || zf) {
            const bool okd = z ? zbf16::decode_object(reinterpret_cast<const uint8_t*>(host), src_bytes,
                                                      reinterpret_cast<uint8_t*>(ptr))
                               : zf32::decode_object(reinterpret_cast<const uint8_t*>(host), src_bytes,
                                                     reinterpret_cast<uint8_t*>(ptr));
            if (!okd) {
                out.message = z ? "malformed zbf16 object" : "malformed zf32 object";
                D.finish(p);
                return out;
            }
            if (ro.verify && !expect.empty()) {  // digests are of the decoded bytes
                std::vector<uint64_t> got(kern::digest_count(src_bytes));
                ssh::host_chunk_digests(reinterpret_cast<const char*>(ptr), src_bytes, got.data());
                for (size_t i = 0; i < got.size() && i < expect.size(); ++i)
                    out.mismatched_chunks += got[i] != expect[i];
            }
            D.finish(p);
            out.ok = out.mismatched_chunks == 0;
            out.message = out.ok ? "ok" : "content digest mismatch";
            return out;
        } else {
            std::memcpy(reinterpret_cast<void*>(ptr), host, src_bytes);
        }
        if (ro.verify && !expect.empty()) {
            std::vector<uint64_t> got(kern::digest_count(src_bytes));
            ssh::host_chunk_digests(host, src_bytes, got.data());
            for (size_t i = 0; i < got.size() && i < expect.size(); ++i) out.mismatched_chunks += got[i] != expect[i];
        }
        D.finish(p);
        out.ok = out.mismatched_chunks == 0;
        out.message = out.ok ? "ok" : "content digest mismatch";
        return out;
    }
    cudaStream_t s = D.stream_of(stream);
    const uint64_t* exp_dev = nullptr;
    if (ro.verify && !expect.empty()) {
        p.exp = D.pool.get(expect.size() * 8);  // returned to the pool when the copy retires
        std::memcpy(p.exp.host, expect.data(), expect.size() * 8);
        exp_dev = static_cast<const uint64_t*>(p.exp.dev);
        p.mism = D.pool.get(64);
        std::memset(p.mism.host, 0, 4);
        mism_dev = static_cast<uint32_t*>(p.mism.dev);
    }
    if (zf) {
        // zf32: decode into the destination (through the staging ring when
        // the run's largest coded row is known) or, for a cast, into a
        // temporary fp32 copy that K2 then casts (and verifies)
        const bool ce = D.opt.coded_restore == "copy_engine" && zmax > 0 &&
                        (reinterpret_cast<uintptr_t>(host) & 15) == 0;
        void* tmp = nullptr;
        uint8_t* into = reinterpret_cast<uint8_t*>(ptr);
        if (ro.cast != 0 || (ptr & 15) != 0) {  // the decoders write 16-byte aligned vectors
            CUDA_OK(cudaMallocAsync(&tmp, src_bytes, s));
            into = static_cast<uint8_t*>(tmp);
        }
        if (ce)
            D.restore_zf32_ce(host, into, src_bytes, zmax, s);
        else
            CUDA_OK(kern::restore_zf32(dev, into, src_bytes, s, D.opt.restore_ctas));
        if (tmp && ro.cast != 0) {
            CUDA_OK(kern::restore_cast(tmp, reinterpret_cast<void*>(ptr), src_bytes, kern::Cast(ro.cast),
                                       reinterpret_cast<float*>(ro.scales_ptr), exp_dev, mism_dev, s,
                                       D.opt.restore_ctas));
            CUDA_OK(cudaFreeAsync(tmp, s));
            exp_dev = nullptr;  // verified by the cast's pass
        } else if (tmp) {
            CUDA_OK(cudaMemcpyAsync(reinterpret_cast<void*>(ptr), tmp, src_bytes, cudaMemcpyDeviceToDevice, s));
            CUDA_OK(cudaFreeAsync(tmp, s));
        }
        if (exp_dev) {
            const uint64_t nd = kern::digest_count(src_bytes);
            p.dig = D.pool.get(nd * 8);
            CUDA_OK(kern::hash_device(reinterpret_cast<const void*>(ptr), src_bytes, static_cast<uint64_t*>(p.dig.dev),
                                      s, D.opt.hash_ctas));
            CUDA_OK(kern::compare_digests(static_cast<const uint64_t*>(p.dig.dev), exp_dev, nd, mism_dev, s));
        }
    } else if (z && D.opt.coded_restore == "copy_engine" && ro.cast == 0 && !exp_dev && zmax > 0 &&
        (reinterpret_cast<uintptr_t>(host) & 15) == 0 && (ptr & 15) == 0) {
        D.restore_z_ce(host, reinterpret_cast<uint8_t*>(ptr), src_bytes, zmax, s);
    } else if (z) {
        CUDA_OK(kern::restore_z(dev, reinterpret_cast<void*>(ptr), src_bytes, kern::Cast(ro.cast),
                                reinterpret_cast<float*>(ro.scales_ptr), exp_dev, mism_dev, s, D.opt.restore_ctas));
    } else if ((D.opt.engine == "copy_engine" || D.opt.uncoded == "copy_engine") && ro.cast == 0 && !exp_dev) {
        CUDA_OK(cudaMemcpyAsync(reinterpret_cast<void*>(ptr), host, src_bytes, cudaMemcpyHostToDevice, s));
    } else if (D.opt.uncoded == "bulk" && ro.cast == 0 && !exp_dev &&
               kern::bulk_ok(dev, reinterpret_cast<void*>(ptr), src_bytes)) {
        p.err = D.pool.get(16);
        *static_cast<volatile uint32_t*>(p.err.host) = 0;
        CUDA_OK(kern::restore_bulk(dev, reinterpret_cast<void*>(ptr), src_bytes, static_cast<uint32_t*>(p.err.dev), s,
                                   D.opt.restore_ctas));
    } else {
        CUDA_OK(kern::restore_cast(dev, reinterpret_cast<void*>(ptr), src_bytes, kern::Cast(ro.cast),
                                   reinterpret_cast<float*>(ro.scales_ptr), exp_dev, mism_dev, s, D.opt.restore_ctas));
    }
    CUDA_OK(cudaEventCreateWithFlags(&p.ev, cudaEventDisableTiming));
    CUDA_OK(cudaEventRecord(p.ev, s));
    if (wait) {
        CUDA_OK(cudaEventSynchronize(p.ev));
        if (mism_dev) out.mismatched_chunks = *static_cast<volatile uint32_t*>(p.mism.host);
        const bool dev_err = p.err.host && *static_cast<volatile uint32_t*>(p.err.host) != 0;
        D.finish(p);
        out.ok = out.mismatched_chunks == 0 && !dev_err;
        out.message = dev_err ? "restore: device copy incomplete (bounded wait expired)"
                              : out.ok ? "ok" : "content digest mismatch";
        return out;
    }
    D.complete_or_queue(std::move(p), false);
    out.ok = true;
    out.message = "ok";
    return out;
}

// Batched restore: prefetch requests and K2 launches go in groups of about
// batch_group_bytes (one round trip and one launch per group, the next
// group's round trip overlapping this group's copy). Items the daemon still
// has to read back from a cold tier are asked for again after the rest.
std::vector<RestoreOutcome> Agent::restore_batch(const std::vector<BatchItem>& items, StreamHandle stream, bool wait) {
    if (d_->opt.v1_only) {  // no batch opcodes: one restore per item
        std::vector<RestoreOutcome> out;
        out.reserve(items.size());
        for (const BatchItem& it : items)
            out.push_back(restore(it.tensor_id, it.version, it.ptr, it.nbytes, stream, wait, RestoreOptions{}));
        return out;
    }
    NvtxRange nvtx_("ofld.restore_batch");
    Impl& D = *d_;
    std::vector<RestoreOutcome> out(items.size());
    std::vector<RequestPrefetchRequest> reqs;
    for (const BatchItem& it : items) {
        RequestPrefetchRequest pr;
        pr.tensor_id = it.tensor_id;
        pr.version = it.version;
        pr.nbytes = it.nbytes;
        pr.gpu_id = D.gpu ? uint32_t(D.opt.device) : 0;
        pr.numa_node = uint32_t(D.numa);
        pr.flags = OFLD_FLAG_SUBMIT_ON_READY;
        reqs.push_back(pr);
    }
    std::vector<size_t> pending(items.size());
    for (size_t i = 0; i < items.size(); ++i) pending[i] = i;
    cudaStream_t s = D.stream_of(stream);
    std::vector<Impl::Pending> launched;
    cudaEvent_t last_ev = nullptr;
    const uint64_t deadline = mono_ns() + 600ull * 1000000000ull;
    const uint64_t group_bytes = std::max<uint64_t>(D.opt.batch_group_bytes, 1);
    while (!pending.empty()) {
        std::vector<size_t> again;
        for (size_t g0 = 0; g0 < pending.size();) {
            size_t g1 = g0;
            uint64_t bytes = 0;
            while (g1 < pending.size() && (g1 == g0 || bytes < group_bytes)) bytes += items[pending[g1++]].nbytes;
            BatchRequestPrefetchRequest q;
            q.rank_id = D.opt.rank_id;
            q.rank_epoch = D.epoch;
            for (size_t k = g0; k < g1; ++k) q.items.push_back(reqs[pending[k]]);
            BatchRequestPrefetchResponse resp = D.call<Op::kBatchRequestPrefetch>(q);
            std::vector<kern::XferJob> jobs;  // this group's ready items, one K2 launch
            const size_t first = launched.size();
            uint64_t total_chunks = 0;
            for (size_t k = g0; k < g1; ++k) {
                const size_t i = pending[k];
                if (k - g0 >= resp.results.size()) {
                    out[i].message = resp.message.empty() ? "no prefetch result" : resp.message;
                    continue;
                }
                const RequestPrefetchResponse& r = resp.results[k - g0];
                if (!r.ok) {
                    out[i].message = r.message;
                    continue;
                }
                if (!r.ready) {
                    again.push_back(i);
                    continue;
                }
                char *host = nullptr, *dev = nullptr;
                D.resolve(r.arena_id, r.arena_offset, r.nbytes, &host, &dev);
                Impl::Pending p;
                p.d2h = false;
                p.lease = r.lease_id;
                p.tid = items[i].tensor_id;
                p.ver = r.version;
                p.slot = r.slot_id;
                p.nbytes = r.nbytes;
                D.inflight_h2d += p.nbytes;
                ++D.restores;
                const bool z = D.run_is_z(r.slot_id);
                const bool zf = D.run_is_zf32(r.slot_id);
                if (zf) {  // a zf32 run (evicted singly): its own decode
                    if (D.gpu) {
                        CUDA_OK(kern::restore_zf32(dev, reinterpret_cast<void*>(items[i].ptr), r.nbytes, s,
                                                   D.opt.restore_ctas));
                        CUDA_OK(cudaEventCreateWithFlags(&p.ev, cudaEventDisableTiming));
                        CUDA_OK(cudaEventRecord(p.ev, s));
                        last_ev = p.ev;
                    } else if (!zf32::decode_object(reinterpret_cast<const uint8_t*>(host), r.nbytes,
                                                    reinterpret_cast<uint8_t*>(items[i].ptr))) {
                        out[i].message = "malformed zf32 object";
                        D.finish(p);
                        continue;
                    }
                } else if (D.batch_kernel_ok(items[i].ptr, r.nbytes) && (z || D.opt.uncoded != "copy_engine")) {
                    // uncoded items (no digests to compute on restore) take the copy
                    // engine by default: 51.1 GB/s for 4 MiB KV blocks beside a
                    // training step, against 48.8 in the job kernel
                    kern::XferJob j{};
                    j.src = dev;
                    j.dst = reinterpret_cast<void*>(items[i].ptr);
                    j.nbytes = r.nbytes;
                    j.chunk_begin = total_chunks;
                    j.coded = z ? 1u : 0u;
                    total_chunks += kern::digest_count(r.nbytes);
                    jobs.push_back(j);
                } else if (D.gpu) {
                    if (z)
                        CUDA_OK(kern::restore_z(dev, reinterpret_cast<void*>(items[i].ptr), r.nbytes,
                                                kern::Cast::kNone, nullptr, nullptr, nullptr, s, D.opt.restore_ctas));
                    else if (D.opt.engine == "copy_engine" || D.opt.uncoded == "copy_engine")
                        CUDA_OK(cudaMemcpyAsync(reinterpret_cast<void*>(items[i].ptr), host, r.nbytes,
                                                cudaMemcpyHostToDevice, s));
                    else
                        CUDA_OK(kern::restore_cast(dev, reinterpret_cast<void*>(items[i].ptr), r.nbytes,
                                                   kern::Cast::kNone, nullptr, nullptr, nullptr, s,
                                                   D.opt.restore_ctas));
                    CUDA_OK(cudaEventCreateWithFlags(&p.ev, cudaEventDisableTiming));
                    CUDA_OK(cudaEventRecord(p.ev, s));
                    last_ev = p.ev;
                } else if (z) {
                    if (!zbf16::decode_object(reinterpret_cast<const uint8_t*>(host), r.nbytes,
                                              reinterpret_cast<uint8_t*>(items[i].ptr))) {
                        out[i].message = "malformed zbf16 object";
                        D.finish(p);
                        continue;
                    }
                } else {
                    std::memcpy(reinterpret_cast<void*>(items[i].ptr), host, r.nbytes);
                }
                out[i].ok = true;
                out[i].message = "ok";
                launched.push_back(std::move(p));
            }
            if (!jobs.empty()) {
                PinnedPool::Buf tab = D.pool.get(jobs.size() * sizeof(kern::XferJob));
                std::memcpy(tab.host, jobs.data(), jobs.size() * sizeof(kern::XferJob));
                CUDA_OK(kern::restore_jobs(static_cast<const kern::XferJob*>(tab.dev), int(jobs.size()), total_chunks,
                                           s, D.opt.restore_ctas));
                cudaEvent_t ev;
                CUDA_OK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
                CUDA_OK(cudaEventRecord(ev, s));
                auto keep = D.make_batch_keep(ev, tab);
                for (size_t k = first; k < launched.size(); ++k)
                    if (!launched[k].ev) {
                        launched[k].ev = ev;
                        launched[k].batch_keep = keep;
                    }
                last_ev = ev;
            }
            g0 = g1;
        }
        pending.swap(again);
        if (!pending.empty()) {
            // Items still waiting (readback in flight, or no pinned run free for
            // one) may need the runs this batch holds: hand on the completions
            // of what was launched first, so its prefetch leases return to the
            // daemon before we ask again.
            if (D.gpu && last_ev) CUDA_OK(cudaEventSynchronize(last_ev));
            for (Impl::Pending& p : launched) D.finish(p);
            launched.clear();
            last_ev = nullptr;
            if (mono_ns() > deadline) {
                for (size_t i : pending) out[i].message = "readback timed out";
                break;
            }
            sleep_us(D.opt.prefetch_poll_us);
        }
    }
    if (wait && D.gpu && last_ev) CUDA_OK(cudaEventSynchronize(last_ev));
    for (Impl::Pending& p : launched) {
        if (!D.gpu || wait)
            D.finish(p);
        else
            D.complete_or_queue(std::move(p), false);
    }
    return out;
}

bool Agent::is_offloaded(uint64_t tid, uint64_t ver) const {
    std::lock_guard<std::mutex> g(d_->tab_mu);
    auto it = d_->tensors.find({tid, ver});
    return it != d_->tensors.end() && it->second.offloaded;
}

void Agent::wait_offloaded(uint64_t tid, uint64_t ver) {
    std::unique_lock<std::mutex> g(d_->tab_mu);
    d_->tab_cv.wait(g, [&] {
        auto it = d_->tensors.find({tid, ver});
        return it == d_->tensors.end() || it->second.offloaded;
    });
}

bool Agent::is_restored(uint64_t tid, uint64_t ver) const {
    std::lock_guard<std::mutex> g(d_->tab_mu);
    auto it = d_->tensors.find({tid, ver});
    return it != d_->tensors.end() && it->second.restored;
}

void Agent::wait_restored(uint64_t tid, uint64_t ver) {
    std::unique_lock<std::mutex> g(d_->tab_mu);
    d_->tab_cv.wait(g, [&] {
        auto it = d_->tensors.find({tid, ver});
        return it == d_->tensors.end() || it->second.restored;
    });
}

bool Agent::tensor_hash(uint64_t tid, uint64_t ver, uint64_t* lo, uint64_t* hi) const {
    std::lock_guard<std::mutex> g(d_->tab_mu);
    auto it = d_->tensors.find({tid, ver});
    if (it == d_->tensors.end() || !it->second.offloaded) return false;
    *lo = it->second.hash_lo;
    *hi = it->second.hash_hi;
    return true;
}

std::string Agent::location(uint64_t tid, uint64_t ver) {
    LocationQueryResponse r = d_->call<Op::kQueryLocation>(LocationQueryRequest{tid, ver});
    if (!r.ok) return "none";
    switch (r.location_kind) {
        case OFLD_LOC_GPU: return "gpu";
        case OFLD_LOC_PINNED: return "pinned";
        case OFLD_LOC_PAGEABLE: return "pageable";
        case OFLD_LOC_NVME: return "nvme";
        default: return "none";
    }
}

// A copy that a drain, readback or restore is moving cannot be dropped yet;
// the daemon answers "retry" and the call waits (bounded) for the transfer to
// settle, so a discard never leaves the tensor's pinned or cold copy behind.
void Agent::discard(uint64_t tid, uint64_t ver) {
    Impl& D = *d_;
    if (D.opt.v1_only) {
        // StateSpectre's discard: release the lease the evict was granted
        uint64_t lease = 0;
        uint32_t slot = 0;
        {
            std::lock_guard<std::mutex> g(D.tab_mu);
            auto it = D.tensors.find({tid, ver});
            if (it != D.tensors.end()) {
                lease = it->second.lease;
                slot = it->second.slot;
            }
        }
        if (lease) {
            StatusResponse s = D.call<Op::kReleaseLease>(ReleaseLeaseRequest{D.opt.rank_id, D.epoch, lease, slot,
                                                                              "discard"});
            if (!s.ok) LOG_WARN(TAG, "discard(%llu:%llu): %s", (unsigned long long)tid, (unsigned long long)ver,
                                s.message.c_str());
        }
        std::lock_guard<std::mutex> g(D.tab_mu);
        D.tensors.erase({tid, ver});
        D.tab_cv.notify_all();
        return;
    }
    DiscardTensorRequest r{D.opt.rank_id, D.epoch, tid, ver};
    StatusResponse s = D.call<Op::kDiscardTensor>(r);
    const uint64_t deadline = mono_ns() + 30ull * 1000000000ull;
    uint64_t backoff_us = 100;
    while (!s.ok && s.message.find("retry") != std::string::npos && mono_ns() < deadline) {
        sleep_us(backoff_us);
        backoff_us = std::min<uint64_t>(backoff_us * 2, 5000);
        s = D.call<Op::kDiscardTensor>(r);
    }
    if (!s.ok) LOG_WARN(TAG, "discard(%llu:%llu): %s", (unsigned long long)tid, (unsigned long long)ver, s.message.c_str());
    std::lock_guard<std::mutex> g(D.tab_mu);
    D.tensors.erase({tid, ver});
    D.tab_cv.notify_all();
}

void Agent::discard_batch(const std::vector<std::pair<uint64_t, uint64_t>>& items) {
    Impl& D = *d_;
    if (D.opt.v1_only) {
        for (const auto& tv : items) discard(tv.first, tv.second);
        return;
    }
    std::vector<std::pair<uint64_t, uint64_t>> todo = items;
    const uint64_t deadline = mono_ns() + 30ull * 1000000000ull;
    uint64_t backoff_us = 100;
    while (!todo.empty()) {
        BatchDiscardTensorRequest r;
        r.rank_id = D.opt.rank_id;
        r.rank_epoch = D.epoch;
        for (auto& tv : todo) r.items.push_back(TensorVersion{tv.first, tv.second});
        BatchDiscardTensorResponse resp = D.call<Op::kBatchDiscardTensor>(r);
        if (!resp.ok) {
            LOG_WARN(TAG, "discard_batch: %s", resp.message.c_str());
            break;
        }
        std::vector<std::pair<uint64_t, uint64_t>> again;
        for (size_t i = 0; i < todo.size() && i < resp.results.size(); ++i) {
            const StatusResponse& st = resp.results[i];
            if (!st.ok && st.message.find("retry") != std::string::npos && mono_ns() < deadline)
                again.push_back(todo[i]);
            else if (!st.ok)
                LOG_WARN(TAG, "discard(%llu:%llu): %s", (unsigned long long)todo[i].first,
                         (unsigned long long)todo[i].second, st.message.c_str());
        }
        todo.swap(again);
        if (!todo.empty()) {
            sleep_us(backoff_us);
            backoff_us = std::min<uint64_t>(backoff_us * 2, 5000);
        }
    }
    std::lock_guard<std::mutex> g(D.tab_mu);
    for (auto& tv : items) D.tensors.erase({tv.first, tv.second});
    D.tab_cv.notify_all();
}

void Agent::assert_no_inflight() const {
    std::lock_guard<std::mutex> g(d_->inflight_mu);
    if (!d_->inflight.empty())
        throw std::runtime_error("assert_no_inflight: " + std::to_string(d_->inflight.size()) + " transfers in flight");
}

void Agent::synchronize() {
    for (;;) {
        {
            std::lock_guard<std::mutex> g(d_->inflight_mu);
            if (d_->inflight.empty()) return;
        }
        sleep_us(50);
    }
}

// ---------------------------------------------------------------------------
// Canonical model state
// ---------------------------------------------------------------------------
RegisterJobResponse Agent::register_job(const RegisterJobRequest& r) { return d_->call<Op::kRegisterJob>(r); }

// A canonical evict in phases. request: the attach-or-create round trip
// (attach, wait and verify-only answers finish there). scan: for a create of
// a bf16 object, the zbf16 pre-pass decides whether the bytes cross PCIe
// coded. launch: the run's coding (SetRunFormat), the submitted mark and the
// copy (copy engine or K1, chunk digests of the raw bytes from the same
// pass). end: wait for the copy, fold the digests, mark it complete and
// commit. canonical_evict runs the phases in turn; canonical_evict_batch
// requests every item, scans every candidate with one stream wait, then
// launches and ends them, so each item's round trips overlap earlier copies.
struct Agent::CanonPending {
    CanonicalOutcome out;
    bool create = false;    // the daemon asked this rank to copy the object
    bool copying = false;   // launched, not yet ended
    bool zcand = false;     // a bf16 object that may cross PCIe coded
    bool z = false;         // the pre-pass found every chunk codable
    bool trusted = false;
    uint64_t ptr = 0, nbytes = 0;
    cudaStream_t s = nullptr;
    char *host = nullptr, *dev = nullptr;
    TransferMark mark{};
    RequestCanonicalEvictResponse resp;
    DoneCallback cb;
    bool destructive = false;
    PinnedPool::Buf zb;
    std::unique_ptr<Impl::Pending> p;
};

void Agent::canonical_request(CanonPending& c, uint64_t ptr, uint64_t nbytes, StreamHandle stream, bool destructive,
                              const RequestCanonicalEvictRequest& in, DoneCallback on_invalidate) {
    Impl& D = *d_;
    RequestCanonicalEvictRequest req = in;
    req.rank_id = D.opt.rank_id;
    req.rank_epoch = D.epoch;
    req.gpu_id = D.gpu ? uint32_t(D.opt.device) : 0;
    req.numa_node = uint32_t(D.numa);
    req.destructive = destructive;
    req.key.nbytes = nbytes;
    if (req.key.shard_nbytes == 0) req.key.shard_nbytes = nbytes;
    c.ptr = ptr;
    c.nbytes = nbytes;
    c.destructive = destructive;
    c.cb = std::move(on_invalidate);
    c.trusted = req.dedup_mode == offload_v2::DEDUP_SEMANTIC_TRUSTED || req.dedup_mode == offload_v2::DEDUP_DISABLED;
    c.resp = D.call<Op::kRequestCanonicalEvict>(req);
    const RequestCanonicalEvictResponse& resp = c.resp;
    CanonicalOutcome& out = c.out;
    out.action = resp.action;
    out.object_id = resp.object_id;
    out.message = resp.message;
    if (!resp.ok) return;
    c.s = D.stream_of(stream);

    const bool attached = resp.action == offload_v2::ATTACH_ACTION_ATTACHED_EXISTING ||
                          resp.action == 7 /* attached after a peer byte compare */;
    if (attached || resp.action == offload_v2::ATTACH_ACTION_WAIT_FOR_CREATOR) {
        out.ok = true;
        if (attached && destructive && c.cb) {
            if (D.gpu) CUDA_OK(cudaStreamSynchronize(c.s));  // producer kernels done before the storage goes
            c.cb();
        }
        return;
    }
    if (resp.action == 6 /* verify-hash-only */) {
        // Replica verification without a copy: hash the local GPU bytes.
        hash_buffer(ptr, nbytes, stream, &out.hash_lo, &out.hash_hi);
        CommitCanonicalObjectRequest cm;
        cm.rank_id = D.opt.rank_id;
        cm.rank_epoch = D.epoch;
        cm.object_id = resp.object_id;
        cm.lease_id = 0;
        cm.content_hash_lo = out.hash_lo;
        cm.content_hash_hi = out.hash_hi;
        CommitCanonicalObjectResponse cr = D.call<Op::kCommitCanonicalObject>(cm);
        out.ok = cr.ok;
        out.message = cr.message;
        if (cr.ok && destructive && c.cb) c.cb();
        return;
    }
    if (resp.action != offload_v2::ATTACH_ACTION_NEED_D2H_CREATE &&
        resp.action != offload_v2::ATTACH_ACTION_DUPLICATE_CANDIDATE)
        return;
    c.create = true;
    D.resolve(resp.arena_id, resp.arena_offset, nbytes, &c.host, &c.dev);
    c.zcand = D.opt.compress_canonical && req.key.dtype == kScalarBf16 && D.want_z(ptr, nbytes, kFmtBf16) &&
              (reinterpret_cast<uintptr_t>(c.host) & 15) == 0;
}

void Agent::canonical_launch(CanonPending& c) {
    Impl& D = *d_;
    if (!c.create) return;
    const RequestCanonicalEvictResponse& resp = c.resp;
    c.mark = TransferMark{D.opt.rank_id, D.epoch, resp.lease_id, resp.synthetic_tid, 1, resp.slot_id, 0, real_ns()};
    if (c.z) {
        SetRunFormatRequest f{D.opt.rank_id, D.epoch, resp.lease_id, resp.slot_id, OFLD_FLAG_FORMAT_ZBF16};
        StatusResponse fr = D.call<Op::kSetRunFormat>(f);
        if (!fr.ok) {  // a daemon that cannot record the coding gets the raw bytes
            LOG_WARN(TAG, "SetRunFormat: %s (object moves uncoded)", fr.message.c_str());
            D.pool.put(c.zb);
            c.zb = PinnedPool::Buf{};
            c.z = false;
        }
    }
    StatusResponse sr = D.call<Op::kMarkD2HSubmitted>(c.mark);
    if (!sr.ok) LOG_WARN(TAG, "canonical MarkD2HSubmitted: %s", sr.message.c_str());
    ++D.evicts;
    c.p.reset(new Impl::Pending());
    c.p->nbytes = c.nbytes;
    c.p->z = c.z;
    c.p->zb = c.zb;
    c.zb = PinnedPool::Buf{};
    D.launch_d2h(*c.p, c.ptr, c.host, c.dev, c.s, true);
    c.copying = true;
}

void Agent::canonical_end(CanonPending& c) {
    Impl& D = *d_;
    if (!c.copying) return;
    c.copying = false;
    Impl::Pending& p = *c.p;
    CanonicalOutcome& out = c.out;
    if (p.ev) CUDA_OK(cudaEventSynchronize(p.ev));
    if (p.ev) cudaEventDestroy(p.ev);
    p.ev = nullptr;
    Impl::host_digests(p);
    ssh::Object h{0, 0};
    if (p.dig.host) {
        h = ssh::fold_digests(static_cast<const uint64_t*>(p.dig.host), p.ndig, c.nbytes);
        if (D.gpu)
            D.pool.put(p.dig);
        else
            std::free(p.dig.host);
        p.dig = {};
    }
    D.pool.put(p.zb);
    p.zb = PinnedPool::Buf{};
    D.d2h_bytes += c.nbytes;
    ++D.d2h_done;
    if (c.z) ++D.coded_canonical;
    MarkD2HCompleteResponse dr = D.call<Op::kMarkD2HComplete>(c.mark);
    if (!dr.ok) {
        out.message = "canonical MarkD2HComplete rejected";
        return;
    }
    CommitCanonicalObjectRequest cm;
    cm.rank_id = D.opt.rank_id;
    cm.rank_epoch = D.epoch;
    cm.object_id = c.resp.object_id;
    cm.lease_id = c.resp.lease_id;
    cm.slot_id = c.resp.slot_id;
    if (!(c.trusted && D.opt.zero_canonical_hash)) {
        cm.content_hash_lo = h.lo;
        cm.content_hash_hi = h.hi;
    }
    CommitCanonicalObjectResponse cr = D.call<Op::kCommitCanonicalObject>(cm);
    out.ok = cr.ok;
    out.did_d2h = true;
    out.message = cr.message;
    out.hash_lo = h.lo;
    out.hash_hi = h.hi;
    if (cr.ok && c.destructive && c.cb) c.cb();
}

// The pre-pass of every coding candidate among `cs`: all launched on their
// streams, then one wait per distinct stream (a stream's wait also covers the
// producers of its objects, as the copies that follow must).
void Agent::canonical_scan(std::vector<CanonPending*>& cs) {
    Impl& D = *d_;
    std::vector<cudaStream_t> streams;
    for (CanonPending* c : cs) {
        if (!c->zcand) continue;
        D.zscan_launch(c->ptr, c->nbytes, c->s, &c->zb);
        if (std::find(streams.begin(), streams.end(), c->s) == streams.end()) streams.push_back(c->s);
    }
    for (cudaStream_t s : streams) D.stream_wait(s);
    for (CanonPending* c : cs)
        if (c->zcand) c->z = D.zscan_result(c->nbytes, &c->zb);
}

CanonicalOutcome Agent::canonical_evict(uint64_t ptr, uint64_t nbytes, StreamHandle stream, bool destructive,
                                        const RequestCanonicalEvictRequest& in, DoneCallback on_invalidate, bool) {
    NvtxRange nvtx_("ofld.canonical_evict");
    CanonPending c;
    canonical_request(c, ptr, nbytes, stream, destructive, in, std::move(on_invalidate));
    std::vector<CanonPending*> one{&c};
    canonical_scan(one);
    canonical_launch(c);
    canonical_end(c);
    return c.out;
}

// Many canonical evicts on one stream: every item's attach-or-create round
// trip, then one pre-pass wait for the coding candidates, then the copies
// back to back while the host marks and commits the earlier items. At most
// `max_inflight_bytes` of copies are outstanding (0: no limit); beyond it the
// oldest item is ended before the next is launched.
std::vector<CanonicalOutcome> Agent::canonical_evict_batch(const std::vector<CanonicalItem>& items,
                                                           StreamHandle stream, bool destructive,
                                                           uint64_t max_inflight_bytes) {
    NvtxRange nvtx_("ofld.canonical_evict_batch");
    std::vector<CanonPending> cs(items.size());
    for (size_t i = 0; i < items.size(); ++i)
        canonical_request(cs[i], items[i].ptr, items[i].nbytes, stream, destructive, items[i].req,
                          items[i].on_invalidate);
    std::vector<CanonPending*> all;
    for (CanonPending& c : cs) all.push_back(&c);
    canonical_scan(all);
    size_t done = 0;
    uint64_t inflight = 0;
    for (size_t i = 0; i < cs.size(); ++i) {
        while (max_inflight_bytes && inflight > 0 && inflight + cs[i].nbytes > max_inflight_bytes && done < i) {
            if (cs[done].copying) inflight -= cs[done].nbytes;
            canonical_end(cs[done++]);
        }
        canonical_launch(cs[i]);
        if (cs[i].copying) inflight += cs[i].nbytes;
    }
    for (; done < cs.size(); ++done) canonical_end(cs[done]);
    std::vector<CanonicalOutcome> out;
    out.reserve(cs.size());
    for (CanonPending& c : cs) out.push_back(std::move(c.out));
    return out;
}

RestoreOutcome Agent::canonical_restore(uint64_t object_id, uint64_t ptr, uint64_t nbytes, StreamHandle stream,
                                        bool wait, const RestoreOptions& ro) {
    Impl& D = *d_;
    RestoreOutcome out;
    RequestCanonicalRestoreRequest rq{D.opt.rank_id, D.epoch, object_id, D.gpu ? uint32_t(D.opt.device) : 0,
                                      uint32_t(D.numa)};
    RequestCanonicalRestoreResponse rr;
    const uint64_t deadline = mono_ns() + 600ull * 1000000000ull;
    for (;;) {
        rr = D.call<Op::kRequestCanonicalRestore>(rq);
        if (rr.ok || !rr.retriable) break;
        if (mono_ns() > deadline) {
            out.message = "canonical_restore: object stuck transitioning";
            return out;
        }
        sleep_us(D.opt.prefetch_poll_us);
    }
    if (!rr.ok) {
        out.message = rr.message;
        return out;
    }
    auto release = [&] {
        try {
            D.call<Op::kReleaseCanonicalRestore>(ReleaseCanonicalRestoreRequest{D.opt.rank_id, D.epoch, object_id});
        } catch (...) {
        }
    };
    if (ro.cast == 0 && nbytes > rr.nbytes) {
        release();
        out.message = "canonical_restore: destination larger than object";
        return out;
    }
    try {
        char *host = nullptr, *dev = nullptr;
        D.resolve(rr.arena_id, rr.arena_offset, rr.nbytes, &host, &dev);
        ++D.restores;
        uint64_t n = ro.cast == 0 ? nbytes : rr.nbytes;
        const int64_t slot = D.slot_at(rr.arena_id, rr.arena_offset);
        const bool coded = slot >= 0 && D.run_is_z(uint32_t(slot));
        if (!D.gpu && coded) {
            // a host-mode consumer of an object a GPU rank stored coded
            if (ro.cast != 0) throw std::runtime_error("host-mode restore of a coded object cannot cast");
            if (n != rr.nbytes && n % zbf16::kChunk)
                throw std::runtime_error("partial restore of a coded object must be a multiple of 64 KiB");
            std::vector<uint32_t> keys;
            if (!zbf16::decode_range(zbf16::Coding::kZbf16, reinterpret_cast<const uint8_t*>(host), rr.nbytes, 0, n,
                                     reinterpret_cast<uint8_t*>(ptr), keys))
                throw std::runtime_error("malformed coded object");
        } else if (!D.gpu) {
            std::memcpy(reinterpret_cast<void*>(ptr), host, n);
        } else if (coded) {
            // zbf16 run: K2 decodes from host memory. A prefix of the object
            // decodes on its own only at a chunk boundary.
            if (n != rr.nbytes && n % zbf16::kChunk)
                throw std::runtime_error("partial restore of a coded object must be a multiple of 64 KiB");
            if ((ptr & 15) || !zbf16::eligible(n)) throw std::runtime_error("coded object: destination not 16-byte aligned");
            cudaStream_t s = D.stream_of(stream);
            CUDA_OK(kern::restore_z(dev, reinterpret_cast<void*>(ptr), n, kern::Cast(ro.cast),
                                    reinterpret_cast<float*>(ro.scales_ptr), nullptr, nullptr, s, D.opt.restore_ctas));
            CUDA_OK(cudaStreamSynchronize(s));
        } else {
            cudaStream_t s = D.stream_of(stream);
            CUDA_OK(kern::restore_cast(dev, reinterpret_cast<void*>(ptr), n, kern::Cast(ro.cast),
                                       reinterpret_cast<float*>(ro.scales_ptr), nullptr, nullptr, s,
                                       D.opt.restore_ctas));
            // The hold is released only after the copy finished reading.
            CUDA_OK(cudaStreamSynchronize(s));
        }
        D.h2d_bytes += n;
        ++D.h2d_done;
        out.ok = true;
        out.message = "ok";
    } catch (const std::exception& e) {
        out.message = std::string("canonical_restore: ") + e.what();
    }
    release();
    (void)wait;
    return out;
}

SealModelVersionResponse Agent::seal(const SealModelVersionRequest& r) { return d_->call<Op::kSealModelVersion>(r); }
GetLatestSealedVersionResponse Agent::latest(const GetLatestSealedVersionRequest& r) {
    return d_->call<Op::kGetLatestSealedVersion>(r);
}
GetManifestResponse Agent::manifest(const GetManifestRequest& r) { return d_->call<Op::kGetManifest>(r); }
PullTensorResponse Agent::pull(const PullTensorRequest& r) { return d_->call<Op::kPullTensor>(r); }
DropCanonicalVersionResponse Agent::drop_version(const DropCanonicalVersionRequest& r) {
    return d_->call<Op::kDropCanonicalVersion>(r);
}
ReleaseCanonicalResponse Agent::release(const ReleaseCanonicalRequest& in) {
    ReleaseCanonicalRequest r = in;
    r.rank_id = d_->opt.rank_id;
    r.rank_epoch = d_->epoch;
    return d_->call<Op::kReleaseCanonical>(r);
}
CarryForwardResponse Agent::carry_forward(const CarryForwardRequest& in) {
    d_->need_ext("carry_forward");
    CarryForwardRequest r = in;
    r.rank_id = d_->opt.rank_id;
    r.rank_epoch = d_->epoch;
    return d_->call<Op::kCarryForward>(r);
}
ExportManifestResponse Agent::export_manifest(const ExportManifestRequest& r) {
    d_->need_ext("export_manifest");
    return d_->call<Op::kExportManifest>(r);
}
GetJobStatsResponse Agent::job_stats(const GetJobStatsRequest& r) {
    d_->need_ext("job_stats");
    return d_->call<Op::kGetJobStats>(r);
}
GetStatsResponse Agent::daemon_stats() { return d_->call<Op::kGetStats>(GetStatsRequest{}); }

StatusResponse Agent::publish_peer_buffer(const PeerBufferDesc& desc, int fd) {
    d_->need_ext("publish_peer_buffer");
    PublishPeerBufferRequest r;
    r.rank_id = d_->opt.rank_id;
    r.rank_epoch = d_->epoch;
    r.desc = desc;
    ++d_->rpc_count;
    std::vector<int> fds;
    if (fd >= 0) fds.push_back(fd);
    return d_->rpc->call<Op::kPublishPeerBuffer>(r, nullptr, fds);
}

LookupPeerBufferResponse Agent::lookup_peer_buffer(const std::string& key, uint32_t wait_ms, int* fd_out) {
    d_->need_ext("lookup_peer_buffer");
    ++d_->rpc_count;
    std::vector<int> fds;
    LookupPeerBufferResponse r = d_->rpc->call<Op::kLookupPeerBuffer>(LookupPeerBufferRequest{key, wait_ms}, &fds);
    if (fd_out) *fd_out = fds.empty() ? -1 : fds[0];
    for (size_t i = fd_out ? 1 : 0; i < fds.size(); ++i) ::close(fds[i]);
    return r;
}

void Agent::hash_buffer(uint64_t ptr, uint64_t nbytes, StreamHandle stream, uint64_t* lo, uint64_t* hi) {
    Impl& D = *d_;
    if (!D.gpu) {
        ssh::Object o = ssh::host_hash(reinterpret_cast<const void*>(ptr), nbytes);
        *lo = o.lo;
        *hi = o.hi;
        return;
    }
    uint64_t n = kern::digest_count(nbytes);
    PinnedPool::Buf b = D.pool.get(std::max<uint64_t>(n, 1) * 8);
    cudaStream_t s = D.stream_of(stream);
    CUDA_OK(kern::hash_device(reinterpret_cast<const void*>(ptr), nbytes, static_cast<uint64_t*>(b.dev), s,
                              D.opt.hash_ctas));
    CUDA_OK(cudaStreamSynchronize(s));
    ssh::Object o = ssh::fold_digests(static_cast<const uint64_t*>(b.host), n, nbytes);
    D.pool.put(b);
    *lo = o.lo;
    *hi = o.hi;
}

uint64_t Agent::map_arena(uint64_t arena_id, uint64_t offset) const {
    for (const Impl::ArenaMap& m : d_->arenas)
        if (m.id == arena_id) return reinterpret_cast<uint64_t>(m.base + offset);
    return 0;
}

AgentStats Agent::stats() const {
    const Impl& D = *d_;
    AgentStats s;
    s.rank_id = D.opt.rank_id;
    s.gpu_id = D.gpu ? D.opt.device : -1;
    s.numa_node = D.numa;
    s.registered_pinned_bytes = D.registered_bytes;
    s.inflight_d2h_bytes = D.inflight_d2h;
    s.inflight_h2d_bytes = D.inflight_h2d;
    s.evict_count = D.evicts;
    s.restore_count = D.restores;
    s.d2h_completed = D.d2h_done;
    s.h2d_completed = D.h2d_done;
    s.rank_epoch = D.epoch;
    s.num_slots = D.num_slots;
    s.d2h_bytes = D.d2h_bytes;
    s.h2d_bytes = D.h2d_bytes;
    s.kernel_launches = D.gpu ? kern::launch_count() : 0;
    s.rpc_count = D.rpc_count;
    s.d2h_ns = D.d2h_ns;
    s.h2d_ns = D.h2d_ns;
    s.registration_ns = D.reg_ns;
    s.coded_canonical = D.coded_canonical;
    return s;
}

std::string Agent::summary_string() const {
    AgentStats s = stats();
    char buf[768];
    std::snprintf(buf, sizeof(buf),
                  "Agent rank=%u gpu=%d numa=%d epoch=%llu\n"
                  "  registered_pinned_bytes=%llu\n"
                  "  inflight: d2h=%llu bytes  h2d=%llu bytes\n"
                  "  counts: evict=%llu restore=%llu d2h_done=%llu h2d_done=%llu\n"
                  "  bytes: d2h=%llu h2d=%llu  kernel_launches=%llu rpcs=%llu\n"
                  "  slots=%llu",
                  s.rank_id, s.gpu_id, s.numa_node, (unsigned long long)s.rank_epoch,
                  (unsigned long long)s.registered_pinned_bytes, (unsigned long long)s.inflight_d2h_bytes,
                  (unsigned long long)s.inflight_h2d_bytes, (unsigned long long)s.evict_count,
                  (unsigned long long)s.restore_count, (unsigned long long)s.d2h_completed,
                  (unsigned long long)s.h2d_completed, (unsigned long long)s.d2h_bytes,
                  (unsigned long long)s.h2d_bytes, (unsigned long long)s.kernel_launches,
                  (unsigned long long)s.rpc_count, (unsigned long long)s.num_slots);
    return buf;
}

int Agent::device() const { return d_->gpu ? d_->opt.device : -1; }
int Agent::numa_node() const { return d_->numa; }
uint32_t Agent::rank_id() const { return d_->opt.rank_id; }
uint64_t Agent::rank_epoch() const { return d_->epoch; }
void Agent::pause_heartbeat(bool paused) { d_->hb_paused.store(paused); }

}  // namespace ofld
