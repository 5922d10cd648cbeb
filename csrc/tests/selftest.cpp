// ofld_selftest: native unit tests of the pieces every process shares (wire
// codec and framing, config parser, control-region layout, completion ring,
// ssh128 hash, zbf16 codec). No GPU, no daemon. Exit status 0 when every
// check passes; each failure prints file:line and the expression.
//
//   statespectre_b200/bin/ofld_selftest [filter]
#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "../daemon/config.h"
#include "ofld/chunk_hash.h"
#include "ofld/codec.h"
#include "ofld/protocol.h"
#include "ofld/shm.h"
#include "ofld/zbf16.h"

namespace {

int g_checks = 0, g_failed = 0;

#define CHECK(cond)                                                                   \
    do {                                                                              \
        ++g_checks;                                                                   \
        if (!(cond)) {                                                                \
            ++g_failed;                                                               \
            std::fprintf(stderr, "  FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond);    \
        }                                                                             \
    } while (0)

#define CHECK_THROWS(expr)                                                            \
    do {                                                                              \
        bool threw = false;                                                           \
        try {                                                                         \
            expr;                                                                     \
        } catch (const std::exception&) {                                             \
            threw = true;                                                             \
        }                                                                             \
        CHECK(threw);                                                                 \
    } while (0)

struct Case {
    const char* name;
    std::function<void()> fn;
};

using namespace ofld;

void codec_round_trips() {
    RequestOffloadRequest r;
    r.rank_id = 7;
    r.rank_epoch = 3;
    r.tensor_id = 0x123456789ull;
    r.version = 2;
    r.nbytes = 1ull << 33;
    r.flags = OFLD_FLAG_DESTRUCTIVE | OFLD_FLAG_FORMAT_ZBF16;
    r.debug_name = "layers.0.mlp";
    auto b = encode(r);
    auto r2 = decode<RequestOffloadRequest>(b);
    CHECK(r2.rank_id == 7 && r2.tensor_id == r.tensor_id && r2.nbytes == r.nbytes && r2.flags == r.flags);
    CHECK(r2.debug_name == "layers.0.mlp");

    GetManifestResponse m;
    m.ok = true;
    m.message = "ok";
    m.model_version = 9;
    for (int i = 0; i < 3; ++i) {
        TensorManifestEntryWire e;
        e.object_id = 100 + i;
        e.nbytes = 4096u * (i + 1);
        e.key.param_fqn_debug = "w" + std::to_string(i);
        e.key.expert_id = -1;
        m.tensors.push_back(e);
    }
    auto m2 = decode<GetManifestResponse>(encode(m));
    CHECK(m2.tensors.size() == 3 && m2.tensors[2].object_id == 102 && m2.tensors[1].key.param_fqn_debug == "w1");
    CHECK(m2.tensors[0].key.expert_id == -1);
}

void codec_rejects_truncation() {
    RegisterJobRequest r;
    r.job_name = "trainer";
    r.label_keys = {"a", "b"};
    r.label_values = {"1", "2"};
    auto b = encode(r);
    for (size_t cut : {size_t(1), b.size() / 2, b.size() - 1}) {
        std::vector<uint8_t> t(b.begin(), b.begin() + long(cut));
        CHECK_THROWS(decode<RegisterJobRequest>(t));
    }
}

void framing() {
    std::vector<uint8_t> body = {1, 2, 3, 4, 5};
    auto f = make_frame(Op::kGetStats, body, 0);
    FrameHeader h = parse_frame_header(f.data(), f.size());
    CHECK(h.opcode == uint16_t(Op::kGetStats) && h.payload_len == body.size());
    f[0] ^= 0xFF;
    CHECK_THROWS(parse_frame_header(f.data(), f.size()));
    CHECK_THROWS(parse_frame_header(f.data(), 3));
}

void config_parse() {
    const std::string y =
        "daemon:\n  socket_path: /tmp/x.sock\n  heartbeat_timeout_ms: 1234\n"
        "arenas:\n  allocation_granularity_mb: 2\n  per_numa:\n    - numa_node: 0\n      size_gb: 4\n"
        "      gpu_windows:\n        - gpu: 0\n          size_gb: 2\n      overflow_gb: 1\n"
        "manifest:\n  retain_sealed_versions: 3\n";
    DaemonConfig c = parse_config(y);
    CHECK(c.socket_path == "/tmp/x.sock" && c.heartbeat_timeout_ms == 1234);
    CHECK(c.allocation_granularity_bytes == (2ull << 20) && c.per_numa.size() == 1);
    CHECK(c.v2_retain_sealed_versions == 3);
    CHECK_THROWS(parse_config("daemon:\n\tsocket_path: /x\n"));  // tabs
    CHECK(parse_size("512MiB") == (512ull << 20) && parse_size("4096") == 4096);
    CHECK_THROWS(parse_size("lots"));
}

void layout_and_ring() {
    ControlLayout L = control_layout(2, 1000, 8 * ring_stride_bytes(64));
    CHECK(L.arena_desc_offset % OFLD_CACHELINE == 0 && L.slot_entries_offset % OFLD_CACHELINE == 0);
    CHECK(L.arena_desc_offset < L.slot_entries_offset && L.slot_entries_offset < L.ring_offset);
    CHECK(L.ring_offset + L.ring_bytes <= L.total_bytes && L.total_bytes % 4096 == 0);

    std::vector<uint8_t> mem(ring_stride_bytes(8) + OFLD_CACHELINE);
    void* p = mem.data() + (OFLD_CACHELINE - reinterpret_cast<uintptr_t>(mem.data()) % OFLD_CACHELINE) %
                               OFLD_CACHELINE;
    auto* r = new (p) RingHeader();
    r->capacity = 8;
    r->head.store(0);
    r->tail.store(0);
    ofld_completion_entry_t e{};
    int pushed = 0;
    for (int i = 0; i < 10; ++i) {
        e.tensor_id = uint64_t(i);
        pushed += ring_push(r, e);
    }
    CHECK(pushed == 8);  // full at capacity
    ofld_completion_entry_t o{};
    for (int i = 0; i < 8; ++i) CHECK(ring_pop(r, &o) && o.tensor_id == uint64_t(i));
    CHECK(!ring_pop(r, &o));
    // A producer that scribbles over its header (capacity, a tail more than a
    // ring ahead) cannot make the consumer read outside the ring or loop over
    // entries that were never published.
    CHECK(ring_push(r, e));
    r->capacity = 1u << 30;
    CHECK(ring_pop(r, 8, &o) && o.tensor_id == e.tensor_id);
    r->tail.store(r->head.load() + 1000);
    CHECK(!ring_pop(r, 8, &o) && r->head.load() == r->tail.load());
}

void hash_properties() {
    std::vector<uint8_t> d(3 * 65536 + 777);
    std::mt19937_64 rng(1);
    for (auto& x : d) x = uint8_t(rng());
    ssh::Object a = ssh::host_hash(d.data(), d.size());
    ssh::Object b = ssh::host_hash(d.data(), d.size());
    CHECK(a.lo == b.lo && a.hi == b.hi);
    d[65536 * 2 + 5] ^= 1;
    ssh::Object c = ssh::host_hash(d.data(), d.size());
    CHECK(c.lo != a.lo && c.hi != a.hi);
    ssh::Object e = ssh::host_hash(d.data(), 0);
    CHECK(e.lo != 0 || e.hi != 0);
}

void zbf16_codec() {
    std::mt19937 rng(7);
    std::normal_distribution<float> nd(0.f, 0.02f);
    const uint64_t n = 5 * 65536 / 2 + 1024;  // 5 chunks + a 2 KiB raw tail
    std::vector<uint16_t> h(n);
    for (auto& x : h) {
        float f = nd(rng);
        uint32_t u;
        std::memcpy(&u, &f, 4);
        x = uint16_t((u + 0x8000u) >> 16);
    }
    std::vector<uint8_t> coded(n * 2), back(n * 2);
    CHECK(zbf16::encode_object(reinterpret_cast<uint8_t*>(h.data()), n * 2, coded.data()));
    CHECK(zbf16::decode_object(coded.data(), n * 2, back.data()));
    CHECK(std::memcmp(back.data(), h.data(), n * 2) == 0);
    CHECK(zbf16::coded_bytes(coded.data(), n * 2) < n * 2 * 77 / 100);
    for (auto& x : h) x = uint16_t(rng());  // uniform bit patterns do not code
    CHECK(!zbf16::encode_object(reinterpret_cast<uint8_t*>(h.data()), n * 2, coded.data()));
}

// The export decoder agrees with the reference decoder on coded objects
// (whole and in 64 KiB-aligned ranges) and, on chunks with a consistent
// header but arbitrary planes, decodes or refuses without touching memory
// outside the chunk (this runs under AddressSanitizer too).
void zbf16_export_decoder() {
    std::mt19937 rng(11);
    std::normal_distribution<float> nd(0.f, 1.f);
    const uint64_t n = 7 * 65536 / 2 + 2048;
    std::vector<uint16_t> h(n);
    for (size_t i = 0; i < n; ++i) {
        float f = nd(rng) * (i % 13 == 0 ? 300.f : 1.f) * (i % 97 == 0 ? 1e-6f : 1.f);
        uint32_t u;
        std::memcpy(&u, &f, 4);
        h[i] = uint16_t((u + 0x8000u) >> 16);
    }
    std::vector<uint8_t> coded(n * 2), a(n * 2), b(n * 2);
    CHECK(zbf16::encode_object(reinterpret_cast<uint8_t*>(h.data()), n * 2, coded.data()));
    CHECK(zbf16::decode_object(coded.data(), n * 2, a.data()));
    std::vector<uint32_t> keys;
    CHECK(zbf16::decode_range(zbf16::Coding::kZbf16, coded.data(), n * 2, 0, n * 2, b.data(), keys));
    CHECK(a == b);
    std::fill(b.begin(), b.end(), 0);
    CHECK(zbf16::decode_range(zbf16::Coding::kZbf16, coded.data() + 2 * 65536, n * 2, 2 * 65536, 3 * 65536,
                              b.data(), keys));
    CHECK(std::memcmp(b.data(), a.data() + 2 * 65536, 3 * 65536) == 0);
    for (int trial = 0; trial < 400; ++trial) {
        const uint32_t len = (trial % 3 == 0) ? 4096 : (trial % 3 == 1) ? 16384 : 65536;
        const uint32_t mode = 1 + trial % 2, ne = len / 2;
        const uint32_t plane = mode == 2 ? (ne / 8) * 3 : ne / 2;
        const uint32_t room = len - 16 - ne - plane;
        const uint32_t n_esc = uint32_t(rng() % (room + 1));
        std::vector<uint8_t> chunk(len), out(len);
        for (auto& c : chunk) c = uint8_t(rng());
        zbf16::Header hd{zbf16::kTag, uint8_t(mode), uint8_t(rng()), n_esc, len, 16 + ne + plane + n_esc};
        std::memcpy(chunk.data(), &hd, sizeof(hd));
        (void)zbf16::decode_chunk_fast(chunk.data(), len, out.data(), keys);
    }
}

}  // namespace

int main(int argc, char** argv) {
    const std::vector<Case> cases = {
        {"codec_round_trips", codec_round_trips}, {"codec_rejects_truncation", codec_rejects_truncation},
        {"framing", framing},                     {"config_parse", config_parse},
        {"layout_and_ring", layout_and_ring},     {"hash_properties", hash_properties},
        {"zbf16_codec", zbf16_codec},             {"zbf16_export_decoder", zbf16_export_decoder},
    };
    const char* filter = argc > 1 ? argv[1] : nullptr;
    for (const Case& c : cases) {
        if (filter && !std::strstr(c.name, filter)) continue;
        const int before = g_failed;
        try {
            c.fn();
        } catch (const std::exception& e) {
            ++g_failed;
            std::fprintf(stderr, "  FAIL %s: uncaught %s\n", c.name, e.what());
        }
        std::printf("%-28s %s\n", c.name, g_failed == before ? "ok" : "FAILED");
    }
    std::printf("%d checks, %d failed\n", g_checks, g_failed);
    return g_failed ? 1 : 0;
}
