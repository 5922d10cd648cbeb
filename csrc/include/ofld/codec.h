// Schema-driven little-endian codec and frame envelope.
//
// Encoding rules (shared with the Python mirror): integers are little-endian
// fixed width, bool is one byte (0/1, any non-zero decodes as true), int32 is
// its two's-complement u32, strings and vectors are a u32 count followed by the
// elements. A frame is [u32 magic "OFRP"][u16 opcode][u16 flags][u32 len][body].
#pragma once

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

#include "ofld/protocol.h"

namespace ofld {

class WireError : public std::runtime_error {
 public:
    explicit WireError(const std::string& m) : std::runtime_error(m) {}
};

constexpr size_t kFrameHeaderSize = 12;
constexpr uint32_t kMaxFramePayload = 256u << 20;

namespace detail {
template <class T, class = void>
struct has_fields : std::false_type {};
struct Probe {
    template <class... A>
    void operator()(A&...) {}
};
template <class T>
struct has_fields<T, std::void_t<decltype(fields(std::declval<Probe&>(), std::declval<T&>()))>>
    : std::true_type {};
}  // namespace detail

class Encoder {
 public:
    explicit Encoder(std::vector<uint8_t>& out) : out_(out) {}
    template <class... A>
    void operator()(A&... a) {
        (put(a), ...);
    }
    void put(bool x) { out_.push_back(x ? 1 : 0); }
    void put(uint8_t x) { out_.push_back(x); }
    void put(uint16_t x) { raw(&x, 2); }
    void put(uint32_t x) { raw(&x, 4); }
    void put(int32_t x) { raw(&x, 4); }
    void put(uint64_t x) { raw(&x, 8); }
    void put(const std::string& s) {
        if (s.size() > 0xFFFFFFFFull) throw WireError("string too long");
        put(static_cast<uint32_t>(s.size()));
        out_.insert(out_.end(), s.begin(), s.end());
    }
    template <class T>
    void put(const std::vector<T>& v) {
        put(static_cast<uint32_t>(v.size()));
        for (const T& e : v) put(e);
    }
    template <class T, std::enable_if_t<detail::has_fields<T>::value, int> = 0>
    void put(const T& m) {
        fields(*this, const_cast<T&>(m));
    }

 private:
    void raw(const void* p, size_t n) {
        const uint8_t* c = static_cast<const uint8_t*>(p);
        out_.insert(out_.end(), c, c + n);
    }
    std::vector<uint8_t>& out_;
};

class Decoder {
 public:
    Decoder(const uint8_t* p, size_t n) : p_(p), end_(p + n) {}
    template <class... A>
    void operator()(A&... a) {
        (get(a), ...);
    }
    void get(bool& x) { x = take1() != 0; }
    void get(uint8_t& x) { x = take1(); }
    void get(uint16_t& x) { raw(&x, 2); }
    void get(uint32_t& x) { raw(&x, 4); }
    void get(int32_t& x) { raw(&x, 4); }
    void get(uint64_t& x) { raw(&x, 8); }
    void get(std::string& s) {
        uint32_t n;
        get(n);
        need(n);
        s.assign(reinterpret_cast<const char*>(p_), n);
        p_ += n;
    }
    template <class T>
    void get(std::vector<T>& v) {
        uint32_t n;
        get(n);
        // Every element takes at least one byte: reject absurd counts early.
        if (n > remaining()) throw WireError("truncated wire message");
        v.clear();
        v.resize(n);
        for (T& e : v) get(e);
    }
    template <class T, std::enable_if_t<detail::has_fields<T>::value, int> = 0>
    void get(T& m) {
        fields(*this, m);
    }
    size_t remaining() const { return static_cast<size_t>(end_ - p_); }

 private:
    void need(size_t n) {
        if (remaining() < n) throw WireError("truncated wire message");
    }
    uint8_t take1() {
        need(1);
        return *p_++;
    }
    void raw(void* d, size_t n) {
        need(n);
        std::memcpy(d, p_, n);
        p_ += n;
    }
    const uint8_t* p_;
    const uint8_t* end_;
};

template <class T>
std::vector<uint8_t> encode(const T& m) {
    std::vector<uint8_t> b;
    Encoder e(b);
    e.put(m);
    return b;
}

template <class T>
T decode(const uint8_t* p, size_t n) {
    T m;
    Decoder d(p, n);
    d.get(m);
    return m;
}
template <class T>
T decode(const std::vector<uint8_t>& b) {
    return decode<T>(b.data(), b.size());
}

struct FrameHeader {
    uint32_t magic = kRpcMagic;
    uint16_t opcode = 0;
    uint16_t flags = 0;
    uint32_t payload_len = 0;
};

std::vector<uint8_t> make_frame(Op op, const std::vector<uint8_t>& body, uint16_t flags = 0);
FrameHeader parse_frame_header(const uint8_t* p, size_t n);

// Request/response type of every opcode (used by the RPC client and the
// daemon's dispatch table).
template <Op O>
struct OpTypes;
#define OFLD_OP(OPC, REQ, RESP)     \
    template <>                     \
    struct OpTypes<Op::OPC> {       \
        using Request = REQ;        \
        using Response = RESP;      \
    };
OFLD_OP(kRegisterRank, RegisterRankRequest, RegisterRankResponse)
OFLD_OP(kHeartbeat, HeartbeatRequest, HeartbeatResponse)
OFLD_OP(kRequestOffload, RequestOffloadRequest, RequestOffloadResponse)
OFLD_OP(kMarkD2HSubmitted, MarkD2HSubmittedRequest, MarkD2HSubmittedResponse)
OFLD_OP(kMarkD2HComplete, MarkD2HCompleteRequest, MarkD2HCompleteResponse)
OFLD_OP(kRequestPrefetch, RequestPrefetchRequest, RequestPrefetchResponse)
OFLD_OP(kMarkH2DSubmitted, MarkH2DSubmittedRequest, MarkH2DSubmittedResponse)
OFLD_OP(kMarkH2DComplete, MarkH2DCompleteRequest, MarkH2DCompleteResponse)
OFLD_OP(kReleaseLease, ReleaseLeaseRequest, ReleaseLeaseResponse)
OFLD_OP(kQueryLocation, LocationQueryRequest, LocationQueryResponse)
OFLD_OP(kBatchComplete, BatchCompleteRequest, BatchCompleteResponse)
OFLD_OP(kShutdown, ShutdownRequest, ShutdownResponse)
OFLD_OP(kGetStats, GetStatsRequest, GetStatsResponse)
OFLD_OP(kRegisterJob, RegisterJobRequest, RegisterJobResponse)
OFLD_OP(kRequestCanonicalEvict, RequestCanonicalEvictRequest, RequestCanonicalEvictResponse)
OFLD_OP(kCommitCanonicalObject, CommitCanonicalObjectRequest, CommitCanonicalObjectResponse)
OFLD_OP(kSealModelVersion, SealModelVersionRequest, SealModelVersionResponse)
OFLD_OP(kGetLatestSealedVersion, GetLatestSealedVersionRequest, GetLatestSealedVersionResponse)
OFLD_OP(kGetManifest, GetManifestRequest, GetManifestResponse)
OFLD_OP(kPullTensor, PullTensorRequest, PullTensorResponse)
OFLD_OP(kRequestCanonicalRestore, RequestCanonicalRestoreRequest, RequestCanonicalRestoreResponse)
OFLD_OP(kReleaseCanonicalRestore, ReleaseCanonicalRestoreRequest, ReleaseCanonicalRestoreResponse)
OFLD_OP(kDropCanonicalVersion, DropCanonicalVersionRequest, DropCanonicalVersionResponse)
OFLD_OP(kReleaseCanonical, ReleaseCanonicalRequest, ReleaseCanonicalResponse)
OFLD_OP(kBatchRequestOffload, BatchRequestOffloadRequest, BatchRequestOffloadResponse)
OFLD_OP(kBatchRequestPrefetch, BatchRequestPrefetchRequest, BatchRequestPrefetchResponse)
OFLD_OP(kPublishPeerBuffer, PublishPeerBufferRequest, StatusResponse)
OFLD_OP(kLookupPeerBuffer, LookupPeerBufferRequest, LookupPeerBufferResponse)
OFLD_OP(kGetJobStats, GetJobStatsRequest, GetJobStatsResponse)
OFLD_OP(kExportManifest, ExportManifestRequest, ExportManifestResponse)
OFLD_OP(kDiscardTensor, DiscardTensorRequest, StatusResponse)
OFLD_OP(kCarryForward, CarryForwardRequest, CarryForwardResponse)
OFLD_OP(kGetAgentOptions, GetAgentOptionsRequest, GetAgentOptionsResponse)
OFLD_OP(kBatchDiscardTensor, BatchDiscardTensorRequest, BatchDiscardTensorResponse)
OFLD_OP(kSetRunFormat, SetRunFormatRequest, StatusResponse)
#undef OFLD_OP

// Re-encode a body through the C++ schema (decode then encode). Used by the
// cross-language codec tests; throws WireError on malformed input.
std::vector<uint8_t> reencode_body(Op op, bool response, const std::vector<uint8_t>& body);

}  // namespace ofld
