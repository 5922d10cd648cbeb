#include "ofld/codec.h"

#include <cstdarg>

#include "ofld/log.h"

namespace ofld {

const char* op_name(Op op) {
    switch (op) {
        case Op::kInvalid: return "Invalid";
        case Op::kRegisterRank: return "RegisterRank";
        case Op::kHeartbeat: return "Heartbeat";
        case Op::kRequestOffload: return "RequestOffload";
        case Op::kMarkD2HSubmitted: return "MarkD2HSubmitted";
        case Op::kMarkD2HComplete: return "MarkD2HComplete";
        case Op::kRequestPrefetch: return "RequestPrefetch";
        case Op::kMarkH2DSubmitted: return "MarkH2DSubmitted";
        case Op::kMarkH2DComplete: return "MarkH2DComplete";
        case Op::kReleaseLease: return "ReleaseLease";
        case Op::kQueryLocation: return "QueryLocation";
        case Op::kBatchComplete: return "BatchComplete";
        case Op::kShutdown: return "Shutdown";
        case Op::kGetStats: return "GetStats";
        case Op::kRegisterJob: return "RegisterJob";
        case Op::kRequestCanonicalEvict: return "RequestCanonicalEvict";
        case Op::kCommitCanonicalObject: return "CommitCanonicalObject";
        case Op::kSealModelVersion: return "SealModelVersion";
        case Op::kGetLatestSealedVersion: return "GetLatestSealedVersion";
        case Op::kGetManifest: return "GetManifest";
        case Op::kPullTensor: return "PullTensor";
        case Op::kRequestCanonicalRestore: return "RequestCanonicalRestore";
        case Op::kReleaseCanonicalRestore: return "ReleaseCanonicalRestore";
        case Op::kDropCanonicalVersion: return "DropCanonicalVersion";
        case Op::kReleaseCanonical: return "ReleaseCanonical";
        case Op::kBatchRequestOffload: return "BatchRequestOffload";
        case Op::kBatchRequestPrefetch: return "BatchRequestPrefetch";
        case Op::kPublishPeerBuffer: return "PublishPeerBuffer";
        case Op::kLookupPeerBuffer: return "LookupPeerBuffer";
        case Op::kGetJobStats: return "GetJobStats";
        case Op::kExportManifest: return "ExportManifest";
        case Op::kDiscardTensor: return "DiscardTensor";
        case Op::kCarryForward: return "CarryForward";
        case Op::kGetAgentOptions: return "GetAgentOptions";
        case Op::kBatchDiscardTensor: return "BatchDiscardTensor";
        case Op::kSetRunFormat: return "SetRunFormat";
    }
    return "Unknown";
}

std::vector<uint8_t> make_frame(Op op, const std::vector<uint8_t>& body, uint16_t flags) {
    if (body.size() > 0xFFFFFFFFull) throw WireError("frame body too large");
    std::vector<uint8_t> f;
    f.reserve(kFrameHeaderSize + body.size());
    Encoder e(f);
    e.put(kRpcMagic);
    e.put(static_cast<uint16_t>(op));
    e.put(flags);
    e.put(static_cast<uint32_t>(body.size()));
    f.insert(f.end(), body.begin(), body.end());
    return f;
}

FrameHeader parse_frame_header(const uint8_t* p, size_t n) {
    if (n < kFrameHeaderSize) throw WireError("short frame header");
    Decoder d(p, n);
    FrameHeader h;
    d(h.magic, h.opcode, h.flags, h.payload_len);
    if (h.magic != kRpcMagic) throw WireError("bad frame magic");
    return h;
}

namespace {
template <Op O>
std::vector<uint8_t> rt(bool response, const std::vector<uint8_t>& b) {
    if (response) return encode(decode<typename OpTypes<O>::Response>(b));
    return encode(decode<typename OpTypes<O>::Request>(b));
}
}  // namespace

std::vector<uint8_t> reencode_body(Op op, bool response, const std::vector<uint8_t>& body) {
    switch (op) {
#define CASE(O) \
    case Op::O: return rt<Op::O>(response, body);
        CASE(kRegisterRank) CASE(kHeartbeat) CASE(kRequestOffload) CASE(kMarkD2HSubmitted)
        CASE(kMarkD2HComplete) CASE(kRequestPrefetch) CASE(kMarkH2DSubmitted)
        CASE(kMarkH2DComplete) CASE(kReleaseLease) CASE(kQueryLocation) CASE(kBatchComplete)
        CASE(kShutdown) CASE(kGetStats) CASE(kRegisterJob) CASE(kRequestCanonicalEvict)
        CASE(kCommitCanonicalObject) CASE(kSealModelVersion) CASE(kGetLatestSealedVersion)
        CASE(kGetManifest) CASE(kPullTensor) CASE(kRequestCanonicalRestore)
        CASE(kReleaseCanonicalRestore) CASE(kDropCanonicalVersion) CASE(kReleaseCanonical)
        CASE(kBatchRequestOffload) CASE(kBatchRequestPrefetch) CASE(kPublishPeerBuffer)
        CASE(kLookupPeerBuffer) CASE(kGetJobStats) CASE(kExportManifest) CASE(kDiscardTensor)
        CASE(kCarryForward)
        CASE(kGetAgentOptions)
        CASE(kBatchDiscardTensor)
        CASE(kSetRunFormat)
#undef CASE
        default: break;
    }
    throw WireError("unknown opcode");
}

void log_write(Level lvl, const char* tag, const char* fmt, ...) {
    static std::mutex mu;
    static const char* names[] = {"ERROR", "WARN ", "INFO ", "DEBUG"};
    char buf[2048];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    std::lock_guard<std::mutex> g(mu);
    std::fprintf(stderr, "[%s][%s] %s\n", names[static_cast<int>(lvl)], tag, buf);
}

}  // namespace ofld
