#include "ofld/metrics.h"

#include <algorithm>
#include <cmath>

#include "ofld/log.h"

namespace ofld {

const char* metric_name(M m) {
    switch (m) {
#define OFLD_NAME(id, name) \
    case M::id: return name;
        OFLD_METRICS(OFLD_NAME)
#undef OFLD_NAME
        case M::kCount: break;
    }
    return "unknown";
}

Metrics& Metrics::get() {
    static Metrics m;
    return m;
}

Metrics::Metrics() {
    for (auto& c : c_) c.store(0, std::memory_order_relaxed);
    bw_ring_.reserve(8192);
}

void Metrics::reset() {
    for (auto& c : c_) c.store(0, std::memory_order_relaxed);
    std::lock_guard<std::mutex> g(bw_mu_);
    bw_ring_.clear();
    bw_next_ = 0;
}

void Metrics::record_mbps(double mbps) {
    if (!(mbps > 0.0) || std::isinf(mbps)) return;
    std::lock_guard<std::mutex> g(bw_mu_);
    // Fixed-size ring of the most recent 8192 samples.
    if (bw_ring_.size() < 8192) {
        bw_ring_.push_back(mbps);
    } else {
        bw_ring_[bw_next_] = mbps;
        bw_next_ = (bw_next_ + 1) % bw_ring_.size();
    }
}

double Metrics::mbps_percentile(double p) const {
    std::vector<double> v;
    {
        std::lock_guard<std::mutex> g(bw_mu_);
        v = bw_ring_;
    }
    if (v.empty()) return 0.0;
    std::sort(v.begin(), v.end());
    p = std::min(1.0, std::max(0.0, p));
    return v[static_cast<size_t>(std::lround(p * double(v.size() - 1)))];
}

std::vector<std::pair<std::string, uint64_t>> Metrics::snapshot() const {
    std::vector<std::pair<std::string, uint64_t>> out;
    out.reserve(size_t(M::kCount) + 3);
    for (int i = 0; i < int(M::kCount); ++i)
        out.emplace_back(metric_name(M(i)), c_[i].load(std::memory_order_relaxed));
    out.emplace_back("bandwidth_mbps_p50", uint64_t(mbps_percentile(0.50)));
    out.emplace_back("bandwidth_mbps_p90", uint64_t(mbps_percentile(0.90)));
    out.emplace_back("bandwidth_mbps_p99", uint64_t(mbps_percentile(0.99)));
    return out;
}

Trace& Trace::get() {
    static Trace t;
    return t;
}

void Trace::open(const std::string& path) {
    std::lock_guard<std::mutex> g(mu_);
    FILE* old = fp_.exchange(nullptr);
    if (old) std::fclose(old);
    FILE* f = std::fopen(path.c_str(), "w");
    if (!f) {
        LOG_WARN("trace", "cannot open trace file %s", path.c_str());
        return;
    }
    fp_.store(f, std::memory_order_release);
}

void Trace::close() {
    std::lock_guard<std::mutex> g(mu_);
    FILE* old = fp_.exchange(nullptr);
    if (old) std::fclose(old);
}

void Trace::event(const char* name, uint32_t rank, uint32_t gpu, uint64_t tensor_id,
                  uint64_t version, uint64_t lease_id, uint32_t slot_id, uint64_t nbytes) {
    if (!on()) return;
    std::lock_guard<std::mutex> g(mu_);
    FILE* f = fp_.load(std::memory_order_relaxed);
    if (!f) return;
    std::fprintf(f,
                 "{\"ts_ns\":%llu,\"rank\":%u,\"gpu\":%u,\"tensor_id\":%llu,\"version\":%llu,"
                 "\"lease_id\":%llu,\"slot_id\":%u,\"event\":\"%s\",\"nbytes\":%llu}\n",
                 (unsigned long long)real_ns(), rank, gpu, (unsigned long long)tensor_id,
                 (unsigned long long)version, (unsigned long long)lease_id, slot_id, name,
                 (unsigned long long)nbytes);
    std::fflush(f);
}

}  // namespace ofld
