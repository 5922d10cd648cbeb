// StateSpectre's C++ rank-agent interface over this runtime's agent.
//
// C++ programs written against StateSpectre's `offload::OffloadAgent`
// (reference: src/agent/agent.h, its structs AgentConfig, TensorMeta,
// OffloadTicket, RestoreResult, CanonicalEvictResult, AgentSummary and the
// method list of OffloadAgent) compile against this header unchanged: every
// call forwards to `ofld::Agent`, so they get the sm_100a data path (fused
// hash, zbf16 coding, job kernels) without code changes. Differences that a
// caller can observe: the content hash is always computed during the copy
// (`hash_on_commit` is accepted and ignored), and stream 0 selects the
// agent's internal stream as it does in StateSpectre.
#pragma once

#include <cstdint>
#include <functional>
#include <memory>
#include <string>

#include "agent/agent.h"

namespace offload {

using StreamHandle = uintptr_t;
using InvalidateCallback = std::function<void(uint64_t cookie)>;

using ofld::DropCanonicalVersionRequest;
using ofld::DropCanonicalVersionResponse;
using ofld::GetLatestSealedVersionRequest;
using ofld::GetLatestSealedVersionResponse;
using ofld::GetManifestRequest;
using ofld::GetManifestResponse;
using ofld::PullTensorRequest;
using ofld::PullTensorResponse;
using ofld::RegisterJobRequest;
using ofld::RegisterJobResponse;
using ofld::ReleaseCanonicalRequest;
using ofld::ReleaseCanonicalResponse;
using ofld::RequestCanonicalEvictRequest;
using ofld::SealModelVersionRequest;
using ofld::SealModelVersionResponse;

struct AgentConfig {
    std::string socket_path = "/tmp/state_spectre.sock";
    int cuda_device = 0;  // -1: host mode (CPU buffers)
    uint32_t rank_id = 0;
    uint32_t local_rank = 0;
    uint32_t world_rank = 0;
    int numa_node = -1;
    uint64_t registration_chunk_bytes = 512ull << 20;  // accepted; arenas register whole
    bool eager_register = false;
    uint64_t heartbeat_interval_ms = 1000;
    uint64_t progress_poll_us = 200;
};

struct TensorMeta {
    uint64_t tensor_id = 0;
    uint64_t version = 0;
    uint64_t nbytes = 0;
    std::string name;
};

struct OffloadTicket {
    uint64_t tensor_id = 0;
    uint64_t version = 0;
    uint64_t nbytes = 0;
    uint64_t lease_id = 0;
    uint32_t slot_id = 0;
    bool ok = false;
    std::string message;
};

struct RestoreResult {
    bool ok = false;
    std::string message;
};

struct CanonicalEvictResult {
    bool ok = false;
    std::string message;
    uint32_t action = 0;
    uint64_t object_id = 0;
    bool did_d2h = false;
};

struct AgentSummary {
    uint32_t rank_id = 0;
    int gpu_id = 0;
    int numa_node = 0;
    uint64_t registered_pinned_bytes = 0;
    uint64_t inflight_d2h_bytes = 0;
    uint64_t inflight_h2d_bytes = 0;
    uint64_t evict_count = 0;
    uint64_t restore_count = 0;
    uint64_t d2h_completed = 0;
    uint64_t h2d_completed = 0;
    uint64_t rank_epoch = 0;
    uint64_t num_slots = 0;
};

class OffloadAgent {
 public:
    explicit OffloadAgent(const AgentConfig& cfg) : device_(cfg.cuda_device) {
        ofld::AgentOptions o;
        o.socket_path = cfg.socket_path;
        o.device = cfg.cuda_device;
        o.rank_id = cfg.rank_id;
        o.local_rank = cfg.local_rank;
        o.world_rank = cfg.world_rank;
        o.numa_node = cfg.numa_node;
        o.eager_register = cfg.eager_register;
        o.heartbeat_ms = cfg.heartbeat_interval_ms;
        o.progress_poll_us = cfg.progress_poll_us;
        a_.reset(new ofld::Agent(o));
    }
    OffloadAgent(const OffloadAgent&) = delete;
    OffloadAgent& operator=(const OffloadAgent&) = delete;

    OffloadTicket evict(uint64_t dev_ptr, uint64_t nbytes, StreamHandle stream, bool destructive,
                        const TensorMeta& meta, InvalidateCallback invalidate_cb, uint64_t cookie, bool wait) {
        ofld::DoneCallback done;
        if (destructive && invalidate_cb) done = [invalidate_cb, cookie] { invalidate_cb(cookie); };
        ofld::EvictTicket t = a_->evict(dev_ptr, nbytes, s(stream), destructive, meta.tensor_id, meta.version,
                                        meta.name, std::move(done), wait);
        OffloadTicket r;
        r.tensor_id = t.tensor_id;
        r.version = t.version;
        r.nbytes = t.nbytes;
        r.lease_id = t.lease_id;
        r.slot_id = t.slot_id;
        r.ok = t.ok;
        r.message = t.message;
        return r;
    }
    bool is_offloaded(uint64_t tensor_id, uint64_t version) const { return a_->is_offloaded(tensor_id, version); }
    void wait_offloaded(uint64_t tensor_id, uint64_t version) { a_->wait_offloaded(tensor_id, version); }
    RestoreResult restore(uint64_t tensor_id, uint64_t version, uint64_t dev_ptr, uint64_t nbytes,
                          StreamHandle stream, bool wait) {
        ofld::RestoreOutcome o = a_->restore(tensor_id, version, dev_ptr, nbytes, s(stream), wait, {});
        return RestoreResult{o.ok, o.message};
    }
    std::string summary_string() const { return a_->summary_string(); }
    AgentSummary summary() const {
        ofld::AgentStats st = a_->stats();
        AgentSummary r;
        r.rank_id = st.rank_id;
        r.gpu_id = st.gpu_id;
        r.numa_node = st.numa_node;
        r.registered_pinned_bytes = st.registered_pinned_bytes;
        r.inflight_d2h_bytes = st.inflight_d2h_bytes;
        r.inflight_h2d_bytes = st.inflight_h2d_bytes;
        r.evict_count = st.evict_count;
        r.restore_count = st.restore_count;
        r.d2h_completed = st.d2h_completed;
        r.h2d_completed = st.h2d_completed;
        r.rank_epoch = st.rank_epoch;
        r.num_slots = st.num_slots;
        return r;
    }
    void assert_no_inflight() const { a_->assert_no_inflight(); }
    std::string location(uint64_t tensor_id, uint64_t version) const { return a_->location(tensor_id, version); }
    void discard(uint64_t tensor_id, uint64_t version) { a_->discard(tensor_id, version); }
    int cuda_device() const { return device_; }
    int numa_node() const { return a_->numa_node(); }
    uint32_t rank_id() const { return a_->rank_id(); }

    RegisterJobResponse register_job(const RegisterJobRequest& req) { return a_->register_job(req); }
    CanonicalEvictResult canonical_evict(uint64_t dev_ptr, uint64_t nbytes, StreamHandle stream, bool destructive,
                                         const RequestCanonicalEvictRequest& req, InvalidateCallback invalidate_cb,
                                         uint64_t cookie, bool /*hash_on_commit*/, bool wait) {
        ofld::DoneCallback done;
        if (destructive && invalidate_cb) done = [invalidate_cb, cookie] { invalidate_cb(cookie); };
        ofld::CanonicalOutcome o = a_->canonical_evict(dev_ptr, nbytes, s(stream), destructive, req, std::move(done),
                                                       wait);
        return CanonicalEvictResult{o.ok, o.message, o.action, o.object_id, o.did_d2h};
    }
    SealModelVersionResponse seal_model_version(const SealModelVersionRequest& r) { return a_->seal(r); }
    GetLatestSealedVersionResponse get_latest_sealed_version(const GetLatestSealedVersionRequest& r) {
        return a_->latest(r);
    }
    GetManifestResponse get_manifest(const GetManifestRequest& r) { return a_->manifest(r); }
    PullTensorResponse pull_tensor(const PullTensorRequest& r) { return a_->pull(r); }
    RestoreResult canonical_restore(uint64_t object_id, uint64_t dev_ptr, uint64_t nbytes, StreamHandle stream,
                                    bool wait) {
        ofld::RestoreOutcome o = a_->canonical_restore(object_id, dev_ptr, nbytes, s(stream), wait, {});
        return RestoreResult{o.ok, o.message};
    }
    DropCanonicalVersionResponse drop_canonical_version(const DropCanonicalVersionRequest& req) {
        return a_->drop_version(req);
    }
    ReleaseCanonicalResponse release_canonical(const ReleaseCanonicalRequest& req) { return a_->release(req); }

    // This runtime's agent, for the calls StateSpectre's interface lacks
    // (batches, carry-forward, peer buffers, statistics).
    ofld::Agent& native() { return *a_; }

 private:
    static ofld::StreamHandle s(StreamHandle h) { return h == 0 ? ofld::kInternalStream : ofld::StreamHandle(h); }
    std::unique_ptr<ofld::Agent> a_;
    int device_ = 0;
};

}  // namespace offload
