// A program written against StateSpectre's C++ agent interface
// (offload::OffloadAgent), built unchanged against this runtime: host-mode
// evict / restore / location / discard of a buffer, then job registration,
// canonical evict, seal and manifest. Exits 0 when every step checks out.
//
//   ofld_compat_agent <daemon socket>
#include <cstdio>
#include <cstring>
#include <vector>

#include "ofld/offload_agent.h"

#define EXPECT(c)                                                         \
    do {                                                                  \
        if (!(c)) {                                                       \
            std::fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #c); \
            return 1;                                                     \
        }                                                                 \
    } while (0)

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s <socket>\n", argv[0]);
        return 2;
    }
    offload::AgentConfig cfg;
    cfg.socket_path = argv[1];
    cfg.cuda_device = -1;  // host mode
    cfg.rank_id = 7;
    offload::OffloadAgent agent(cfg);

    std::vector<float> src(100000), dst(100000, 0.f);
    for (size_t i = 0; i < src.size(); ++i) src[i] = float(i) * 0.5f;
    const uint64_t nbytes = src.size() * sizeof(float);
    offload::TensorMeta meta{1001, 1, nbytes, "compat.w"};
    bool invalidated = false;
    offload::OffloadTicket t = agent.evict(reinterpret_cast<uint64_t>(src.data()), nbytes, 0, true, meta,
                                           [&](uint64_t cookie) { invalidated = cookie == 42; }, 42, true);
    EXPECT(t.ok);
    EXPECT(invalidated);
    EXPECT(agent.is_offloaded(1001, 1));
    EXPECT(agent.location(1001, 1) == "pinned");
    offload::RestoreResult r = agent.restore(1001, 1, reinterpret_cast<uint64_t>(dst.data()), nbytes, 0, true);
    EXPECT(r.ok);
    EXPECT(std::memcmp(src.data(), dst.data(), nbytes) == 0);
    offload::AgentSummary s = agent.summary();
    EXPECT(s.rank_id == 7 && s.evict_count == 1 && s.restore_count == 1);
    agent.discard(1001, 1);
    EXPECT(agent.location(1001, 1) == "none");
    agent.assert_no_inflight();

    offload::RegisterJobRequest jr;
    jr.tenant_id = 0;
    jr.job_name = "compat-job";
    offload::RegisterJobResponse job = agent.register_job(jr);
    EXPECT(job.ok);
    offload::RequestCanonicalEvictRequest ce;
    ce.rank_id = agent.rank_id();
    ce.rank_epoch = s.rank_epoch;
    ce.key.job = job.job;
    ce.key.model_role = 2;  // policy_rollout
    ce.key.model_version = 1;
    ce.key.param_id = 77;
    ce.key.param_fqn_debug = "compat.w";
    ce.key.dtype = 7;
    ce.key.nbytes = nbytes;
    ce.local_tensor_id = 2001;
    ce.local_version = 1;
    ce.destructive = false;
    offload::CanonicalEvictResult cr = agent.canonical_evict(reinterpret_cast<uint64_t>(dst.data()), nbytes, 0,
                                                             false, ce, nullptr, 0, false, true);
    EXPECT(cr.ok && cr.did_d2h && cr.object_id != 0);
    offload::SealModelVersionRequest sr;
    sr.job = job.job;
    sr.model_role = 2;
    sr.model_version = 1;
    sr.promote = true;
    EXPECT(agent.seal_model_version(sr).ok);
    offload::GetManifestRequest mr;
    mr.job = job.job;
    mr.model_role = 2;
    mr.model_version = 1;
    offload::GetManifestResponse man = agent.get_manifest(mr);
    EXPECT(man.ok && man.tensors.size() == 1 && man.tensors[0].object_id == cr.object_id);
    std::vector<float> back(src.size(), 0.f);
    EXPECT(agent.canonical_restore(cr.object_id, reinterpret_cast<uint64_t>(back.data()), nbytes, 0, true).ok);
    EXPECT(std::memcmp(src.data(), back.data(), nbytes) == 0);
    std::printf("compat agent: ok\n");
    return 0;
}
