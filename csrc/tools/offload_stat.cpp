// offload-stat: query a running offloadd and print its counters.
//
// Flags follow StateSpectre's tool (reference: src/tools/offload_stat.cpp:12-97):
//   offload-stat [--socket PATH | --tcp HOST:PORT] [--prometheus] [--watch N]
//                [--jobs] [--shutdown]
// --jobs prints the per-job accounting table (an addition of this runtime).
#include <unistd.h>

#include <sys/socket.h>
#include <sys/time.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "ofld/codec.h"
#include "ofld/transport.h"

using namespace ofld;

namespace {
void usage() {
    std::fprintf(stderr,
                 "usage: offload-stat [--socket PATH | --tcp HOST:PORT] [--prometheus] [--watch SECONDS]\n"
                 "                    [--jobs] [--shutdown]\n");
}

std::string human(uint64_t v) {
    const char* u[] = {"B", "KiB", "MiB", "GiB", "TiB"};
    double d = double(v);
    int i = 0;
    while (d >= 1024 && i < 4) {
        d /= 1024;
        ++i;
    }
    char b[64];
    std::snprintf(b, sizeof(b), "%.2f %s", d, u[i]);
    return b;
}

bool is_bytes(const std::string& k) { return k.find("bytes") != std::string::npos; }

void print_table(const GetStatsResponse& r) {
    std::printf("%-44s %20s\n", "metric", "value");
    for (const StatEntry& e : r.stats) {
        if (is_bytes(e.key))
            std::printf("%-44s %20s\n", e.key.c_str(), human(e.value).c_str());
        else
            std::printf("%-44s %20llu\n", e.key.c_str(), (unsigned long long)e.value);
    }
}

// "gpu3.window_used_bytes" -> ("window_used_bytes", gpu="3");
// "numa1_overflow.window_bytes" -> ("window_bytes", numa="1",pool="overflow").
std::pair<std::string, std::string> split_scope(const std::string& key) {
    const size_t dot = key.find('.');
    if (dot == std::string::npos) return {key, ""};
    const std::string scope = key.substr(0, dot), name = key.substr(dot + 1);
    std::string labels;
    if (scope.rfind("gpu", 0) == 0) {
        labels = "gpu=\"" + scope.substr(3) + "\"";
    } else if (scope.rfind("numa", 0) == 0) {
        const size_t us = scope.find('_');
        labels = "numa=\"" + scope.substr(4, us == std::string::npos ? std::string::npos : us - 4) + "\"";
        if (us != std::string::npos) labels += ",pool=\"" + scope.substr(us + 1) + "\"";
    } else {
        labels = "scope=\"" + scope + "\"";
    }
    return {name, labels};
}

// Exposition of StateSpectre's offload-stat, so its dashboards keep working:
// `offload_<key>`, a HELP line "offload daemon metric <key>", and gauges for
// levels (names with "bytes", used_ / inflight_ / draining_ prefixes, the
// bandwidth percentiles), counters for everything else.
bool prom_gauge(const std::string& key) {
    auto has = [&](const char* s) { return key.find(s) != std::string::npos; };
    auto starts = [&](const char* s) { return key.rfind(s, 0) == 0; };
    return has("bytes") || starts("used_") || starts("inflight_") || starts("draining_") || has("bandwidth_mbps");
}

// One HELP and TYPE line per metric family; scoped keys become labelled samples.
void print_prometheus(const GetStatsResponse& r, const GetJobStatsResponse* jobs) {
    std::map<std::string, std::vector<std::pair<std::string, uint64_t>>> fams;
    std::vector<std::string> order;
    for (const StatEntry& e : r.stats) {
        auto nl = split_scope(e.key);
        const std::string name = "offload_" + nl.first;
        if (!fams.count(name)) order.push_back(name);
        fams[name].push_back({nl.second, e.value});
    }
    if (jobs) {
        for (const JobStatsEntry& j : jobs->jobs) {
            const std::string l = "job=\"" + j.job.job_name + "\",job_id=\"" + std::to_string(j.job.job_id) +
                                  "\",tenant=\"" + std::to_string(j.job.tenant_id) + "\"";
            const std::pair<const char*, uint64_t> vals[] = {
                {"offload_job_pinned_bytes", j.pinned_bytes},
                {"offload_job_pageable_bytes", j.pageable_bytes},
                {"offload_job_nvme_bytes", j.nvme_bytes},
                {"offload_job_inflight_d2h_bytes", j.inflight_d2h_bytes},
                {"offload_job_inflight_export_bytes", j.inflight_export_bytes},
                {"offload_job_canonical_objects", j.canonical_object_count},
                {"offload_job_dedup_bytes_saved", j.dedup_bytes_saved}};
            for (const auto& v : vals) {
                if (!fams.count(v.first)) order.push_back(v.first);
                fams[v.first].push_back({l, v.second});
            }
        }
    }
    for (const std::string& name : order) {
        const std::string key = name.substr(8);  // after "offload_"
        std::printf("# HELP %s offload daemon metric %s\n", name.c_str(), key.c_str());
        std::printf("# TYPE %s %s\n", name.c_str(), prom_gauge(key) ? "gauge" : "counter");
        for (const auto& sample : fams[name]) {
            if (sample.first.empty())
                std::printf("%s %llu\n", name.c_str(), (unsigned long long)sample.second);
            else
                std::printf("%s{%s} %llu\n", name.c_str(), sample.first.c_str(), (unsigned long long)sample.second);
        }
    }
}

void print_jobs(const GetJobStatsResponse& r) {
    std::printf("%-24s %20s %6s %12s %12s %12s %8s %14s\n", "job", "job_id", "epoch", "pinned", "pageable", "nvme",
                "objects", "dedup_saved");
    for (const JobStatsEntry& j : r.jobs)
        std::printf("%-24s %20llu %6llu %12s %12s %12s %8llu %14s\n", j.job.job_name.c_str(),
                    (unsigned long long)j.job.job_id, (unsigned long long)j.job.launch_epoch,
                    human(j.pinned_bytes).c_str(), human(j.pageable_bytes).c_str(), human(j.nvme_bytes).c_str(),
                    (unsigned long long)j.canonical_object_count, human(j.dedup_bytes_saved).c_str());
}
}  // namespace

int main(int argc, char** argv) {
    std::string sock = "/tmp/state_spectre.sock", tcp;
    bool prom = false, shutdown = false, jobs = false;
    int watch = 0;
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        if (a == "--socket" && i + 1 < argc) sock = argv[++i];
        else if (a == "--tcp" && i + 1 < argc) tcp = argv[++i];
        else if (a == "--prometheus") prom = true;
        else if (a == "--watch" && i + 1 < argc) watch = std::atoi(argv[++i]);
        else if (a == "--shutdown") shutdown = true;
        else if (a == "--jobs") jobs = true;
        else if (a == "-h" || a == "--help") {
            usage();
            return 0;
        } else {
            usage();
            return 2;
        }
    }
    try {
        int fd;
        if (!tcp.empty()) {
            std::string host;
            uint16_t port;
            if (!split_host_port(tcp, &host, &port)) throw std::runtime_error("bad --tcp HOST:PORT");
            fd = tcp_connect(host, port, 3000);
        } else {
            fd = uds_connect(sock, 3000);
        }
        RpcClient c(fd);
        if (shutdown) {
            StatusResponse r = c.call<Op::kShutdown>(ShutdownRequest{});
            std::printf("%s\n", r.message.c_str());
            return r.ok ? 0 : 1;
        }
        // Per-job labels for the Prometheus output come from an additive
        // opcode: StateSpectre's own daemon logs it as unknown and never
        // answers, so ask on a second connection that gives up after 2 s and
        // print the daemon-wide counters alone then.
        auto job_stats = [&](GetJobStatsResponse* out) -> bool {
            try {
                int fd2 = !tcp.empty() ? tcp_connect(tcp.substr(0, tcp.rfind(':')),
                                                     uint16_t(std::stoi(tcp.substr(tcp.rfind(':') + 1))), 3000)
                                       : uds_connect(sock, 3000);
                timeval tv{2, 0};
                ::setsockopt(fd2, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
                RpcClient c2(fd2);
                *out = c2.call<Op::kGetJobStats>(GetJobStatsRequest{});
                return out->ok;
            } catch (const std::exception&) {
                return false;
            }
        };
        do {
            if (jobs) {
                GetJobStatsResponse js;
                if (!job_stats(&js)) throw std::runtime_error("the daemon does not answer GetJobStats (opcode 44)");
                print_jobs(js);
            } else {
                GetStatsResponse r = c.call<Op::kGetStats>(GetStatsRequest{});
                if (prom) {
                    GetJobStatsResponse js;
                    const bool have_jobs = job_stats(&js);
                    print_prometheus(r, have_jobs ? &js : nullptr);
                } else {
                    print_table(r);
                }
            }
            std::fflush(stdout);
            if (watch > 0) {
                sleep(unsigned(watch));
                if (!prom) std::printf("\n");
            }
        } while (watch > 0);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "offload-stat: %s\n", e.what());
        return 1;
    }
    return 0;
}
