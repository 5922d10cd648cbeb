// offloadd command line (flags match StateSpectre's daemon, reference:
// src/daemon/main.cpp:50-76):
//   offloadd --config PATH [--socket PATH] [--trace PATH] [--tcp-port N]
//   offloadd --smoke-arena-mb N [--numa N] [--gpu N] [--socket PATH] ...
// Extra flags: --nvme-dir PATH (enable NVMe in a smoke config),
//              --drain-on-complete 0|1, --slot-mb N, --print-config.
#include <csignal>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "config.h"
#include "daemon.h"
#include "ofld/log.h"
#include "ofld/metrics.h"

namespace {
ofld::Daemon* g_daemon = nullptr;
void on_signal(int) {
    if (g_daemon) g_daemon->stop();
}
void usage(const char* a0) {
    std::fprintf(stderr,
                 "usage: %s [--config PATH] [--socket PATH] [--trace PATH] [--tcp-port N]\n"
                 "          [--smoke-arena-mb N] [--numa N] [--gpu N] [--slot-mb N]\n"
                 "          [--nvme-dir PATH] [--drain-on-complete 0|1] [--print-config]\n",
                 a0);
}
}  // namespace

int main(int argc, char** argv) {
    std::string config_path, socket_path, trace_path, nvme_dir;
    uint64_t smoke_mb = 0, slot_mb = 0;
    uint32_t numa = 0, gpu = 0, tcp_port = 0;
    int drain_on_complete = -1;
    bool print_config = false;
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        auto next = [&]() -> std::string {
            if (i + 1 >= argc) {
                usage(argv[0]);
                std::exit(2);
            }
            return argv[++i];
        };
        if (a == "--config") config_path = next();
        else if (a == "--socket") socket_path = next();
        else if (a == "--trace") trace_path = next();
        else if (a == "--smoke-arena-mb") smoke_mb = std::strtoull(next().c_str(), nullptr, 10);
        else if (a == "--numa") numa = uint32_t(std::strtoul(next().c_str(), nullptr, 10));
        else if (a == "--gpu") gpu = uint32_t(std::strtoul(next().c_str(), nullptr, 10));
        else if (a == "--tcp-port") tcp_port = uint32_t(std::strtoul(next().c_str(), nullptr, 10));
        else if (a == "--slot-mb") slot_mb = std::strtoull(next().c_str(), nullptr, 10);
        else if (a == "--nvme-dir") nvme_dir = next();
        else if (a == "--drain-on-complete") drain_on_complete = std::atoi(next().c_str());
        else if (a == "--print-config") print_config = true;
        else if (a == "-h" || a == "--help") {
            usage(argv[0]);
            return 0;
        } else {
            std::fprintf(stderr, "unknown argument '%s'\n", a.c_str());
            usage(argv[0]);
            return 2;
        }
    }
    ofld::DaemonConfig cfg;
    try {
        if (!config_path.empty())
            cfg = ofld::load_config(config_path);
        else
            cfg = ofld::smoke_config((smoke_mb ? smoke_mb : 256) << 20, numa, gpu);
        if (slot_mb) cfg.allocation_granularity_bytes = slot_mb << 20;
        if (!nvme_dir.empty()) {
            cfg.nvme_enabled = true;
            cfg.nvme_path = nvme_dir;
        }
        if (drain_on_complete >= 0) cfg.drain_on_d2h_complete = drain_on_complete != 0;
        if (!socket_path.empty()) cfg.socket_path = socket_path;
        if (tcp_port) cfg.v2_control_tcp_port = tcp_port;
        ofld::validate(cfg);
    } catch (const std::exception& e) {
        LOG_ERR("main", "config error: %s", e.what());
        return 1;
    }
    if (print_config) {
        std::printf("socket_path=%s\nslot_bytes=%llu\narenas=%zu\ndrain_target=%s\nnvme=%d\ntcp_port=%u\n",
                    cfg.socket_path.c_str(), (unsigned long long)cfg.allocation_granularity_bytes,
                    cfg.per_numa.size(), ofld::drain_target_name(cfg.drain_target), int(cfg.nvme_enabled),
                    cfg.v2_control_tcp_port);
        return 0;
    }
    if (!trace_path.empty())
        ofld::Trace::get().open(trace_path);
    else if (const char* env = std::getenv("OFLD_TRACE"))
        if (env[0]) ofld::Trace::get().open(env);
    std::signal(SIGPIPE, SIG_IGN);
    try {
        ofld::Daemon d(cfg);
        g_daemon = &d;
        struct sigaction sa;
        std::memset(&sa, 0, sizeof(sa));
        sa.sa_handler = on_signal;
        sigaction(SIGINT, &sa, nullptr);
        sigaction(SIGTERM, &sa, nullptr);
        d.run();
        g_daemon = nullptr;
    } catch (const std::exception& e) {
        LOG_ERR("main", "fatal: %s", e.what());
        return 1;
    }
    ofld::Trace::get().close();
    return 0;
}
