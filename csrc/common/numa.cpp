#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "ofld/numa.h"

#include <dirent.h>
#include <errno.h>
#include <sched.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cstring>
#include <fstream>
#include <sstream>

namespace ofld {

namespace {
constexpr int kMpolBind = 2;        // MPOL_BIND
constexpr unsigned kMpolMfMove = 2;  // MPOL_MF_MOVE

std::string read_file(const std::string& p) {
    std::ifstream f(p);
    if (!f) return {};
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}
}  // namespace

std::vector<int> parse_cpulist(const std::string& s) {
    std::vector<int> out;
    std::stringstream ss(s);
    std::string tok;
    while (std::getline(ss, tok, ',')) {
        tok.erase(std::remove_if(tok.begin(), tok.end(), [](unsigned char c) { return std::isspace(c); }),
                  tok.end());
        if (tok.empty()) continue;
        size_t dash = tok.find('-');
        try {
            if (dash == std::string::npos) {
                out.push_back(std::stoi(tok));
            } else {
                int a = std::stoi(tok.substr(0, dash)), b = std::stoi(tok.substr(dash + 1));
                for (int i = a; i <= b; ++i) out.push_back(i);
            }
        } catch (...) {
            return {};
        }
    }
    return out;
}

int numa_max_node() {
    int mx = 0;
    DIR* d = opendir("/sys/devices/system/node");
    if (!d) return 0;
    while (dirent* e = readdir(d)) {
        if (std::strncmp(e->d_name, "node", 4) != 0 || !std::isdigit((unsigned char)e->d_name[4]))
            continue;
        mx = std::max(mx, std::atoi(e->d_name + 4));
    }
    closedir(d);
    return mx;
}

std::vector<int> numa_node_cpus(int node) {
    if (node < 0) return {};
    return parse_cpulist(read_file("/sys/devices/system/node/node" + std::to_string(node) + "/cpulist"));
}

int pin_thread_to_node(int node) {
    std::vector<int> cpus = numa_node_cpus(node);
    if (cpus.empty()) return -1;
    cpu_set_t set;
    CPU_ZERO(&set);
    for (int c : cpus)
        if (c >= 0 && c < CPU_SETSIZE) CPU_SET(c, &set);
    return sched_setaffinity(0, sizeof(set), &set) == 0 ? 0 : -errno;
}

int bind_range_to_node(void* addr, uint64_t len, int node, bool move) {
    if (node < 0 || len == 0) return 0;
    if (node > numa_max_node()) return -EINVAL;
    unsigned long mask[16] = {0};  // up to 1024 nodes
    if (node >= int(sizeof(mask) * 8)) return -EINVAL;
    mask[node / 64] |= 1ul << (node % 64);
    long rc = syscall(SYS_mbind, addr, len, kMpolBind, mask, (unsigned long)(node + 2),
                      move ? kMpolMfMove : 0u);
    if (rc == 0) return 0;
    if (errno == ENOSYS || errno == EPERM) return 0;  // NUMA policy unavailable: no-op
    return -errno;
}

void first_touch(void* addr, uint64_t len) {
    const long page = sysconf(_SC_PAGESIZE);
    volatile char* p = static_cast<volatile char*>(addr);
    for (uint64_t off = 0; off < len; off += uint64_t(page)) p[off] = 0;
}

int pci_numa_node(const std::string& bus_id) {
    std::string id = bus_id;
    std::transform(id.begin(), id.end(), id.begin(), [](unsigned char c) { return std::tolower(c); });
    // cudaDeviceGetPCIBusId yields "0000:1B:00.0"; sysfs uses lower case.
    std::string s = read_file("/sys/bus/pci/devices/" + id + "/numa_node");
    if (s.empty()) return -1;
    try {
        int n = std::stoi(s);
        return n < 0 ? -1 : n;
    } catch (...) {
        return -1;
    }
}

}  // namespace ofld
