// NUMA placement through raw syscalls and sysfs (no libnuma dependency).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace ofld {

// Highest NUMA node id present (0 on single-node or non-NUMA hosts).
int numa_max_node();
// CPUs of `node` parsed from /sys/devices/system/node/nodeN/cpulist.
std::vector<int> numa_node_cpus(int node);
// Restrict the calling thread to the CPUs of `node`. Returns 0 on success.
int pin_thread_to_node(int node);
// mbind(MPOL_BIND) [addr, addr+len) to `node`; `move` migrates resident pages.
// Returns 0 on success or when NUMA is unavailable, else -errno.
int bind_range_to_node(void* addr, uint64_t len, int node, bool move);
// Fault every page of [addr, addr+len) in by writing one byte per page.
void first_touch(void* addr, uint64_t len);
// NUMA node of a PCI device ("0000:1b:00.0"), or -1 when unknown.
int pci_numa_node(const std::string& bus_id);
// Parse a sysfs cpulist such as "0-3,8,10-11".
std::vector<int> parse_cpulist(const std::string& s);

}  // namespace ofld
