/* Minimal libnuma-compatible interface for building StateSpectre (the
 * reference implementation) on hosts without libnuma.
 *
 * Only the calls that StateSpectre's src/common/numa_util.cpp:19-143 makes are
 * declared. The implementation (numa_shim.c) reads sysfs and uses raw
 * syscalls; it is a build aid for the same-box comparison, not part of the
 * statespectre_b200 runtime. */
#ifndef OFLD_SHIM_NUMA_H
#define OFLD_SHIM_NUMA_H

#include <numaif.h>

#ifdef __cplusplus
extern "C" {
#endif

struct bitmask {
    unsigned long size;   /* number of bits */
    unsigned long *maskp; /* ceil(size / bits-per-long) words */
};

/* 0 when the kernel offers memory policies, -1 otherwise. */
int numa_available(void);
/* Highest NUMA node number present on the host (0 on a single-node host). */
int numa_max_node(void);
/* CPUs the host was configured with (online or not). */
int numa_num_configured_cpus(void);
/* A zeroed CPU mask wide enough for every configured CPU; free with numa_free_cpumask. */
struct bitmask *numa_allocate_cpumask(void);
void numa_free_cpumask(struct bitmask *mask);
/* Fill `mask` with the CPUs of `node`; 0 on success, -1 with errno set on failure. */
int numa_node_to_cpus(int node, struct bitmask *mask);
/* 1 when bit `n` is set, 0 when clear or out of range. */
int numa_bitmask_isbitset(const struct bitmask *mask, unsigned int n);

#ifdef __cplusplus
}
#endif

#endif
