/* Minimal <numaif.h>: the memory-policy constants come from the kernel's
 * UAPI header; mbind is the raw system call (numa_shim.c). */
#ifndef OFLD_SHIM_NUMAIF_H
#define OFLD_SHIM_NUMAIF_H

#include <linux/mempolicy.h>

#ifdef __cplusplus
extern "C" {
#endif

long mbind(void *start, unsigned long len, int mode, const unsigned long *nmask, unsigned long maxnode,
           unsigned flags);

#ifdef __cplusplus
}
#endif

#endif
