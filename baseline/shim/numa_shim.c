/* libnuma subset over sysfs and raw syscalls (see include/numa.h). */
#define _GNU_SOURCE
#include <numa.h>

#include <ctype.h>
#include <dirent.h>
#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/syscall.h>
#include <unistd.h>

#define BITS_PER_LONG (8 * sizeof(unsigned long))

long mbind(void *start, unsigned long len, int mode, const unsigned long *nmask, unsigned long maxnode,
           unsigned flags) {
    return syscall(SYS_mbind, start, len, mode, nmask, maxnode, flags);
}

int numa_available(void) {
    int mode = 0;
    /* get_mempolicy(&mode, NULL, 0, NULL, 0) fails with ENOSYS on kernels without NUMA */
    if (syscall(SYS_get_mempolicy, &mode, NULL, 0UL, NULL, 0UL) < 0 && errno == ENOSYS) return -1;
    return 0;
}

int numa_max_node(void) {
    DIR *d = opendir("/sys/devices/system/node");
    int best = 0;
    if (!d) return 0;
    struct dirent *e;
    while ((e = readdir(d)) != NULL) {
        if (strncmp(e->d_name, "node", 4) != 0 || !isdigit((unsigned char)e->d_name[4])) continue;
        int n = atoi(e->d_name + 4);
        if (n > best) best = n;
    }
    closedir(d);
    return best;
}

int numa_num_configured_cpus(void) {
    long n = sysconf(_SC_NPROCESSORS_CONF);
    return n > 0 ? (int)n : 1;
}

struct bitmask *numa_allocate_cpumask(void) {
    unsigned long bits = (unsigned long)numa_num_configured_cpus();
    unsigned long words = (bits + BITS_PER_LONG - 1) / BITS_PER_LONG;
    struct bitmask *m = (struct bitmask *)malloc(sizeof(*m));
    if (!m) return NULL;
    m->size = words * BITS_PER_LONG;
    m->maskp = (unsigned long *)calloc(words ? words : 1, sizeof(unsigned long));
    if (!m->maskp) {
        free(m);
        return NULL;
    }
    return m;
}

void numa_free_cpumask(struct bitmask *mask) {
    if (!mask) return;
    free(mask->maskp);
    free(mask);
}

int numa_bitmask_isbitset(const struct bitmask *mask, unsigned int n) {
    if (!mask || n >= mask->size) return 0;
    return (int)((mask->maskp[n / BITS_PER_LONG] >> (n % BITS_PER_LONG)) & 1UL);
}

/* Parse a sysfs cpulist ("0-15,32-47") into the mask. */
int numa_node_to_cpus(int node, struct bitmask *mask) {
    char path[96];
    char buf[4096];
    if (!mask || node < 0) {
        errno = EINVAL;
        return -1;
    }
    snprintf(path, sizeof(path), "/sys/devices/system/node/node%d/cpulist", node);
    FILE *f = fopen(path, "r");
    if (!f) {
        if (node != 0) {
            errno = ENOENT;
            return -1;
        }
        /* no node directory: a host without NUMA reports every CPU on node 0 */
        for (unsigned long c = 0; c < mask->size && c < (unsigned long)numa_num_configured_cpus(); ++c)
            mask->maskp[c / BITS_PER_LONG] |= 1UL << (c % BITS_PER_LONG);
        return 0;
    }
    size_t n = fread(buf, 1, sizeof(buf) - 1, f);
    fclose(f);
    buf[n] = 0;
    memset(mask->maskp, 0, ((mask->size + BITS_PER_LONG - 1) / BITS_PER_LONG) * sizeof(unsigned long));
    char *p = buf;
    while (*p) {
        while (*p == ',' || isspace((unsigned char)*p)) ++p;
        if (!isdigit((unsigned char)*p)) break;
        unsigned long lo = strtoul(p, &p, 10), hi = lo;
        if (*p == '-') hi = strtoul(p + 1, &p, 10);
        for (unsigned long c = lo; c <= hi && c < mask->size; ++c)
            mask->maskp[c / BITS_PER_LONG] |= 1UL << (c % BITS_PER_LONG);
    }
    return 0;
}
