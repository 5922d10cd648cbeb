// Virtual-memory-managed device buffers and NVLink SHARP (NVLS) multicast
// teams, shared between rank processes as POSIX file descriptors.
//
// A rollout rank allocates its weight buffer with cuMemCreate (shareable as
// an fd) and maps it for its own GPU. A trainer rank either maps the same
// physical memory into its address space (P2P: plain stores over NVLink), or
// builds a multicast team of its GPU and every rollout GPU that holds a
// replica of its shard: each member binds an equal-sized buffer, the trainer
// maps the multicast object, and one `multimem.st` from the trainer lands in
// every member's buffer through the NVSwitch.
//
// Driver entry points are resolved through cudaGetDriverEntryPoint, so there
// is no link-time libcuda dependency. All calls throw std::runtime_error with
// the driver's error name on failure.
#pragma once

#include <cstdint>

namespace ofld {
namespace fabric {

struct Vmm {
    uint64_t ptr = 0;     // device address in this process
    uint64_t size = 0;    // mapped bytes (a multiple of the granularity)
    uint64_t handle = 0;  // CUmemGenericAllocationHandle
    int device = -1;      // physical location
    bool imported = false;
};

struct Team {
    uint64_t handle = 0;  // multicast object
    uint64_t size = 0;    // bytes bound per member
    uint64_t mc_ptr = 0;  // multicast mapping in this process (0: not mapped)
    int ndevices = 0;
    int map_device = -1;  // device the mapping was made for
};

// True when `device` supports switch multicast (NVLS) and the driver entry
// points are present.
bool multicast_supported(int device);
// Allocation granularity for `device`; with `multicast`, also a multiple of
// the multicast team's minimum granularity for `ndevices` members.
uint64_t granularity(int device, bool multicast, int ndevices);

// Device memory on `device`, shareable as a POSIX fd, mapped read/write for
// `device`. `nbytes` is rounded up to the granularity.
Vmm vmm_alloc(int device, uint64_t nbytes, uint64_t align_to);
void vmm_free(Vmm& v);
// A new fd for the allocation (the caller closes it).
int vmm_export(const Vmm& v);
// Maps another process's allocation (`fd`, `size` bytes, located on
// `owner_device`) into this process, accessible from `access_device`. The fd
// is not closed.
Vmm vmm_import(int fd, uint64_t size, int owner_device, int access_device);

// A multicast object for `ndevices` members of `size` bytes each (rounded to
// the minimum multicast granularity), shareable as a POSIX fd.
Team team_create(int ndevices, uint64_t size);
int team_export(const Team& t);
Team team_import(int fd, int ndevices, uint64_t size);
void team_add_device(const Team& t, int device);
// Binds [0, t.size) of `mem` (which must be at least t.size bytes, on a team
// device) to the team.
void team_bind(const Team& t, const Vmm& mem);
// Maps the multicast object for `device` (blocks until every member is
// added); returns the address `multimem` instructions use.
uint64_t team_map(Team& t, int device);
void team_unbind(const Team& t, int device);
// Unmaps (when mapped) and releases this process's reference.
void team_release(Team& t);

}  // namespace fabric
}  // namespace ofld
