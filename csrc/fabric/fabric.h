// Intra-node GPU fabric: sharing device buffers between rank processes so
// kernels on one GPU load from / store to another GPU's memory over NVLink.
//
// Export: the allocation containing a device pointer (found with the driver's
// cuMemGetAddressRange, resolved through cudaGetDriverEntryPoint so there is
// no link-time libcuda dependency) is exported as a CUDA IPC memory handle
// plus the pointer's offset inside it. Import: the handle is opened once per
// process (cudaIpcOpenMemHandle with lazy peer access) and cached with a
// reference count; the peer pointer is base + offset. Handles travel between
// ranks through offloadd's peer-buffer broker (PublishPeerBuffer /
// LookupPeerBuffer).
#pragma once

#include <cstdint>
#include <string>

namespace ofld {
namespace fabric {

struct Export {
    std::string handle;   // 64-byte cudaIpcMemHandle_t
    uint64_t base = 0;    // allocation base in the exporting process
    uint64_t offset = 0;  // pointer - base
    uint64_t alloc_size = 0;
    int device = 0;
};

// Throws std::runtime_error on failure.
Export export_ptr(uint64_t dev_ptr);
// Opens (or reuses) the allocation and returns the peer pointer (base + offset).
uint64_t open_handle(const std::string& handle, uint64_t offset);
// Drops one reference of the allocation that contains `peer_ptr`.
void close_ptr(uint64_t peer_ptr);
bool can_access_peer(int device, int peer);
// Enable direct peer access from the current device to `peer` (idempotent).
void enable_peer(int peer);
int open_count();

}  // namespace fabric
}  // namespace ofld
