#include "fabric.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>

namespace ofld {
namespace fabric {

namespace {

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
    static AddressRangeFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return AddressRangeFn(nullptr);
        return reinterpret_cast<AddressRangeFn>(p);
    }();
    return fn;
}

struct Opened {
    uint64_t base = 0;
    int refs = 0;
};
std::mutex g_mu;
std::map<std::string, Opened> g_by_handle;   // handle bytes -> mapping
std::map<uint64_t, std::string> g_by_base;   // base -> handle bytes

}  // namespace

Export export_ptr(uint64_t dev_ptr) {
    AddressRangeFn fn = address_range_fn();
    if (!fn) throw std::runtime_error("cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, CUdeviceptr(dev_ptr)) != CUDA_SUCCESS)
        throw std::runtime_error("cuMemGetAddressRange failed (not a device allocation?)");
    cudaIpcMemHandle_t h;
    check(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
    cudaPointerAttributes attr;
    check(cudaPointerGetAttributes(&attr, reinterpret_cast<void*>(dev_ptr)), "cudaPointerGetAttributes");
    Export e;
    e.handle.assign(reinterpret_cast<const char*>(&h), sizeof(h));
    e.base = uint64_t(base);
    e.offset = dev_ptr - uint64_t(base);
    e.alloc_size = size;
    e.device = attr.device;
    return e;
}

uint64_t open_handle(const std::string& handle, uint64_t offset) {
    if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("bad IPC handle size");
    std::lock_guard<std::mutex> g(g_mu);
    auto it = g_by_handle.find(handle);
    if (it == g_by_handle.end()) {
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handle.data(), sizeof(h));
        void* p = nullptr;
        check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
        Opened o;
        o.base = reinterpret_cast<uint64_t>(p);
        it = g_by_handle.emplace(handle, o).first;
        g_by_base[o.base] = handle;
    }
    it->second.refs++;
    return it->second.base + offset;
}

void close_ptr(uint64_t peer_ptr) {
    std::lock_guard<std::mutex> g(g_mu);
    auto b = g_by_base.upper_bound(peer_ptr);
    if (b == g_by_base.begin()) return;
    --b;
    auto it = g_by_handle.find(b->second);
    if (it == g_by_handle.end()) return;
    if (--it->second.refs > 0) return;
    cudaIpcCloseMemHandle(reinterpret_cast<void*>(it->second.base));
    g_by_base.erase(b);
    g_by_handle.erase(it);
}

bool can_access_peer(int device, int peer) {
    int ok = 0;
    return cudaDeviceCanAccessPeer(&ok, device, peer) == cudaSuccess && ok;
}

void enable_peer(int peer) {
    cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        return;
    }
    check(e, "cudaDeviceEnablePeerAccess");
}

int open_count() {
    std::lock_guard<std::mutex> g(g_mu);
    return int(g_by_handle.size());
}

}  // namespace fabric
}  // namespace ofld
