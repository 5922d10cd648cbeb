#include "vmm.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>

namespace ofld {
namespace fabric {

namespace {

// Driver entry points, resolved once.
struct Driver {
    decltype(&cuGetErrorName) error_name = nullptr;
    decltype(&cuDeviceGet) device_get = nullptr;
    decltype(&cuDeviceGetAttribute) device_attr = nullptr;
    decltype(&cuMemCreate) mem_create = nullptr;
    decltype(&cuMemRelease) mem_release = nullptr;
    decltype(&cuMemAddressReserve) addr_reserve = nullptr;
    decltype(&cuMemAddressFree) addr_free = nullptr;
    decltype(&cuMemMap) mem_map = nullptr;
    decltype(&cuMemUnmap) mem_unmap = nullptr;
    decltype(&cuMemSetAccess) set_access = nullptr;
    decltype(&cuMemGetAllocationGranularity) alloc_gran = nullptr;
    decltype(&cuMemExportToShareableHandle) export_handle = nullptr;
    decltype(&cuMemImportFromShareableHandle) import_handle = nullptr;
    decltype(&cuMulticastCreate) mc_create = nullptr;
    decltype(&cuMulticastAddDevice) mc_add = nullptr;
    decltype(&cuMulticastBindMem) mc_bind = nullptr;
    decltype(&cuMulticastUnbind) mc_unbind = nullptr;
    decltype(&cuMulticastGetGranularity) mc_gran = nullptr;
    bool vmm_ok = false, mc_ok = false;
};

template <class F>
void resolve(const char* name, F& fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
        fn = reinterpret_cast<F>(p);
    else
        cudaGetLastError();
}

const Driver& drv() {
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        resolve("cuGetErrorName", d.error_name);
        resolve("cuDeviceGet", d.device_get);
        resolve("cuDeviceGetAttribute", d.device_attr);
        resolve("cuMemCreate", d.mem_create);
        resolve("cuMemRelease", d.mem_release);
        resolve("cuMemAddressReserve", d.addr_reserve);
        resolve("cuMemAddressFree", d.addr_free);
        resolve("cuMemMap", d.mem_map);
        resolve("cuMemUnmap", d.mem_unmap);
        resolve("cuMemSetAccess", d.set_access);
        resolve("cuMemGetAllocationGranularity", d.alloc_gran);
        resolve("cuMemExportToShareableHandle", d.export_handle);
        resolve("cuMemImportFromShareableHandle", d.import_handle);
        resolve("cuMulticastCreate", d.mc_create);
        resolve("cuMulticastAddDevice", d.mc_add);
        resolve("cuMulticastBindMem", d.mc_bind);
        resolve("cuMulticastUnbind", d.mc_unbind);
        resolve("cuMulticastGetGranularity", d.mc_gran);
        d.vmm_ok = d.error_name && d.device_get && d.device_attr && d.mem_create && d.mem_release &&
                   d.addr_reserve && d.addr_free && d.mem_map && d.mem_unmap && d.set_access && d.alloc_gran &&
                   d.export_handle && d.import_handle;
        d.mc_ok = d.vmm_ok && d.mc_create && d.mc_add && d.mc_bind && d.mc_unbind && d.mc_gran;
    });
    return d;
}

void check(CUresult r, const char* what) {
    if (r == CUDA_SUCCESS) return;
    const char* name = nullptr;
    if (drv().error_name) drv().error_name(r, &name);
    throw std::runtime_error(std::string(what) + ": " + (name ? name : "CUresult " + std::to_string(int(r))));
}

const Driver& need_vmm() {
    const Driver& d = drv();
    if (!d.vmm_ok) throw std::runtime_error("CUDA virtual memory management entry points unavailable");
    return d;
}

const Driver& need_mc() {
    const Driver& d = drv();
    if (!d.mc_ok) throw std::runtime_error("CUDA multicast entry points unavailable");
    return d;
}

// Runs `fn` with `device`'s primary context current on this thread.
template <class F>
auto on_device(int device, F fn) -> decltype(fn()) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) throw std::runtime_error("cudaSetDevice failed");
    cudaFree(nullptr);  // creates the primary context if needed
    struct Restore {
        int d;
        ~Restore() { cudaSetDevice(d); }
    } restore{prev};
    return fn();
}

uint64_t round_up(uint64_t n, uint64_t g) { return (n + g - 1) / g * g; }

uint64_t gcd(uint64_t a, uint64_t b) {
    while (b) {
        uint64_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

CUmemAllocationProp alloc_prop(int device) {
    CUmemAllocationProp p{};
    p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    p.location.id = device;
    p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    return p;
}

void map_rw(const Driver& d, CUdeviceptr va, uint64_t size, CUmemGenericAllocationHandle h, int device) {
    check(d.mem_map(va, size, 0, h, 0), "cuMemMap");
    CUmemAccessDesc a{};
    a.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    a.location.id = device;
    a.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    CUresult r = d.set_access(va, size, &a, 1);
    if (r != CUDA_SUCCESS) {
        d.mem_unmap(va, size);
        check(r, "cuMemSetAccess");
    }
}

}  // namespace

bool multicast_supported(int device) {
    const Driver& d = drv();
    if (!d.mc_ok) return false;
    CUdevice dev;
    int v = 0;
    if (d.device_get(&dev, device) != CUDA_SUCCESS) return false;
    if (d.device_attr(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev) != CUDA_SUCCESS) return false;
    return v != 0;
}

uint64_t granularity(int device, bool multicast, int ndevices) {
    const Driver& d = need_vmm();
    CUmemAllocationProp p = alloc_prop(device);
    size_t g = 0;
    check(d.alloc_gran(&g, &p, CU_MEM_ALLOC_GRANULARITY_MINIMUM), "cuMemGetAllocationGranularity");
    uint64_t out = g;
    if (multicast) {
        const Driver& m = need_mc();
        CUmulticastObjectProp mp{};
        mp.numDevices = unsigned(ndevices > 0 ? ndevices : 1);
        mp.size = g;
        mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
        size_t mg = 0;
        check(m.mc_gran(&mg, &mp, CU_MULTICAST_GRANULARITY_MINIMUM), "cuMulticastGetGranularity");
        out = out / gcd(out, mg) * mg;
    }
    return out;
}

Vmm vmm_alloc(int device, uint64_t nbytes, uint64_t align_to) {
    const Driver& d = need_vmm();
    return on_device(device, [&] {
        uint64_t g = granularity(device, false, 0);
        if (align_to > 1) g = g / gcd(g, align_to) * align_to;
        Vmm v;
        v.device = device;
        v.size = round_up(nbytes ? nbytes : 1, g);
        CUmemAllocationProp p = alloc_prop(device);
        CUmemGenericAllocationHandle h = 0;
        check(d.mem_create(&h, v.size, &p, 0), "cuMemCreate");
        CUdeviceptr va = 0;
        CUresult r = d.addr_reserve(&va, v.size, g, 0, 0);
        if (r != CUDA_SUCCESS) {
            d.mem_release(h);
            check(r, "cuMemAddressReserve");
        }
        try {
            map_rw(d, va, v.size, h, device);
        } catch (...) {
            d.addr_free(va, v.size);
            d.mem_release(h);
            throw;
        }
        v.ptr = uint64_t(va);
        v.handle = uint64_t(h);
        return v;
    });
}

void vmm_free(Vmm& v) {
    if (!v.ptr && !v.handle) return;
    const Driver& d = need_vmm();
    on_device(v.device >= 0 ? v.device : 0, [&] {
        if (v.ptr) {
            d.mem_unmap(CUdeviceptr(v.ptr), v.size);
            d.addr_free(CUdeviceptr(v.ptr), v.size);
        }
        if (v.handle) d.mem_release(CUmemGenericAllocationHandle(v.handle));
        return 0;
    });
    v = Vmm{};
}

int vmm_export(const Vmm& v) {
    const Driver& d = need_vmm();
    int fd = -1;
    check(d.export_handle(&fd, CUmemGenericAllocationHandle(v.handle), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
          "cuMemExportToShareableHandle");
    return fd;
}

Vmm vmm_import(int fd, uint64_t size, int owner_device, int access_device) {
    const Driver& d = need_vmm();
    return on_device(access_device, [&] {
        CUmemGenericAllocationHandle h = 0;
        check(d.import_handle(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                              CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
              "cuMemImportFromShareableHandle");
        const uint64_t g = granularity(owner_device, false, 0);
        CUdeviceptr va = 0;
        CUresult r = d.addr_reserve(&va, size, g, 0, 0);
        if (r != CUDA_SUCCESS) {
            d.mem_release(h);
            check(r, "cuMemAddressReserve");
        }
        try {
            map_rw(d, va, size, h, access_device);
        } catch (...) {
            d.addr_free(va, size);
            d.mem_release(h);
            throw;
        }
        Vmm v;
        v.ptr = uint64_t(va);
        v.size = size;
        v.handle = uint64_t(h);
        v.device = access_device;
        v.imported = true;
        return v;
    });
}

Team team_create(int ndevices, uint64_t size) {
    const Driver& d = need_mc();
    CUmulticastObjectProp p{};
    p.numDevices = unsigned(ndevices);
    p.size = size;
    p.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t mg = 0;
    check(d.mc_gran(&mg, &p, CU_MULTICAST_GRANULARITY_MINIMUM), "cuMulticastGetGranularity");
    p.size = round_up(size, mg);
    CUmemGenericAllocationHandle h = 0;
    check(d.mc_create(&h, &p), "cuMulticastCreate");
    Team t;
    t.handle = uint64_t(h);
    t.size = p.size;
    t.ndevices = ndevices;
    return t;
}

int team_export(const Team& t) {
    const Driver& d = need_mc();
    int fd = -1;
    check(d.export_handle(&fd, CUmemGenericAllocationHandle(t.handle), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
          "cuMemExportToShareableHandle(multicast)");
    return fd;
}

Team team_import(int fd, int ndevices, uint64_t size) {
    const Driver& d = need_mc();
    CUmemGenericAllocationHandle h = 0;
    check(d.import_handle(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                          CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
          "cuMemImportFromShareableHandle(multicast)");
    Team t;
    t.handle = uint64_t(h);
    t.size = size;
    t.ndevices = ndevices;
    return t;
}

void team_add_device(const Team& t, int device) {
    const Driver& d = need_mc();
    on_device(device, [&] {
        CUdevice dev;
        check(d.device_get(&dev, device), "cuDeviceGet");
        check(d.mc_add(CUmemGenericAllocationHandle(t.handle), dev), "cuMulticastAddDevice");
        return 0;
    });
}

void team_bind(const Team& t, const Vmm& mem) {
    const Driver& d = need_mc();
    if (mem.imported) throw std::runtime_error("team_bind: only this process's own allocations can be bound");
    if (mem.size < t.size) throw std::runtime_error("team_bind: buffer smaller than the team's size");
    on_device(mem.device, [&] {
        check(d.mc_bind(CUmemGenericAllocationHandle(t.handle), 0, CUmemGenericAllocationHandle(mem.handle), 0, t.size,
                        0),
              "cuMulticastBindMem");
        return 0;
    });
}

uint64_t team_map(Team& t, int device) {
    const Driver& d = need_mc();
    if (t.mc_ptr) return t.mc_ptr;
    return on_device(device, [&] {
        CUmulticastObjectProp p{};
        p.numDevices = unsigned(t.ndevices);
        p.size = t.size;
        p.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
        size_t mg = 0;
        check(d.mc_gran(&mg, &p, CU_MULTICAST_GRANULARITY_MINIMUM), "cuMulticastGetGranularity");
        CUdeviceptr va = 0;
        check(d.addr_reserve(&va, t.size, mg, 0, 0), "cuMemAddressReserve(multicast)");
        try {
            map_rw(d, va, t.size, CUmemGenericAllocationHandle(t.handle), device);
        } catch (...) {
            d.addr_free(va, t.size);
            throw;
        }
        t.mc_ptr = uint64_t(va);
        t.map_device = device;
        return t.mc_ptr;
    });
}

void team_unbind(const Team& t, int device) {
    const Driver& d = need_mc();
    on_device(device, [&] {
        CUdevice dev;
        check(d.device_get(&dev, device), "cuDeviceGet");
        check(d.mc_unbind(CUmemGenericAllocationHandle(t.handle), dev, 0, t.size), "cuMulticastUnbind");
        return 0;
    });
}

void team_release(Team& t) {
    if (!t.handle) return;
    const Driver& d = need_mc();
    on_device(t.map_device >= 0 ? t.map_device : 0, [&] {
        if (t.mc_ptr) {
            d.mem_unmap(CUdeviceptr(t.mc_ptr), t.size);
            d.addr_free(CUdeviceptr(t.mc_ptr), t.size);
        }
        d.mem_release(CUmemGenericAllocationHandle(t.handle));
        return 0;
    });
    t = Team{};
}

}  // namespace fabric
}  // namespace ofld
