// Python bindings of the intra-node fabric (CUDA IPC export / open of device
// buffers) and of the K4 weight-sync push kernel. Pointers cross as integers,
// IPC handles as 64-byte `bytes`.
#include <cuda_runtime.h>
#include <pybind11/pybind11.h>

#include <stdexcept>
#include <string>

#include "../fabric/fabric.h"
#include "../kernels/kernels.h"

namespace py = pybind11;
using namespace ofld;

void bind_fabric(py::module_& m) {
    m.def("ipc_export", [](uint64_t ptr) {
        fabric::Export e = fabric::export_ptr(ptr);
        py::dict d;
        d["handle"] = py::bytes(e.handle);
        d["base"] = e.base;
        d["offset"] = e.offset;
        d["alloc_size"] = e.alloc_size;
        d["device"] = e.device;
        return d;
    });
    m.def(
        "ipc_open",
        [](py::bytes handle, uint64_t offset) {
            py::gil_scoped_release r;
            return fabric::open_handle(std::string(handle), offset);
        },
        py::arg("handle"), py::arg("offset") = 0);
    m.def("ipc_close", [](uint64_t ptr) { fabric::close_ptr(ptr); });
    m.def("ipc_open_count", &fabric::open_count);
    m.def("can_access_peer", &fabric::can_access_peer);
    m.def("enable_peer", &fabric::enable_peer);
    m.def("push_item_bytes", [] { return int(sizeof(kern::PushItem)); });
    m.def(
        "k_push",
        [](uint64_t items, int nitems, uint64_t total_chunks, uint64_t digests, uint64_t item_hash, uint64_t stats,
           uint64_t error, uint64_t stream, int ctas, uint32_t launch_flags) {
            kern::PushState st{reinterpret_cast<uint64_t*>(digests), reinterpret_cast<uint64_t*>(item_hash),
                               reinterpret_cast<unsigned long long*>(stats), reinterpret_cast<uint32_t*>(error)};
            cudaError_t e = kern::push(reinterpret_cast<const kern::PushItem*>(items), nitems, total_chunks, st,
                                       reinterpret_cast<cudaStream_t>(stream), ctas, launch_flags);
            if (e != cudaSuccess) throw std::runtime_error(std::string("push: ") + cudaGetErrorString(e));
        },
        py::arg("items"), py::arg("nitems"), py::arg("total_chunks"), py::arg("digests"), py::arg("item_hash"),
        py::arg("stats"), py::arg("error"), py::arg("stream"), py::arg("ctas") = 0, py::arg("launch_flags") = 0);
    m.def("push_smem_bytes", &kern::push_smem_bytes);
    m.def(
        "k_hash_stream",
        [](uint64_t src, uint64_t n, uint64_t digests, uint64_t error, uint64_t stream, int ctas) {
            cudaError_t e = kern::hash_stream(reinterpret_cast<const void*>(src), n, reinterpret_cast<uint64_t*>(digests),
                                              reinterpret_cast<uint32_t*>(error), reinterpret_cast<cudaStream_t>(stream),
                                              ctas);
            if (e != cudaSuccess) throw std::runtime_error(std::string("hash_stream: ") + cudaGetErrorString(e));
        },
        py::arg("src"), py::arg("nbytes"), py::arg("digests"), py::arg("error"), py::arg("stream"), py::arg("ctas") = 0);
}
