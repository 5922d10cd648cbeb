// Python bindings of the intra-node fabric (CUDA IPC export / open of device
// buffers; VMM buffers and multicast teams shared as fds) and of the K4
// weight-sync push kernel. Pointers cross as integers, IPC handles as 64-byte
// `bytes`.
#include <cuda_runtime.h>
#include <pybind11/pybind11.h>

#include <stdexcept>
#include <string>

#include "../fabric/fabric.h"
#include "../fabric/vmm.h"
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
    py::class_<fabric::Vmm>(m, "Vmm")
        .def_readonly("ptr", &fabric::Vmm::ptr)
        .def_readonly("size", &fabric::Vmm::size)
        .def_readonly("device", &fabric::Vmm::device)
        .def_readonly("imported", &fabric::Vmm::imported);
    py::class_<fabric::Team>(m, "Team")
        .def_readonly("size", &fabric::Team::size)
        .def_readonly("mc_ptr", &fabric::Team::mc_ptr)
        .def_readonly("ndevices", &fabric::Team::ndevices);
    m.def("multicast_supported", &fabric::multicast_supported);
    m.def("vmm_granularity", &fabric::granularity, py::arg("device"), py::arg("multicast") = false,
          py::arg("ndevices") = 1);
    m.def("vmm_alloc", &fabric::vmm_alloc, py::arg("device"), py::arg("nbytes"), py::arg("align_to") = 0);
    m.def("vmm_free", [](fabric::Vmm& v) { fabric::vmm_free(v); });
    m.def("vmm_export", &fabric::vmm_export);
    m.def("vmm_import", &fabric::vmm_import, py::arg("fd"), py::arg("size"), py::arg("owner_device"),
          py::arg("access_device"));
    m.def("team_create", &fabric::team_create);
    m.def("team_export", &fabric::team_export);
    m.def("team_import", &fabric::team_import);
    m.def("team_add_device", [](const fabric::Team& t, int device) {
        py::gil_scoped_release r;
        fabric::team_add_device(t, device);
    });
    m.def("team_bind", [](const fabric::Team& t, const fabric::Vmm& mem) {
        py::gil_scoped_release r;
        fabric::team_bind(t, mem);
    });
    m.def("team_map", [](fabric::Team& t, int device) {
        py::gil_scoped_release r;
        return fabric::team_map(t, device);
    });
    m.def("team_unbind", &fabric::team_unbind);
    m.def("team_release", [](fabric::Team& t) { fabric::team_release(t); });
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
        [](uint64_t src, uint64_t n, uint64_t digests, uint64_t error, uint64_t stream, int ctas, int stages) {
            cudaError_t e = kern::hash_stream(reinterpret_cast<const void*>(src), n, reinterpret_cast<uint64_t*>(digests),
                                              reinterpret_cast<uint32_t*>(error), reinterpret_cast<cudaStream_t>(stream),
                                              ctas, stages);
            if (e != cudaSuccess) throw std::runtime_error(std::string("hash_stream: ") + cudaGetErrorString(e));
        },
        py::arg("src"), py::arg("nbytes"), py::arg("digests"), py::arg("error"), py::arg("stream"), py::arg("ctas") = 0,
        py::arg("stages") = 0);
}
