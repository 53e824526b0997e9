// Python bindings of the host layer (module dtorch_b200._host). Every call that can wait on other rank
// threads or on the GPU releases the GIL.
#include <torch/extension.h>

#include "placement.h"
#include "redistribute.h"
#include "thread_group.h"

namespace py = pybind11;
using namespace dtb;

namespace {

PlacementSeq ParseSeq(const std::vector<std::string>& v) {
    PlacementSeq out;
    for (const auto& s : v) out.push_back(Placement::Parse(s));
    return out;
}

std::vector<std::string> SeqStrings(const PlacementSeq& p) {
    std::vector<std::string> out;
    for (const auto& q : p) out.push_back(q.ToString());
    return out;
}

DeviceMesh Mesh(const std::vector<int64_t>& shape, const std::vector<int64_t>& ids) { return DeviceMesh{shape, ids}; }

LocalShapes Shapes(const std::map<int64_t, std::vector<int64_t>>& m) { return LocalShapes{m}; }

}  // namespace

PYBIND11_MODULE(_host, m) {
    m.doc() = "Host layer of dtorch_b200: ThreadGroup, redistribute executor, placement algebra";

    py::class_<ThreadGroup>(m, "ThreadGroup")
        .def("get_rank", &ThreadGroup::GetRank)
        .def("get_world_size", &ThreadGroup::GetWorldSize)
        .def("get_global_device_id", &ThreadGroup::GetGlobalDeviceId)
        .def("barrier", &ThreadGroup::Barrier, py::call_guard<py::gil_scoped_release>())
        .def("all_reduce", [](ThreadGroup& g, const torch::Tensor& x) { return g.AllReduce(x); },
             py::call_guard<py::gil_scoped_release>())
        .def("all_gather_into_tensor",
             [](ThreadGroup& g, const torch::Tensor& x, const std::map<int64_t, std::vector<int64_t>>& s) {
                 return g.AllGatherIntoTensor(x, Shapes(s));
             },
             py::call_guard<py::gil_scoped_release>())
        .def("equal_shape_all_gather_into_tensor", &ThreadGroup::EqualShapeAllGatherIntoTensor,
             py::call_guard<py::gil_scoped_release>())
        .def("all_gather",
             [](ThreadGroup& g, const torch::Tensor& x, const std::map<int64_t, std::vector<int64_t>>& s, int64_t d) {
                 return g.AllGather(x, Shapes(s), d);
             },
             py::call_guard<py::gil_scoped_release>())
        .def("all_gather_into_vec",
             [](ThreadGroup& g, const torch::Tensor& x, const std::map<int64_t, std::vector<int64_t>>& s) {
                 return g.AllGatherIntoVec(x, Shapes(s));
             },
             py::call_guard<py::gil_scoped_release>())
        .def("reduce_scatter_tensor", [](ThreadGroup& g, const torch::Tensor& x) { return g.ReduceScatterTensor(x); },
             py::call_guard<py::gil_scoped_release>())
        .def("all_to_all",
             [](ThreadGroup& g, const torch::Tensor& x, size_t src, size_t dst,
                const std::map<int64_t, std::vector<int64_t>>& s) { return g.AllToAll(x, src, dst, Shapes(s)); },
             py::call_guard<py::gil_scoped_release>())
        .def("all_to_all_multi",
             [](ThreadGroup& g, const std::vector<torch::Tensor>& xs, size_t src, size_t dst,
                const std::map<int64_t, std::vector<int64_t>>& s) { return g.AllToAllMulti(xs, src, dst, Shapes(s)); },
             py::call_guard<py::gil_scoped_release>())
        .def("replicate_to_shard", &ThreadGroup::ReplicateToShard, py::arg("input"), py::arg("shard_idx"),
             py::arg("sub_split_coordinates") = -1, py::call_guard<py::gil_scoped_release>());

    m.def("get_thread_group",
          [](const std::vector<int64_t>& ids, int64_t current) -> ThreadGroup& {
              return ThreadGroupManager::Global().GetThreadGroup(ids, current);
          },
          py::return_value_policy::reference, py::call_guard<py::gil_scoped_release>(),
          "ThreadGroup of the group `ids` for the rank on device `current` (created on first use)");
    m.def("set_pool_bytes", &SetPoolBytes, py::arg("bytes"),
          "bytes of symmetric pool (NVLS buffer or symmetric heap) each peer-mode group created from now on gets");
    m.def("pool_bytes", &PoolBytes);
    m.def("pool_empty",
          [](const std::vector<int64_t>& ids, int64_t current, const std::vector<int64_t>& shape, py::object dtype,
             size_t bytesAllRanks) {
              const auto st = torch::python::detail::py_object_to_dtype(dtype);
              py::gil_scoped_release nogil;
              ThreadGroup& tg = ThreadGroupManager::Global().GetThreadGroup(ids, current);
              auto opts = torch::TensorOptions().dtype(st).device(torch::kCUDA, CudaDeviceOf(current));
              return tg.NewOutput(shape, opts, bytesAllRanks);
          },
          "a tensor for device `current` from the symmetric pool of the group `ids` (torch.empty when the group has "
          "no pool or it is full); every device of the group must make the same sequence of these calls with the "
          "same bytes_all_ranks");
    m.def("pool_info", [](const std::vector<int64_t>& ids, int64_t current) {
        ThreadGroup& tg = ThreadGroupManager::Global().GetThreadGroup(ids, current);
        py::dict d;
        SymmetricPool* p = tg.Pool();
        d["bytes"] = p ? p->bytes() : 0;
        d["nvls"] = p ? p->nvls() : false;
        d["in_use"] = p ? p->InUse() : 0;
        return d;
    });
    m.def("in_pool", [](const std::vector<int64_t>& ids, int64_t current, const torch::Tensor& t) {
        ThreadGroup& tg = ThreadGroupManager::Global().GetThreadGroup(ids, current);
        SymmetricPool* p = tg.Pool();
        return p != nullptr && t.defined() && p->Owns(tg.GetRank(), t.data_ptr());
    });
    m.def("clear", []() {
        KernelStreamManager::Global().Clear();
        ThreadGroupManager::Global().Clear();
    }, py::call_guard<py::gil_scoped_release>(), "destroy every kernel stream thread and communicator");

    m.def("redistribute",
          [](const std::map<int64_t, torch::Tensor>& locals, const std::vector<int64_t>& meshShape,
             const std::vector<int64_t>& meshIds, const std::vector<std::string>& src, const std::vector<std::string>& dst,
             const std::vector<int64_t>& globalShape, bool handoff) {
              return Redistribute(locals, Mesh(meshShape, meshIds), ParseSeq(src), ParseSeq(dst), globalShape, handoff);
          },
          py::arg("locals"), py::arg("mesh_shape"), py::arg("mesh_ids"), py::arg("src"), py::arg("dst"),
          py::arg("global_shape"), py::arg("handoff") = true, py::call_guard<py::gil_scoped_release>());

    m.def("redistribute_multi",
          [](const std::vector<std::map<int64_t, torch::Tensor>>& locals, const std::vector<int64_t>& meshShape,
             const std::vector<int64_t>& meshIds, const std::vector<std::string>& src, const std::vector<std::string>& dst,
             const std::vector<int64_t>& globalShape, bool handoff) {
              return RedistributeMulti(locals, Mesh(meshShape, meshIds), ParseSeq(src), ParseSeq(dst), globalShape,
                                       handoff);
          },
          py::arg("locals"), py::arg("mesh_shape"), py::arg("mesh_ids"), py::arg("src"), py::arg("dst"),
          py::arg("global_shape"), py::arg("handoff") = true, py::call_guard<py::gil_scoped_release>());
    m.def("kernel_stream", [](int64_t globalDeviceId) {
        auto& ks = KernelStreamManager::Global().Get(globalDeviceId);
        return py::make_tuple(reinterpret_cast<uintptr_t>(ks.Stream().stream()), ks.CudaDevice());
    }, "(cudaStream_t as int, CUDA device) of the kernel stream the executor runs a device's collectives on");

    // placement algebra (host logic; testable without a GPU)
    m.def("shard_sizes", &ShardSizes);
    m.def("get_convert_order", [](const std::vector<std::string>& a, const std::vector<std::string>& b) {
        return GetConvertOrder(ParseSeq(a), ParseSeq(b));
    });
    m.def("get_diff_dims", [](const std::vector<std::string>& a, const std::vector<std::string>& b) {
        return GetDiffDims(ParseSeq(a), ParseSeq(b));
    });
    m.def("normalize", [](std::vector<std::string> p, const std::vector<int64_t>& meshShape, const std::vector<int64_t>& ids,
                          size_t ndim) {
        PlacementSeq q = ParseSeq(p);
        ShardDimToPositive(q, ndim);
        ToReplicateWhenDimSizeEqualOne(q, Mesh(meshShape, ids));
        return SeqStrings(q);
    });
    m.def("check_valid", [](const std::vector<int64_t>& shape, const std::vector<int64_t>& meshShape,
                            const std::vector<int64_t>& ids, const std::vector<std::string>& p) {
        CheckValid(shape, Mesh(meshShape, ids), ParseSeq(p));
    });
    m.def("group_device_ids", [](const std::vector<int64_t>& meshShape, const std::vector<int64_t>& ids, size_t dim,
                                 int64_t device) { return GroupDeviceIds(Mesh(meshShape, ids), dim, device); });
    m.def("compute_local_shapes", [](const std::vector<int64_t>& shape, const std::vector<int64_t>& meshShape,
                                     const std::vector<int64_t>& ids, const std::vector<std::string>& p) {
        return ComputeLocalShapes(shape, Mesh(meshShape, ids), ParseSeq(p));
    });
}
