// ref_harness.cc -- TEST INFRASTRUCTURE ONLY. Drives the reference's own ThreadGroup (compiled out of tree
// from tingkuanpei/dtorch sources, CPU-only) the way the reference drives it: n rank threads in one process,
// each constructing ThreadGroup(initPath, kCpu, ids, rank, n, /*sameDevice=*/true), setting its stream, then
// calling Barrier() and the collective (dtorch/tests/test_nccl.cc:27-65; the Barrier before every
// redistribute is dtorch/core/kernel/kernel_implement/convert_kernel.cc:146). The collective is dispatched as
// ConvertKernel::ConvertPlacements does (convert_kernel.cc:148-182).
//
// Exposed as a C ABI for the oracle tests (golden fixtures) and for bench.py's reference (CPU) arm. The
// reference sources are never copied: the recipe in oracle/Makefile compiles them where they lie.
#include <atomic>
#include <barrier>
#include <chrono>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <torch/torch.h>

#include "dtorch/core/communication/tensor_store/file_tensor_store.h"
#include "dtorch/core/communication/thread_group/thread_group.h"
#include "dtorch/core/operand.h"

namespace dc = dtorch::core;
namespace dcc = dtorch::core::communication;
using dtorch::external::device::DeviceStream;

// The file-backed (cross-process) tensor store is never selected when every rank lives in this process;
// these definitions only satisfy TensorStore::Create's reference to it.
namespace dtorch {
namespace core {
namespace communication {
FileTensorStore::FileTensorStore(const std::string&, int) : mResetCount(0) {
    throw std::runtime_error("oracle harness: file tensor store is not available");
}
FileTensorStore::~FileTensorStore() = default;
void FileTensorStore::SrcSet(const std::string&, const torch::Tensor&, DeviceStream&, size_t, std::optional<DeviceKind>) {}
void FileTensorStore::SrcWaitUntilGetFinished(const std::string&, DeviceStream&) {}
torch::Tensor FileTensorStore::DestGet(const std::string&, DeviceStream&) { return {}; }
void FileTensorStore::DestFinishGet(const std::string&, DeviceStream&) {}
void FileTensorStore::Reset() {}
void FileTensorStore::Barrier() {}
void FileTensorStore::SetLongString(const std::string&, const std::string&) {}
std::string FileTensorStore::GetLongString(const std::string&) const { return {}; }
}  // namespace communication
}  // namespace core
}  // namespace dtorch

namespace {

std::mutex g_err_mu;
std::string g_err;
std::atomic<int> g_group_counter{0};

void set_err(const std::string& e) {
    std::lock_guard<std::mutex> g(g_err_mu);
    g_err = e;
}

torch::ScalarType scalar(int dtype) {
    switch (dtype) {
        case 0: return torch::kFloat32;
        case 1: return torch::kBFloat16;
        case 2: return torch::kFloat16;
        default: return torch::kUInt8;
    }
}

enum class Op { kAllReduce, kReduceScatter, kAllGather, kAllToAll };

struct Job {
    Op op;
    int n;
    int dtype;
    const void* const* ins;
    void* const* outs;
    std::vector<std::vector<int64_t>> shapes;  // per-rank local input shape
    int dim_a = 0;                              // shard dim (all-gather) / src dim (all-to-all)
    int dim_b = 0;                              // dst dim (all-to-all)
    int iters = 1;
    double* secs = nullptr;
};

int run(const Job& job, int torch_threads) {
    if (job.n < 2 || job.n > 64) {
        set_err("n must be >= 2 (the same-device backend asserts world size >= 2)");
        return 1;
    }
    if (torch_threads > 0) torch::set_num_threads(torch_threads);
    const int n = job.n;
    const std::string init = "dtb2_oracle_group_" + std::to_string(g_group_counter.fetch_add(1));
    std::vector<int64_t> ids(n);
    for (int i = 0; i < n; ++i) ids[i] = i;
    std::map<int64_t, dc::Shape> local_shapes;
    bool even = true;
    for (int r = 0; r < n; ++r) {
        local_shapes[r] = dc::Shape(job.shapes[r]);
        if (job.shapes[r] != job.shapes[0]) even = false;
    }
    const dc::Operand operand(local_shapes, even);
    std::vector<std::vector<double>> times(n, std::vector<double>(job.iters, 0.0));
    std::barrier sync(n);
    std::atomic<int> failed{0};
    auto body = [&](int rank) {
        try {
            dcc::ThreadGroup tg(init, dc::DeviceKind::kCpu, ids, rank, n, /*sameDevice=*/true);
            DeviceStream stream(dc::Device(dc::DeviceKind::kCpu));
            tg.SetStream(stream);
            const auto& shp = job.shapes[rank];
            torch::Tensor src = torch::from_blob(const_cast<void*>(job.ins[rank]), shp, torch::TensorOptions().dtype(scalar(job.dtype)));
            torch::Tensor out;
            for (int it = 0; it < job.iters; ++it) {
                // fresh input every repetition: the reference's reduce-scatter folds into rank 0's input
                torch::Tensor input = src.clone();
                sync.arrive_and_wait();
                const auto t0 = std::chrono::steady_clock::now();
                tg.Barrier();
                switch (job.op) {
                    case Op::kAllReduce: out = tg.AllReduce(input); break;
                    case Op::kReduceScatter: out = tg.ReduceScatterTensor(input); break;
                    case Op::kAllGather:
                        out = job.dim_a == 0 ? tg.AllGatherIntoTensor(input, operand) : tg.AllGather(input, operand, job.dim_a);
                        break;
                    case Op::kAllToAll:
                        out = tg.AllToAll(input, static_cast<size_t>(job.dim_a), static_cast<size_t>(job.dim_b), operand);
                        break;
                }
                const auto t1 = std::chrono::steady_clock::now();
                times[rank][it] = std::chrono::duration<double>(t1 - t0).count();
            }
            sync.arrive_and_wait();
            if (job.outs != nullptr && job.outs[rank] != nullptr) {
                torch::Tensor c = out.contiguous();
                std::memcpy(job.outs[rank], c.data_ptr(), c.numel() * c.element_size());
            }
            sync.arrive_and_wait();
        } catch (const std::exception& e) {
            set_err(e.what());
            failed = 1;
            std::_Exit(3);  // a rank failing inside the reference's barriers would leave the others blocked
        }
    };
    std::vector<std::thread> th;
    for (int r = 0; r < n; ++r) th.emplace_back(body, r);
    for (auto& t : th) t.join();
    if (failed) return 2;
    if (job.secs != nullptr) {
        for (int it = 0; it < job.iters; ++it) {
            double m = 0;
            for (int r = 0; r < n; ++r) m = std::max(m, times[r][it]);
            job.secs[it] = m;
        }
    }
    return 0;
}

std::vector<std::vector<int64_t>> split_shapes(int n, int ndim, const int64_t* shapes) {
    std::vector<std::vector<int64_t>> s(n);
    for (int r = 0; r < n; ++r) s[r].assign(shapes + r * ndim, shapes + (r + 1) * ndim);
    return s;
}

}  // namespace

extern "C" {

const char* dtref_last_error(void) { return g_err.c_str(); }

// Partial -> Replicate: ThreadGroup::AllReduce on 1-D inputs of `count` elements.
int dtref_all_reduce(int n, int dtype, const void* const* ins, void* const* outs, int64_t count, int iters,
                     int torch_threads, double* secs) {
    Job j{Op::kAllReduce, n, dtype, ins, outs};
    j.shapes.assign(n, std::vector<int64_t>{count});
    j.iters = iters;
    j.secs = secs;
    return run(j, torch_threads);
}

// Partial -> Shard(0): ThreadGroup::ReduceScatterTensor on 1-D inputs of n * out_count elements.
int dtref_reduce_scatter(int n, int dtype, const void* const* ins, void* const* outs, int64_t out_count, int iters,
                         int torch_threads, double* secs) {
    Job j{Op::kReduceScatter, n, dtype, ins, outs};
    j.shapes.assign(n, std::vector<int64_t>{out_count * n});
    j.iters = iters;
    j.secs = secs;
    return run(j, torch_threads);
}

// Shard(shard_dim) -> Replicate with per-rank local shapes (n x ndim, row-major): AllGatherIntoTensor for
// dim 0 (even -> _allgather_base, uneven -> list allgather + concat), AllGather otherwise.
int dtref_all_gather(int n, int dtype, const void* const* ins, void* const* outs, int ndim, const int64_t* shapes,
                     int shard_dim, int iters, int torch_threads, double* secs) {
    Job j{Op::kAllGather, n, dtype, ins, outs};
    j.shapes = split_shapes(n, ndim, shapes);
    j.dim_a = shard_dim;
    j.iters = iters;
    j.secs = secs;
    return run(j, torch_threads);
}

// Shard(src_dim) -> Shard(dst_dim): ThreadGroup::AllToAll with per-rank local input shapes.
int dtref_all_to_all(int n, int dtype, const void* const* ins, void* const* outs, int ndim, const int64_t* shapes,
                     int src_dim, int dst_dim, int iters, int torch_threads, double* secs) {
    Job j{Op::kAllToAll, n, dtype, ins, outs};
    j.shapes = split_shapes(n, ndim, shapes);
    j.dim_a = src_dim;
    j.dim_b = dst_dim;
    j.iters = iters;
    j.secs = secs;
    return run(j, torch_threads);
}

}  // extern "C"
