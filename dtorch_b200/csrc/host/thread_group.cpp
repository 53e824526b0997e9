// ThreadGroup / P2PBackend / ThreadGroupManager over the C ABI (see thread_group.h).
#include "thread_group.h"

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cstdlib>
#include <numeric>
#include <stdexcept>

#include "placement.h"

namespace dtb {

namespace {

// A Work that is complete on return: every collective here is enqueued on the caller's current stream, so
// anything the caller does next on that stream is ordered after it.
class DoneWork : public c10d::Work {
public:
    DoneWork() : c10d::Work() { finish(); }
};

c10::intrusive_ptr<c10d::Work> Done() { return c10::make_intrusive<DoneWork>(); }

int64_t Prod(const std::vector<int64_t>& v, size_t lo, size_t hi) {
    int64_t p = 1;
    for (size_t i = lo; i < hi; ++i) p *= v[i];
    return p;
}

}  // namespace

bool SameDeviceMode() {
    const char* s = std::getenv("DTORCH_DTENSOR_IN_SAME_DEVICE");
    return s != nullptr && std::string(s) == "1";
}

int CudaDeviceOf(int64_t globalDeviceId) { return SameDeviceMode() ? 0 : static_cast<int>(globalDeviceId); }

std::vector<int64_t> LocalShapes::Get(int64_t deviceId) const {
    auto it = shapes.find(deviceId);
    if (it == shapes.end()) throw std::invalid_argument("no local shape for device " + std::to_string(deviceId));
    return it->second;
}

bool LocalShapes::IsEvenSplit() const {
    if (shapes.empty()) return true;
    const auto& first = shapes.begin()->second;
    for (const auto& kv : shapes)
        if (kv.second != first) return false;
    return true;
}

void Check(int status, const char* where) {
    if (status != DT_OK)
        throw std::runtime_error(std::string(where) + ": " + dt_status_string(status) + " (" + dt_last_error_message() + ")");
}

int DTypeCode(at::ScalarType t) {
    switch (t) {
        case at::kFloat: return DT_FLOAT32;
        case at::kBFloat16: return DT_BFLOAT16;
        case at::kHalf: return DT_FLOAT16;
        default: throw std::invalid_argument(std::string("reductions support float32, bfloat16, float16; got ") + c10::toString(t));
    }
}

SharedComm::SharedComm(const std::vector<int>& cudaDevices) : mDevices(cudaDevices) {
    Check(dt_comm_create(static_cast<int>(cudaDevices.size()), cudaDevices.data(), 0, &mComm), "dt_comm_create");
    const char* t = std::getenv("DTORCH_COMM_TIMEOUT_SECOND");
    if (t != nullptr && std::atoll(t) > 0) Check(dt_comm_set_timeout_ms(mComm, std::atoll(t) * 1000), "dt_comm_set_timeout_ms");
}

SharedComm::~SharedComm() {
    if (mComm != nullptr) dt_comm_destroy(mComm);
}

// ---------------------------------------------------------------------------------------------------------
// P2PBackend
// ---------------------------------------------------------------------------------------------------------
P2PBackend::P2PBackend(std::shared_ptr<SharedComm> comm, int rank, int size) : Backend(rank, size), mComm(std::move(comm)) {}

namespace {
void* CurrentStream(int device) { return c10::cuda::getCurrentCUDAStream(device).stream(); }
}  // namespace

c10::intrusive_ptr<c10d::Work> P2PBackend::allreduce(std::vector<at::Tensor>& tensors, const c10d::AllreduceOptions& opts) {
    if (opts.reduceOp != c10d::ReduceOp::SUM) throw std::invalid_argument("dtorch_b200 allreduce supports SUM only");
    for (auto& t : tensors) {
        TORCH_CHECK(t.is_contiguous(), "allreduce needs contiguous tensors");
        Check(dt_all_reduce(comm(), getRank(), t.data_ptr(), t.data_ptr(), static_cast<size_t>(t.numel()),
                            DTypeCode(t.scalar_type()), DT_SUM, DT_ACCUM_FP32, CurrentStream(cudaDevice())),
              "dt_all_reduce");
    }
    return Done();
}

c10::intrusive_ptr<c10d::Work> P2PBackend::_allgather_base(at::Tensor& output, at::Tensor& input,
                                                           const c10d::AllgatherOptions&) {
    TORCH_CHECK(input.is_contiguous() && output.is_contiguous(), "_allgather_base needs contiguous tensors");
    TORCH_CHECK(output.numel() == input.numel() * getSize(), "_allgather_base: output must be size x input");
    std::vector<int64_t> lens(static_cast<size_t>(getSize()), input.numel());
    Check(dt_all_gather(comm(), getRank(), input.data_ptr(), output.data_ptr(), 1, lens.data(),
                        static_cast<size_t>(input.element_size()), CurrentStream(cudaDevice())),
          "dt_all_gather");
    return Done();
}

c10::intrusive_ptr<c10d::Work> P2PBackend::allgather(std::vector<std::vector<at::Tensor>>& outputs,
                                                     std::vector<at::Tensor>& inputs, const c10d::AllgatherOptions&) {
    TORCH_CHECK(outputs.size() == inputs.size(), "allgather: one output list per input");
    for (size_t i = 0; i < inputs.size(); ++i) {
        auto& outs = outputs[i];
        TORCH_CHECK(static_cast<int>(outs.size()) == getSize(), "allgather: one output per rank");
        at::Tensor in = inputs[i].contiguous();
        std::vector<int64_t> lens;
        int64_t total = 0;
        for (auto& o : outs) {
            lens.push_back(o.numel());
            total += o.numel();
        }
        TORCH_CHECK(lens[static_cast<size_t>(getRank())] == in.numel(), "allgather: own output size must match input");
        at::Tensor flat = at::empty({total}, in.options());
        Check(dt_all_gather(comm(), getRank(), in.data_ptr(), flat.data_ptr(), 1, lens.data(),
                            static_cast<size_t>(in.element_size()), CurrentStream(cudaDevice())),
              "dt_all_gather");
        int64_t off = 0;
        for (auto& o : outs) {
            o.copy_(flat.narrow(0, off, o.numel()).view(o.sizes()));
            off += o.numel();
        }
    }
    return Done();
}

c10::intrusive_ptr<c10d::Work> P2PBackend::_reduce_scatter_base(at::Tensor& output, at::Tensor& input,
                                                                const c10d::ReduceScatterOptions& opts) {
    if (opts.reduceOp != c10d::ReduceOp::SUM) throw std::invalid_argument("dtorch_b200 reduce_scatter supports SUM only");
    TORCH_CHECK(input.is_contiguous() && output.is_contiguous(), "_reduce_scatter_base needs contiguous tensors");
    TORCH_CHECK(input.numel() == output.numel() * getSize(), "_reduce_scatter_base: input must be size x output");
    Check(dt_reduce_scatter(comm(), getRank(), input.data_ptr(), output.data_ptr(), static_cast<size_t>(output.numel()),
                            DTypeCode(input.scalar_type()), DT_SUM, DT_ACCUM_FP32, CurrentStream(cudaDevice())),
          "dt_reduce_scatter");
    return Done();
}

c10::intrusive_ptr<c10d::Work> P2PBackend::alltoall(std::vector<at::Tensor>& outputs, std::vector<at::Tensor>& inputs,
                                                    const c10d::AllToAllOptions&) {
    const int n = getSize();
    TORCH_CHECK(static_cast<int>(inputs.size()) == n && static_cast<int>(outputs.size()) == n, "alltoall: one tensor per rank");
    const int64_t chunk = inputs[0].numel();
    for (int k = 0; k < n; ++k)
        TORCH_CHECK(inputs[k].numel() == chunk && outputs[k].numel() == chunk,
                    "dtorch_b200 alltoall (list form) needs equal chunks; ThreadGroup::AllToAll handles uneven shards");
    // every rank's input viewed as [1, n, chunk]: split along dim 1, chunk k -> rank k, concat along dim 0
    std::vector<at::Tensor> flat_in;
    for (auto& t : inputs) flat_in.push_back(t.reshape({-1}));
    at::Tensor in = at::cat(flat_in, 0).contiguous();
    at::Tensor out = at::empty({n, chunk}, in.options());
    const int64_t shape[3] = {1, n, chunk};
    std::vector<int64_t> lens(static_cast<size_t>(n), 1);
    Check(dt_all_to_all(comm(), getRank(), in.data_ptr(), out.data_ptr(), 3, shape, 0, 1, lens.data(),
                        static_cast<size_t>(in.element_size()), CurrentStream(cudaDevice())),
          "dt_all_to_all");
    for (int k = 0; k < n; ++k) outputs[k].copy_(out[k].view(outputs[k].sizes()));
    return Done();
}

c10::intrusive_ptr<c10d::Work> P2PBackend::barrier(const c10d::BarrierOptions&) {
    Check(dt_barrier(comm(), getRank(), CurrentStream(cudaDevice())), "dt_barrier");
    return Done();
}

// ---------------------------------------------------------------------------------------------------------
// ThreadGroup
// ---------------------------------------------------------------------------------------------------------
ThreadGroup::ThreadGroup(std::shared_ptr<SharedComm> comm, const std::vector<int64_t>& allGlobalDeviceId, int rank, int size)
    : mComm(std::move(comm)), mIds(allGlobalDeviceId), mRank(rank), mSize(size) {
    if (static_cast<int>(mIds.size()) != size || rank < 0 || rank >= size)
        throw std::invalid_argument("ThreadGroup: rank/size do not match the device list");
    mBackend = c10::make_intrusive<P2PBackend>(mComm, rank, size);
}

void* ThreadGroup::Stream() const { return CurrentStream(mComm->CudaDevice(mRank)); }

void ThreadGroup::CheckInput(const torch::Tensor& t) const {
    TORCH_CHECK(t.is_cuda(), "ThreadGroup: the B200 collectives take CUDA tensors (no CPU fallback)");
    TORCH_CHECK(t.get_device() == mComm->CudaDevice(mRank), "ThreadGroup: tensor on cuda:", t.get_device(),
                " but rank ", mRank, " runs on cuda:", mComm->CudaDevice(mRank));
}

void ThreadGroup::Barrier() { mBackend->barrier(); }

torch::Tensor ThreadGroup::AllReduce(const torch::Tensor& input, ReduceOpType) {
    CheckInput(input);
    torch::Tensor in = input.contiguous();
    torch::Tensor out = torch::empty_like(in);
    Check(dt_all_reduce(mComm->get(), mRank, in.data_ptr(), out.data_ptr(), static_cast<size_t>(in.numel()),
                        DTypeCode(in.scalar_type()), DT_SUM, DT_ACCUM_FP32, Stream()),
          "dt_all_reduce");
    return out;
}

torch::Tensor ThreadGroup::AllGatherIntoTensor(const torch::Tensor& input, const LocalShapes& operand) {
    return operand.IsEvenSplit() ? EqualShapeAllGatherIntoTensor(input) : AllGather(input, operand, 0);
}

torch::Tensor ThreadGroup::EqualShapeAllGatherIntoTensor(const torch::Tensor& input) {
    CheckInput(input);
    TORCH_CHECK(input.dim() > 0, "EqualShapeAllGatherIntoTensor: scalar input");
    torch::Tensor in = input.contiguous();
    auto shape = in.sizes().vec();
    const int64_t rows = shape[0];
    shape[0] *= mSize;
    torch::Tensor out = torch::empty(shape, in.options());
    std::vector<int64_t> lens(static_cast<size_t>(mSize), rows);
    const size_t inner = static_cast<size_t>(rows == 0 ? 0 : in.numel() / rows) * in.element_size();
    Check(dt_all_gather(mComm->get(), mRank, in.data_ptr(), out.data_ptr(), 1, lens.data(), inner, Stream()),
          "dt_all_gather");
    return out;
}

torch::Tensor ThreadGroup::AllGather(const torch::Tensor& input, const LocalShapes& operand, int64_t shardIndex) {
    CheckInput(input);
    torch::Tensor in = input.contiguous();
    auto shape = in.sizes().vec();
    const size_t d = static_cast<size_t>(shardIndex);
    TORCH_CHECK(d < shape.size(), "AllGather: shard dim out of range");
    std::vector<int64_t> lens;
    for (auto id : mIds) lens.push_back(operand.Get(id)[d]);
    TORCH_CHECK(lens[static_cast<size_t>(mRank)] == shape[d], "AllGather: local shape disagrees with the operand");
    const int64_t outer = Prod(shape, 0, d);
    const int64_t inner = Prod(shape, d + 1, shape.size()) * in.element_size();
    shape[d] = std::accumulate(lens.begin(), lens.end(), int64_t{0});
    torch::Tensor out = torch::empty(shape, in.options());
    Check(dt_all_gather(mComm->get(), mRank, in.data_ptr(), out.data_ptr(), static_cast<size_t>(outer), lens.data(),
                        static_cast<size_t>(inner), Stream()),
          "dt_all_gather");
    return out;
}

std::vector<torch::Tensor> ThreadGroup::AllGatherIntoVec(const torch::Tensor& input, const LocalShapes& operand) {
    CheckInput(input);
    torch::Tensor in = input.contiguous();
    std::vector<int64_t> lens;
    std::vector<std::vector<int64_t>> shapes;
    for (auto id : mIds) {
        shapes.push_back(operand.Get(id));
        lens.push_back(Prod(shapes.back(), 0, shapes.back().size()));
    }
    TORCH_CHECK(lens[static_cast<size_t>(mRank)] == in.numel(), "AllGatherIntoVec: local shape disagrees with the operand");
    const int64_t total = std::accumulate(lens.begin(), lens.end(), int64_t{0});
    torch::Tensor flat = torch::empty({total}, in.options());
    Check(dt_all_gather(mComm->get(), mRank, in.data_ptr(), flat.data_ptr(), 1, lens.data(),
                        static_cast<size_t>(in.element_size()), Stream()),
          "dt_all_gather");
    std::vector<torch::Tensor> out;
    int64_t off = 0;
    for (size_t r = 0; r < shapes.size(); ++r) {
        out.push_back(flat.narrow(0, off, lens[r]).view(shapes[r]));
        off += lens[r];
    }
    return out;
}

torch::Tensor ThreadGroup::ReduceScatterTensor(const torch::Tensor& input, ReduceOpType) {
    CheckInput(input);
    TORCH_CHECK(input.dim() > 0 && input.size(0) % mSize == 0,
                "ReduceScatterTensor: dim 0 must be divisible by the group size (as in the reference)");
    torch::Tensor in = input.contiguous();
    auto shape = in.sizes().vec();
    shape[0] /= mSize;
    torch::Tensor out = torch::empty(shape, in.options());
    Check(dt_reduce_scatter(mComm->get(), mRank, in.data_ptr(), out.data_ptr(), static_cast<size_t>(out.numel()),
                            DTypeCode(in.scalar_type()), DT_SUM, DT_ACCUM_FP32, Stream()),
          "dt_reduce_scatter");
    return out;
}

torch::Tensor ThreadGroup::AllToAll(const torch::Tensor& input, size_t srcDim, size_t destDim, const LocalShapes& operand) {
    CheckInput(input);
    torch::Tensor in = input.contiguous();
    auto shape = in.sizes().vec();
    TORCH_CHECK(srcDim < shape.size() && destDim < shape.size() && srcDim != destDim, "AllToAll: bad dims");
    std::vector<int64_t> srcLens;
    for (auto id : mIds) srcLens.push_back(operand.Get(id)[srcDim]);
    TORCH_CHECK(srcLens[static_cast<size_t>(mRank)] == shape[srcDim], "AllToAll: local shape disagrees with the operand");
    auto out_shape = shape;
    out_shape[srcDim] = std::accumulate(srcLens.begin(), srcLens.end(), int64_t{0});
    out_shape[destDim] = ShardSizes(shape[destDim], mSize)[static_cast<size_t>(mRank)];
    torch::Tensor out = torch::empty(out_shape, in.options());
    Check(dt_all_to_all(mComm->get(), mRank, in.data_ptr(), out.data_ptr(), static_cast<int>(shape.size()), shape.data(),
                        static_cast<int>(srcDim), static_cast<int>(destDim), srcLens.data(),
                        static_cast<size_t>(in.element_size()), Stream()),
          "dt_all_to_all");
    return out;
}

std::vector<torch::Tensor> ThreadGroup::AllToAllMulti(const std::vector<torch::Tensor>& inputs, size_t srcDim,
                                                      size_t destDim, const LocalShapes& operand) {
    TORCH_CHECK(!inputs.empty() && inputs.size() <= 8, "AllToAllMulti: 1..8 tensors");
    std::vector<torch::Tensor> ins;
    for (const auto& t : inputs) {
        CheckInput(t);
        TORCH_CHECK(t.sizes() == inputs[0].sizes() && t.scalar_type() == inputs[0].scalar_type(),
                    "AllToAllMulti: tensors must share shape and dtype");
        ins.push_back(t.contiguous());
    }
    auto shape = ins[0].sizes().vec();
    TORCH_CHECK(srcDim < shape.size() && destDim < shape.size() && srcDim != destDim, "AllToAllMulti: bad dims");
    std::vector<int64_t> srcLens;
    for (auto id : mIds) srcLens.push_back(operand.Get(id)[srcDim]);
    TORCH_CHECK(srcLens[static_cast<size_t>(mRank)] == shape[srcDim], "AllToAllMulti: local shape disagrees with the operand");
    auto out_shape = shape;
    out_shape[srcDim] = std::accumulate(srcLens.begin(), srcLens.end(), int64_t{0});
    out_shape[destDim] = ShardSizes(shape[destDim], mSize)[static_cast<size_t>(mRank)];
    std::vector<torch::Tensor> outs;
    std::vector<const void*> in_ptrs;
    std::vector<void*> out_ptrs;
    for (auto& t : ins) {
        outs.push_back(torch::empty(out_shape, t.options()));
        in_ptrs.push_back(t.data_ptr());
        out_ptrs.push_back(outs.back().data_ptr());
    }
    Check(dt_all_to_all_multi(mComm->get(), mRank, static_cast<int>(ins.size()), in_ptrs.data(), out_ptrs.data(),
                              static_cast<int>(shape.size()), shape.data(), static_cast<int>(srcDim),
                              static_cast<int>(destDim), srcLens.data(), static_cast<size_t>(ins[0].element_size()),
                              Stream()),
          "dt_all_to_all_multi");
    return outs;
}

torch::Tensor ThreadGroup::ReplicateToShard(const torch::Tensor& input, int64_t shardIdx, int64_t subSplitCoordinates) {
    TORCH_CHECK(shardIdx >= 0 && shardIdx < input.dim(), "ReplicateToShard: shard dim out of range");
    const int64_t len = input.size(shardIdx);
    if (subSplitCoordinates < 0) {
        auto sizes = ShardSizes(len, mSize);
        return torch::split_with_sizes(input, sizes, shardIdx)[static_cast<size_t>(mRank)];
    }
    TORCH_CHECK(subSplitCoordinates > 0 && subSplitCoordinates < len, "Invalid subSplitCoordinates: ",
                subSplitCoordinates, " and sizeInShardDim: ", len);
    auto two = torch::split_with_sizes(input, {subSplitCoordinates + 1, len - subSplitCoordinates - 1}, shardIdx);
    auto front = torch::split_with_sizes(two[0], ShardSizes(subSplitCoordinates + 1, mSize), shardIdx);
    auto back = torch::split_with_sizes(two[1], ShardSizes(len - subSplitCoordinates - 1, mSize), shardIdx);
    return torch::cat({front[static_cast<size_t>(mRank)], back[static_cast<size_t>(mRank)]}, shardIdx);
}

// ---------------------------------------------------------------------------------------------------------
// ThreadGroupManager
// ---------------------------------------------------------------------------------------------------------
ThreadGroupManager& ThreadGroupManager::Global() {
    static ThreadGroupManager m;
    return m;
}

ThreadGroup& ThreadGroupManager::GetThreadGroup(const std::vector<int64_t>& allDeviceId, int64_t currentDeviceId) {
    const int size = static_cast<int>(allDeviceId.size());
    const int rank = static_cast<int>(RankOf(currentDeviceId, allDeviceId));
    std::lock_guard<std::mutex> lock(mMutex);
    auto& entry = mGroups[allDeviceId];
    if (!entry) {
        entry = std::make_unique<Entry>();
        std::vector<int> devices;
        for (auto id : allDeviceId) devices.push_back(CudaDeviceOf(id));
        entry->comm = std::make_shared<SharedComm>(devices);
        entry->ranks.resize(static_cast<size_t>(size));
    }
    auto& tg = entry->ranks[static_cast<size_t>(rank)];
    if (!tg) tg = std::make_unique<ThreadGroup>(entry->comm, allDeviceId, rank, size);
    return *tg;
}

void ThreadGroupManager::Clear() {
    std::lock_guard<std::mutex> lock(mMutex);
    mGroups.clear();
}

}  // namespace dtb
