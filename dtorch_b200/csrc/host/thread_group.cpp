// ThreadGroup / P2PBackend / ThreadGroupManager over the C ABI (see thread_group.h).
#include "thread_group.h"

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <atomic>
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

namespace {
std::atomic<int64_t> gPoolBytesOverride{-1};
}  // namespace

size_t PoolBytes() {
    const int64_t o = gPoolBytesOverride.load();
    if (o >= 0) return static_cast<size_t>(o);
    const char* s = std::getenv("DTORCH_B200_POOL_MB");
    if (s == nullptr || *s == '\0') return 0;
    const long long mb = std::atoll(s);
    return mb > 0 ? static_cast<size_t>(mb) << 20 : 0;
}

void SetPoolBytes(size_t bytes) { gPoolBytesOverride.store(static_cast<int64_t>(bytes)); }

SharedComm::SharedComm(const std::vector<int>& cudaDevices, size_t poolBytes) : mDevices(cudaDevices) {
    const int n = static_cast<int>(cudaDevices.size());
    bool distinct = n > 1;
    for (int i = 1; i < n; ++i) distinct = distinct && cudaDevices[static_cast<size_t>(i)] != cudaDevices[0];
    Check(dt_comm_create(n, cudaDevices.data(), 0, &mComm), "dt_comm_create");
    const char* t = std::getenv("DTORCH_COMM_TIMEOUT_SECOND");
    if (t != nullptr && std::atoll(t) > 0) Check(dt_comm_set_timeout_ms(mComm, std::atoll(t) * 1000), "dt_comm_set_timeout_ms");
    if (poolBytes == 0 || !distinct || dt_comm_same_device(mComm)) return;
    // the symmetric pool: the NVLS buffer where the switch supports it (all-reduces on it reduce in the
    // switch), else a symmetric heap of the same size
    int nvls = 0;
    bool use_nvls = dt_comm_nvls_supported(mComm, &nvls) == DT_OK && nvls && dt_comm_nvls_alloc(mComm, poolBytes) == DT_OK;
    if (!use_nvls) {
        dt_comm_destroy(mComm);
        mComm = nullptr;
        Check(dt_comm_create(n, cudaDevices.data(), poolBytes, &mComm), "dt_comm_create");
        if (t != nullptr && std::atoll(t) > 0) Check(dt_comm_set_timeout_ms(mComm, std::atoll(t) * 1000), "dt_comm_set_timeout_ms");
    }
    std::vector<char*> bases;
    size_t bytes = 0;
    for (int r = 0; r < n; ++r) {
        void* base = nullptr;
        size_t b = 0;
        Check(use_nvls ? dt_comm_nvls_buffer(mComm, r, &base, &b) : dt_comm_heap(mComm, r, &base, &b), "pool base");
        bases.push_back(static_cast<char*>(base));
        bytes = (r == 0) ? b : std::min(bytes, b);
    }
    mPool = std::make_unique<SymmetricPool>(cudaDevices, bases, bytes, use_nvls);
}

SharedComm::~SharedComm() {
    mPool.reset();
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
        std::vector<void*> out_ptrs;
        std::vector<size_t> room;
        for (auto& o : outs) {
            TORCH_CHECK(o.is_contiguous(), "allgather: contiguous outputs");
            out_ptrs.push_back(o.data_ptr());
            room.push_back(static_cast<size_t>(o.nbytes()));
        }
        // every rank's input lands in its own output tensor of every rank, in one launch
        Check(dt_all_gather_list(comm(), getRank(), in.data_ptr(), static_cast<size_t>(in.nbytes()), out_ptrs.data(),
                                 room.data(), CurrentStream(cudaDevice())),
              "dt_all_gather_list");
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
    // inputs[k] goes to rank k, outputs[k] receives rank k's chunk: one launch of peer stores, no cat / copy
    std::vector<at::Tensor> ins;
    std::vector<const void*> in_ptrs;
    std::vector<void*> out_ptrs;
    std::vector<size_t> in_bytes, room;
    for (int k = 0; k < n; ++k) {
        ins.push_back(inputs[k].contiguous());
        TORCH_CHECK(outputs[k].is_contiguous(), "alltoall: contiguous outputs");
        in_ptrs.push_back(ins.back().data_ptr());
        in_bytes.push_back(static_cast<size_t>(ins.back().nbytes()));
        out_ptrs.push_back(outputs[k].data_ptr());
        room.push_back(static_cast<size_t>(outputs[k].nbytes()));
    }
    Check(dt_all_to_all_list(comm(), getRank(), in_ptrs.data(), in_bytes.data(), out_ptrs.data(), room.data(),
                             CurrentStream(cudaDevice())),
          "dt_all_to_all_list");
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

torch::Tensor ThreadGroup::NewOutput(at::IntArrayRef shape, const at::TensorOptions& opts, size_t bytesAllRanks) {
    if (SymmetricPool* pool = mComm->Pool()) {
        torch::Tensor t = pool->Empty(mRank, shape, opts, bytesAllRanks, static_cast<cudaStream_t>(Stream()), mComm);
        if (t.defined()) return t;
    }
    return torch::empty(shape, opts);
}

void ThreadGroup::CheckInput(const torch::Tensor& t) const {
    TORCH_CHECK(t.is_cuda(), "ThreadGroup: the B200 collectives take CUDA tensors (no CPU fallback)");
    TORCH_CHECK(t.get_device() == mComm->CudaDevice(mRank), "ThreadGroup: tensor on cuda:", t.get_device(),
                " but rank ", mRank, " runs on cuda:", mComm->CudaDevice(mRank));
}

void ThreadGroup::Barrier() { mBackend->barrier(); }

torch::Tensor ThreadGroup::AllReduce(const torch::Tensor& input, ReduceOpType) {
    CheckInput(input);
    torch::Tensor in = input.contiguous();
    torch::Tensor out = NewOutput(in.sizes(), in.options(), static_cast<size_t>(in.nbytes()));
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
    torch::Tensor out = NewOutput(shape, in.options(), static_cast<size_t>(in.nbytes()) * static_cast<size_t>(mSize));
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
    torch::Tensor out = NewOutput(shape, in.options(), static_cast<size_t>(Prod(shape, 0, shape.size()) * in.element_size()));
    Check(dt_all_gather(mComm->get(), mRank, in.data_ptr(), out.data_ptr(), static_cast<size_t>(outer), lens.data(),
                        static_cast<size_t>(inner), Stream()),
          "dt_all_gather");
    return out;
}

torch::Tensor ThreadGroup::AllGatherSubSplit(const torch::Tensor& input, const LocalShapes& operand, int64_t shardIndex,
                                             int64_t subSplit) {
    CheckInput(input);
    torch::Tensor in = input.contiguous();
    auto shape = in.sizes().vec();
    const size_t d = static_cast<size_t>(shardIndex);
    TORCH_CHECK(d < shape.size(), "AllGatherSubSplit: shard dim out of range");
    std::vector<int64_t> lens;
    for (auto id : mIds) lens.push_back(operand.Get(id)[d]);
    TORCH_CHECK(lens[static_cast<size_t>(mRank)] == shape[d], "AllGatherSubSplit: local shape disagrees with the operand");
    // rank i's front piece: its share of the first subSplit + 1 rows (the reference's splitSize,
    // distributed_scather_and_gather.cc:166-170)
    const auto fronts = ShardSizes(subSplit + 1, mSize);
    for (size_t i = 0; i < lens.size(); ++i)
        TORCH_CHECK(fronts[i] < lens[i], "sub-split piece smaller than its front part");
    const int64_t outer = Prod(shape, 0, d);
    const int64_t inner = Prod(shape, d + 1, shape.size()) * in.element_size();
    shape[d] = std::accumulate(lens.begin(), lens.end(), int64_t{0});
    torch::Tensor out = NewOutput(shape, in.options(), static_cast<size_t>(Prod(shape, 0, shape.size()) * in.element_size()));
    Check(dt_all_gather_sub_split(mComm->get(), mRank, in.data_ptr(), out.data_ptr(), static_cast<size_t>(outer),
                                  lens.data(), fronts.data(), static_cast<size_t>(inner), Stream()),
          "dt_all_gather_sub_split");
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
    torch::Tensor flat = NewOutput({total}, in.options(), static_cast<size_t>(total * in.element_size()));
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
    torch::Tensor out = NewOutput(shape, in.options(), static_cast<size_t>(in.nbytes()) / static_cast<size_t>(mSize));
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
    const auto destSplit = ShardSizes(shape[destDim], mSize);
    out_shape[destDim] = destSplit[static_cast<size_t>(mRank)];
    auto max_shape = out_shape;
    max_shape[destDim] = destSplit[0];  // the first ranks get the larger chunk
    torch::Tensor out = NewOutput(out_shape, in.options(),
                                  static_cast<size_t>(Prod(max_shape, 0, max_shape.size()) * in.element_size()));
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
    const auto destSplit = ShardSizes(shape[destDim], mSize);
    out_shape[destDim] = destSplit[static_cast<size_t>(mRank)];
    auto max_shape = out_shape;
    max_shape[destDim] = destSplit[0];
    const size_t max_bytes = static_cast<size_t>(Prod(max_shape, 0, max_shape.size()) * ins[0].element_size());
    std::vector<torch::Tensor> outs;
    std::vector<const void*> in_ptrs;
    std::vector<void*> out_ptrs;
    for (auto& t : ins) {
        outs.push_back(NewOutput(out_shape, t.options(), max_bytes));
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
        entry->comm = std::make_shared<SharedComm>(devices, PoolBytes());
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
