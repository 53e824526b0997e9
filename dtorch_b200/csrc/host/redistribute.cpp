// Redistribute executor (see redistribute.h).
#include "redistribute.h"

#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>
#include <stdexcept>

namespace dtb {

// ---------------------------------------------------------------------------------------------------------
// KernelStream
// ---------------------------------------------------------------------------------------------------------
KernelStream::KernelStream(int64_t globalDeviceId, int cudaDevice)
    : mGlobalDeviceId(globalDeviceId),
      mCudaDevice(cudaDevice),
      mStream(c10::cuda::getStreamFromPool(/*isHighPriority=*/true, static_cast<c10::DeviceIndex>(cudaDevice))) {
    mThread = std::thread(&KernelStream::Main, this);
}

KernelStream::~KernelStream() {
    {
        std::lock_guard<std::mutex> lock(mMutex);
        mStop = true;
    }
    mCv.notify_all();
    if (mThread.joinable()) mThread.join();
}

std::future<void> KernelStream::Launch(std::function<void()> task) {
    std::packaged_task<void()> pt(std::move(task));
    auto fut = pt.get_future();
    {
        std::lock_guard<std::mutex> lock(mMutex);
        if (mStop) throw std::runtime_error("KernelStream is shutting down");
        mQueue.push_back(std::move(pt));
    }
    mCv.notify_one();
    return fut;
}

void KernelStream::Main() {
    c10::cuda::CUDAGuard device_guard(static_cast<c10::DeviceIndex>(mCudaDevice));
    c10::cuda::CUDAStreamGuard stream_guard(mStream);
    while (true) {
        std::packaged_task<void()> task;
        {
            std::unique_lock<std::mutex> lock(mMutex);
            mCv.wait(lock, [&] { return mStop || !mQueue.empty(); });
            if (mQueue.empty()) return;  // stopping and drained
            task = std::move(mQueue.front());
            mQueue.pop_front();
        }
        task();  // exceptions land in the future
    }
}

KernelStreamManager& KernelStreamManager::Global() {
    static KernelStreamManager m;
    return m;
}

KernelStream& KernelStreamManager::Get(int64_t globalDeviceId) {
    std::lock_guard<std::mutex> lock(mMutex);
    auto& ks = mStreams[globalDeviceId];
    if (!ks) ks = std::make_unique<KernelStream>(globalDeviceId, CudaDeviceOf(globalDeviceId));
    return *ks;
}

void KernelStreamManager::Clear() {
    std::lock_guard<std::mutex> lock(mMutex);
    mStreams.clear();
}

// ---------------------------------------------------------------------------------------------------------
// Conversion of one mesh dim
// ---------------------------------------------------------------------------------------------------------
namespace {

bool PreCollectiveBarrier() {
    const char* s = std::getenv("DTORCH_B200_PRECOLLECTIVE_BARRIER");
    return s != nullptr && std::string(s) == "1";
}

}  // namespace

torch::Tensor ConvertPlacements(const torch::Tensor& input, const DeviceMesh& mesh, size_t meshDim, const Placement& src,
                                const Placement& dst, int64_t deviceId, const LocalShapes& operand) {
    const auto group = GroupDeviceIds(mesh, meshDim, deviceId);
    ThreadGroup& tg = ThreadGroupManager::Global().GetThreadGroup(group, deviceId);
    if (PreCollectiveBarrier()) tg.Barrier();  // the reference always barriers here (convert_kernel.cc:146)
    if (src.IsShard() && dst.IsShard()) {
        TORCH_CHECK(!src.HasSubSplit() && !dst.HasSubSplit(), "Shard -> Shard with sub-split placements is unsupported "
                    "(as in the reference, convert_kernel.cc:149-150)");
        return tg.AllToAll(input, static_cast<size_t>(src.dim), static_cast<size_t>(dst.dim), operand);
    }
    if (src.IsShard() && dst.IsReplicate()) {
        if (!src.HasSubSplit()) return src.dim == 0 ? tg.AllGatherIntoTensor(input, operand) : tg.AllGather(input, operand, src.dim);
        // one launch places every rank's front and back pieces (the reference gathers, then concatenates twice)
        return tg.AllGatherSubSplit(input, operand, src.dim, src.subSplit);
    }
    if (src.IsReplicate() && dst.IsShard()) return tg.ReplicateToShard(input, dst.dim, dst.subSplit);
    if (src.IsPartial() && dst.IsShard(0)) return tg.ReduceScatterTensor(input);
    if (src.IsPartial() && dst.IsReplicate()) return tg.AllReduce(input);
    throw std::invalid_argument("unsupported placement change: " + src.ToString() + " -> " + dst.ToString());
}

// ---------------------------------------------------------------------------------------------------------
// Redistribute
// ---------------------------------------------------------------------------------------------------------
std::map<int64_t, torch::Tensor> Redistribute(const std::map<int64_t, torch::Tensor>& locals, const DeviceMesh& mesh,
                                              PlacementSeq src, PlacementSeq dst, const std::vector<int64_t>& globalShape) {
    ShardDimToPositive(src, globalShape.size());
    ShardDimToPositive(dst, globalShape.size());
    ToReplicateWhenDimSizeEqualOne(src, mesh);
    ToReplicateWhenDimSizeEqualOne(dst, mesh);
    CheckValid(globalShape, mesh, src);
    CheckValid(globalShape, mesh, dst);
    for (auto id : mesh.ids)
        TORCH_CHECK(locals.count(id) == 1, "Redistribute: no local tensor for device ", id);

    // order every device's kernel stream after the work already queued on the caller's stream
    std::map<int64_t, std::shared_ptr<at::cuda::CUDAEvent>> ready;
    for (auto id : mesh.ids) {
        auto& ks = KernelStreamManager::Global().Get(id);
        auto ev = std::make_shared<at::cuda::CUDAEvent>();
        ev->record(c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(ks.CudaDevice())));
        ready[id] = ev;
    }

    std::map<int64_t, torch::Tensor> cur = locals;
    PlacementSeq cur_p = src;
    bool first = true;
    for (size_t d : GetConvertOrder(src, dst)) {
        PlacementSeq next = cur_p;
        next[d] = dst[d];
        LocalShapes operand;
        operand.shapes = ComputeLocalShapes(globalShape, mesh, cur_p);
        std::map<int64_t, torch::Tensor> out;
        std::map<int64_t, std::future<void>> futs;
        std::mutex out_mu;
        for (auto id : mesh.ids) {
            auto& ks = KernelStreamManager::Global().Get(id);
            torch::Tensor in = cur.at(id);
            std::shared_ptr<at::cuda::CUDAEvent> ev = first ? ready.at(id) : nullptr;
            const Placement s = cur_p[d], t = next[d];
            futs[id] = ks.Launch([&, in, ev, s, t, id, d]() {
                auto stream = c10::cuda::getCurrentCUDAStream();
                if (ev) ev->block(stream);
                // the input is consumed on this stream; keep its memory until this stream is done with it
                if (in.defined() && in.is_cuda()) c10::cuda::CUDACachingAllocator::recordStream(in.storage().data_ptr(), stream);
                torch::Tensor r = ConvertPlacements(in, mesh, d, s, t, id, operand);
                std::lock_guard<std::mutex> g(out_mu);
                out[id] = r;
            });
        }
        std::exception_ptr err;
        for (auto& kv : futs) {
            try {
                kv.second.get();
            } catch (...) {
                if (!err) err = std::current_exception();
            }
        }
        if (err) std::rethrow_exception(err);
        cur = std::move(out);
        cur_p = next;
        first = false;
    }
    if (first) return cur;  // nothing to convert
    // hand the results back to the caller's stream
    for (auto id : mesh.ids) {
        auto& ks = KernelStreamManager::Global().Get(id);
        auto caller = c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(ks.CudaDevice()));
        at::cuda::CUDAEvent done;
        done.record(ks.Stream());
        done.block(caller);
        auto& t = cur.at(id);
        if (t.defined() && t.is_cuda()) c10::cuda::CUDACachingAllocator::recordStream(t.storage().data_ptr(), caller);
    }
    return cur;
}

std::vector<std::map<int64_t, torch::Tensor>> RedistributeMulti(const std::vector<std::map<int64_t, torch::Tensor>>& locals,
                                                                const DeviceMesh& mesh, PlacementSeq src, PlacementSeq dst,
                                                                const std::vector<int64_t>& globalShape) {
    ShardDimToPositive(src, globalShape.size());
    ShardDimToPositive(dst, globalShape.size());
    ToReplicateWhenDimSizeEqualOne(src, mesh);
    ToReplicateWhenDimSizeEqualOne(dst, mesh);
    const auto diff = GetDiffDims(src, dst);
    const bool fused = locals.size() > 1 && locals.size() <= 8 && diff.size() == 1 && src[diff[0]].IsShard() &&
                       dst[diff[0]].IsShard() && !src[diff[0]].HasSubSplit() && !dst[diff[0]].HasSubSplit();
    if (!fused) {
        std::vector<std::map<int64_t, torch::Tensor>> out;
        for (const auto& l : locals) out.push_back(Redistribute(l, mesh, src, dst, globalShape));
        return out;
    }
    CheckValid(globalShape, mesh, src);
    CheckValid(globalShape, mesh, dst);
    const size_t d = diff[0];
    LocalShapes operand;
    operand.shapes = ComputeLocalShapes(globalShape, mesh, src);
    std::vector<std::map<int64_t, torch::Tensor>> out(locals.size());
    std::map<int64_t, std::future<void>> futs;
    std::mutex out_mu;
    for (auto id : mesh.ids) {
        auto& ks = KernelStreamManager::Global().Get(id);
        std::vector<torch::Tensor> ins;
        for (const auto& l : locals) ins.push_back(l.at(id));
        auto ev = std::make_shared<at::cuda::CUDAEvent>();
        ev->record(c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(ks.CudaDevice())));
        futs[id] = ks.Launch([&, ins, ev, id]() {
            auto stream = c10::cuda::getCurrentCUDAStream();
            ev->block(stream);
            for (const auto& t : ins) c10::cuda::CUDACachingAllocator::recordStream(t.storage().data_ptr(), stream);
            const auto group = GroupDeviceIds(mesh, d, id);
            ThreadGroup& tg = ThreadGroupManager::Global().GetThreadGroup(group, id);
            auto r = tg.AllToAllMulti(ins, static_cast<size_t>(src[d].dim), static_cast<size_t>(dst[d].dim), operand);
            std::lock_guard<std::mutex> g(out_mu);
            for (size_t t = 0; t < r.size(); ++t) out[t][id] = r[t];
        });
    }
    std::exception_ptr err;
    for (auto& kv : futs) {
        try {
            kv.second.get();
        } catch (...) {
            if (!err) err = std::current_exception();
        }
    }
    if (err) std::rethrow_exception(err);
    for (auto id : mesh.ids) {
        auto& ks = KernelStreamManager::Global().Get(id);
        auto caller = c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(ks.CudaDevice()));
        at::cuda::CUDAEvent done;
        done.record(ks.Stream());
        done.block(caller);
        for (auto& o : out) c10::cuda::CUDACachingAllocator::recordStream(o.at(id).storage().data_ptr(), caller);
    }
    return out;
}

}  // namespace dtb
