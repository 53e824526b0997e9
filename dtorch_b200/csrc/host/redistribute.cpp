// Redistribute executor (see redistribute.h).
#include "redistribute.h"

#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <stdexcept>
#include <thread>

namespace dtb {

// ---------------------------------------------------------------------------------------------------------
// KernelStream
// ---------------------------------------------------------------------------------------------------------
namespace {

// How long an idle kernel-stream thread, or a poster waiting for its tasks, spins before sleeping:
// DTORCH_B200_SPIN_US, default 2000 us (a redistribute posts its next tasks well within that).
int64_t SpinNs() {
    static const int64_t v = [] {
        const char* s = std::getenv("DTORCH_B200_SPIN_US");
        const long long us = (s != nullptr && *s != '\0') ? std::atoll(s) : 2000;
        return static_cast<int64_t>(std::max<long long>(us, 0)) * 1000;
    }();
    return v;
}

inline void CpuRelax() {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_ia32_pause();
#else
    std::this_thread::yield();
#endif
}

}  // namespace

void TaskBatch::Done(std::exception_ptr e) {
    if (e) {
        std::lock_guard<std::mutex> lock(mMutex);
        if (!mErr) mErr = e;
    }
    mLeft.fetch_sub(1, std::memory_order_acq_rel);
}

void TaskBatch::Wait() {
    const auto t0 = std::chrono::steady_clock::now();
    uint32_t spins = 0;
    while (mLeft.load(std::memory_order_acquire) > 0) {
        if ((++spins & 255u) == 0 &&
            std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count() > SpinNs()) {
            std::this_thread::sleep_for(std::chrono::microseconds(20));
        } else {
            CpuRelax();
        }
    }
    std::lock_guard<std::mutex> lock(mMutex);
    if (mErr) std::rethrow_exception(mErr);
}

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

void KernelStream::Post(std::function<void()> task, TaskBatch* batch, c10::optional<c10::cuda::CUDAStream> stream) {
    bool wake = false;
    {
        std::lock_guard<std::mutex> lock(mMutex);
        if (mStop) throw std::runtime_error("KernelStream is shutting down");
        mQueue.push_back(Item{std::move(task), batch, stream});
        mPending.fetch_add(1, std::memory_order_release);
        wake = mSleeping;
    }
    if (wake) mCv.notify_one();
}

void KernelStream::Main() {
    c10::cuda::CUDAGuard device_guard(static_cast<c10::DeviceIndex>(mCudaDevice));
    c10::cuda::CUDAStreamGuard stream_guard(mStream);
    while (true) {
        // spin a while for the next task (a redistribute posts one per mesh dim in quick succession), then sleep
        const auto t0 = std::chrono::steady_clock::now();
        uint32_t spins = 0;
        while (mPending.load(std::memory_order_acquire) == 0) {
            if ((++spins & 255u) == 0 &&
                std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count() >
                    SpinNs())
                break;
            CpuRelax();
        }
        Item item;
        {
            std::unique_lock<std::mutex> lock(mMutex);
            mSleeping = true;
            mCv.wait(lock, [&] { return mStop || !mQueue.empty(); });
            mSleeping = false;
            if (mQueue.empty()) return;  // stopping and drained
            item = std::move(mQueue.front());
            mQueue.pop_front();
            mPending.fetch_sub(1, std::memory_order_relaxed);
        }
        std::exception_ptr err;
        try {
            if (item.stream) {
                c10::cuda::CUDAStreamGuard g(*item.stream);
                item.fn();
            } else {
                item.fn();
            }
        } catch (...) {
            err = std::current_exception();
        }
        if (item.batch != nullptr) item.batch->Done(err);
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
namespace {

// Where each device's part of a redistribute runs. handoff (the default): on the caller's current stream of that
// device, so results are stream-ordered for the caller with no events at all. Otherwise on the device's own
// kernel stream, ordered after the caller's work by an event and not handed back.
struct StreamPlan {
    bool onCaller;
    std::map<int64_t, c10::cuda::CUDAStream> caller;
    std::map<int64_t, std::shared_ptr<at::cuda::CUDAEvent>> ready;

    StreamPlan(const DeviceMesh& mesh, bool handoff) : onCaller(handoff) {
        for (auto id : mesh.ids) {
            auto& ks = KernelStreamManager::Global().Get(id);
            auto cs = c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(ks.CudaDevice()));
            caller.emplace(id, cs);
            if (!onCaller) {
                auto ev = std::make_shared<at::cuda::CUDAEvent>();
                ev->record(cs);
                ready[id] = ev;
            }
        }
    }
    c10::optional<c10::cuda::CUDAStream> StreamFor(int64_t id) const {
        if (onCaller) return caller.at(id);
        return c10::nullopt;
    }
    // first task on a kernel stream: wait for the caller's work; inputs consumed on that stream stay alive
    void Enter(int64_t id, bool first, const std::vector<torch::Tensor>& ins) const {
        if (onCaller) return;
        auto stream = c10::cuda::getCurrentCUDAStream();
        if (first) ready.at(id)->block(stream);
        for (const auto& in : ins)
            if (in.defined() && in.is_cuda()) c10::cuda::CUDACachingAllocator::recordStream(in.storage().data_ptr(), stream);
    }
};

}  // namespace

std::map<int64_t, torch::Tensor> Redistribute(const std::map<int64_t, torch::Tensor>& locals, const DeviceMesh& mesh,
                                              PlacementSeq src, PlacementSeq dst, const std::vector<int64_t>& globalShape,
                                              bool handoff) {
    ShardDimToPositive(src, globalShape.size());
    ShardDimToPositive(dst, globalShape.size());
    ToReplicateWhenDimSizeEqualOne(src, mesh);
    ToReplicateWhenDimSizeEqualOne(dst, mesh);
    CheckValid(globalShape, mesh, src);
    CheckValid(globalShape, mesh, dst);
    for (auto id : mesh.ids)
        TORCH_CHECK(locals.count(id) == 1, "Redistribute: no local tensor for device ", id);
    const auto order = GetConvertOrder(src, dst);
    if (order.empty()) return locals;
    const StreamPlan plan(mesh, handoff);

    std::map<int64_t, torch::Tensor> cur = locals;
    PlacementSeq cur_p = src;
    bool first = true;
    for (size_t d : order) {
        PlacementSeq next = cur_p;
        next[d] = dst[d];
        LocalShapes operand;
        operand.shapes = ComputeLocalShapes(globalShape, mesh, cur_p);
        std::map<int64_t, torch::Tensor> out;
        for (auto id : mesh.ids) out[id] = torch::Tensor();
        TaskBatch batch(static_cast<int>(mesh.ids.size()));
        for (auto id : mesh.ids) {
            torch::Tensor in = cur.at(id);
            const Placement s = cur_p[d], t = next[d];
            torch::Tensor* slot = &out[id];
            KernelStreamManager::Global().Get(id).Post(
                [&, in, s, t, id, d, slot, first]() {
                    plan.Enter(id, first, {in});
                    *slot = ConvertPlacements(in, mesh, d, s, t, id, operand);
                },
                &batch, plan.StreamFor(id));
        }
        batch.Wait();
        cur = std::move(out);
        cur_p = next;
        first = false;
    }
    return cur;
}

std::vector<std::map<int64_t, torch::Tensor>> RedistributeMulti(const std::vector<std::map<int64_t, torch::Tensor>>& locals,
                                                                const DeviceMesh& mesh, PlacementSeq src, PlacementSeq dst,
                                                                const std::vector<int64_t>& globalShape, bool handoff) {
    ShardDimToPositive(src, globalShape.size());
    ShardDimToPositive(dst, globalShape.size());
    ToReplicateWhenDimSizeEqualOne(src, mesh);
    ToReplicateWhenDimSizeEqualOne(dst, mesh);
    const auto diff = GetDiffDims(src, dst);
    const bool fused = locals.size() > 1 && locals.size() <= 8 && diff.size() == 1 && src[diff[0]].IsShard() &&
                       dst[diff[0]].IsShard() && !src[diff[0]].HasSubSplit() && !dst[diff[0]].HasSubSplit();
    if (!fused) {
        std::vector<std::map<int64_t, torch::Tensor>> out;
        for (const auto& l : locals) out.push_back(Redistribute(l, mesh, src, dst, globalShape, handoff));
        return out;
    }
    CheckValid(globalShape, mesh, src);
    CheckValid(globalShape, mesh, dst);
    const size_t d = diff[0];
    LocalShapes operand;
    operand.shapes = ComputeLocalShapes(globalShape, mesh, src);
    const StreamPlan plan(mesh, handoff);
    std::vector<std::map<int64_t, torch::Tensor>> out(locals.size());
    std::map<int64_t, std::vector<torch::Tensor>> results;
    for (auto id : mesh.ids) results[id] = {};
    TaskBatch batch(static_cast<int>(mesh.ids.size()));
    for (auto id : mesh.ids) {
        std::vector<torch::Tensor> ins;
        for (const auto& l : locals) ins.push_back(l.at(id));
        std::vector<torch::Tensor>* slot = &results[id];
        KernelStreamManager::Global().Get(id).Post(
            [&, ins, id, slot]() {
                plan.Enter(id, true, ins);
                const auto group = GroupDeviceIds(mesh, d, id);
                ThreadGroup& tg = ThreadGroupManager::Global().GetThreadGroup(group, id);
                *slot = tg.AllToAllMulti(ins, static_cast<size_t>(src[d].dim), static_cast<size_t>(dst[d].dim), operand);
            },
            &batch, plan.StreamFor(id));
    }
    batch.Wait();
    for (auto id : mesh.ids)
        for (size_t t = 0; t < out.size(); ++t) out[t][id] = results[id][t];
    return out;
}

}  // namespace dtb
