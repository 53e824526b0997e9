// Redistribute executor: per-device kernel-stream threads and the per-mesh-dim conversion plan.
//
//   KernelStream        one host thread + one CUDA stream per global device (the reference's KernelStream,
//                       dtorch/core/kernel_stream/kernel_stream.cc:41-104, CudaKernelStream::InitInAsyncThread
//                       cuda_kernel_stream.cc:25-58); tasks run in order with the stream current.
//   ConvertPlacements   one mesh dim, one device: build the group along the dim and dispatch to the
//                       ThreadGroup collective (ConvertKernel::ConvertPlacements, convert_kernel.cc:104-185).
//   Redistribute        normalise placements, order the changed mesh dims (GetConvertOrder) and run one
//                       ConvertPlacements per dim on every device's thread (ConvertOpImpl::RunFunc /
//                       ConvertPlacementsOneByOne, dtorch/api/cpp/functional/implement/convert_op_impl.cc:19-66).
#pragma once

#include <c10/cuda/CUDAStream.h>
#include <c10/util/Optional.h>

#include <condition_variable>
#include <deque>
#include <functional>
#include <atomic>
#include <exception>
#include <map>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include <torch/torch.h>

#include "placement.h"
#include "thread_group.h"

namespace dtb {

// Completion of a set of tasks posted to kernel streams: the poster waits for all of them (spinning first --
// a task takes microseconds and a futex wake-up would cost as much) and gets the first exception back.
class TaskBatch {
public:
    explicit TaskBatch(int n) : mLeft(n) {}
    void Done(std::exception_ptr e);
    void Wait();  // rethrows the first task's exception

private:
    std::atomic<int> mLeft;
    std::mutex mMutex;
    std::exception_ptr mErr;
};

class KernelStream {
public:
    KernelStream(int64_t globalDeviceId, int cudaDevice);
    ~KernelStream();
    KernelStream(const KernelStream&) = delete;
    KernelStream& operator=(const KernelStream&) = delete;

    // Run a task on this stream's thread, in order, with the device current and `stream` (default: this
    // KernelStream's own stream) as the current CUDA stream; report to `batch` when done.
    void Post(std::function<void()> task, TaskBatch* batch, c10::optional<c10::cuda::CUDAStream> stream = c10::nullopt);
    c10::cuda::CUDAStream Stream() const { return mStream; }
    int CudaDevice() const { return mCudaDevice; }

private:
    struct Item {
        std::function<void()> fn;
        TaskBatch* batch;
        c10::optional<c10::cuda::CUDAStream> stream;
    };
    void Main();

    int64_t mGlobalDeviceId;
    int mCudaDevice;
    c10::cuda::CUDAStream mStream;
    std::mutex mMutex;
    std::condition_variable mCv;
    std::deque<Item> mQueue;
    std::atomic<int> mPending{0};
    bool mSleeping = false;
    bool mStop = false;
    std::thread mThread;
};

class KernelStreamManager {
public:
    static KernelStreamManager& Global();
    KernelStream& Get(int64_t globalDeviceId);
    void Clear();

private:
    std::mutex mMutex;
    std::map<int64_t, std::unique_ptr<KernelStream>> mStreams;
};

// One mesh-dim conversion on one device (runs on that device's KernelStream thread).
torch::Tensor ConvertPlacements(const torch::Tensor& input, const DeviceMesh& mesh, size_t meshDim, const Placement& src,
                                const Placement& dst, int64_t deviceId, const LocalShapes& operand);

// Redistribute a DTensor given as per-device local tensors (global device id -> tensor on that device).
// Returns the new local tensors, stream-ordered after the caller's current stream on each device and safe
// to use on it.
// With handoff = false the results stay ordered on each device's kernel stream only (the caller's stream is not
// made to wait); the caller orders its consumers itself (an event recorded on KernelStream::Stream() right
// after the call returns covers the call's work) -- this is how compute overlaps a later collective.
std::map<int64_t, torch::Tensor> Redistribute(const std::map<int64_t, torch::Tensor>& locals, const DeviceMesh& mesh,
                                              PlacementSeq src, PlacementSeq dst, const std::vector<int64_t>& globalShape,
                                              bool handoff = true);

// Redistribute several DTensors of one shape and placement the same way. A change of one mesh dim from
// Shard(i) to Shard(j) runs as one fused all-to-all launch per device for all of them (the q/k/v swap of
// Ulysses context parallelism); anything else runs Redistribute per tensor.
std::vector<std::map<int64_t, torch::Tensor>> RedistributeMulti(const std::vector<std::map<int64_t, torch::Tensor>>& locals,
                                                                const DeviceMesh& mesh, PlacementSeq src, PlacementSeq dst,
                                                                const std::vector<int64_t>& globalShape,
                                                                bool handoff = true);

}  // namespace dtb
