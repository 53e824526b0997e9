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

#include <condition_variable>
#include <deque>
#include <functional>
#include <future>
#include <map>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include <torch/torch.h>

#include "placement.h"
#include "thread_group.h"

namespace dtb {

class KernelStream {
public:
    KernelStream(int64_t globalDeviceId, int cudaDevice);
    ~KernelStream();
    KernelStream(const KernelStream&) = delete;
    KernelStream& operator=(const KernelStream&) = delete;

    // Enqueue a task; it runs on this stream's thread with the device and stream current.
    std::future<void> Launch(std::function<void()> task);
    c10::cuda::CUDAStream Stream() const { return mStream; }
    int CudaDevice() const { return mCudaDevice; }

private:
    void Main();

    int64_t mGlobalDeviceId;
    int mCudaDevice;
    c10::cuda::CUDAStream mStream;
    std::mutex mMutex;
    std::condition_variable mCv;
    std::deque<std::packaged_task<void()>> mQueue;
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
std::map<int64_t, torch::Tensor> Redistribute(const std::map<int64_t, torch::Tensor>& locals, const DeviceMesh& mesh,
                                              PlacementSeq src, PlacementSeq dst, const std::vector<int64_t>& globalShape);

// Redistribute several DTensors of one shape and placement the same way. A change of one mesh dim from
// Shard(i) to Shard(j) runs as one fused all-to-all launch per device for all of them (the q/k/v swap of
// Ulysses context parallelism); anything else runs Redistribute per tensor.
std::vector<std::map<int64_t, torch::Tensor>> RedistributeMulti(const std::vector<std::map<int64_t, torch::Tensor>>& locals,
                                                                const DeviceMesh& mesh, PlacementSeq src, PlacementSeq dst,
                                                                const std::vector<int64_t>& globalShape);

}  // namespace dtb
