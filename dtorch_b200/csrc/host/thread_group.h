// ThreadGroup over the B200 collectives: the reference's communicator API
// (dtorch/core/communication/thread_group/thread_group.h:29-78) with the same method names, argument meaning
// and return-by-value outputs, implemented on the C ABI of include/dtorch_b200.h. A c10d::Backend over the
// same ABI (P2PBackend) fills the backend slot the reference's ThreadGroup constructor chooses
// (thread_group.cc:61-90); ThreadGroupManager caches groups per device list (thread_group_manager.cc:91-130).
#pragma once

#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include <torch/csrc/distributed/c10d/Backend.hpp>
#include <torch/torch.h>

#include "../../../include/dtorch_b200.h"
#include "sym_pool.h"

namespace dtb {

enum class ReduceOpType { kSum = 0 };

// CUDA device ordinal of a global device id. DTORCH_DTENSOR_IN_SAME_DEVICE=1 puts every rank on device 0,
// the reference's single-GPU emulation mode (dtorch/core/distributed/cluster_info.cc:66-67).
int CudaDeviceOf(int64_t globalDeviceId);
bool SameDeviceMode();

// Per-device local shapes of the operand being redistributed (the reference's Operand::GetLocalShape and
// IsLocalShapeEventSplit).
struct LocalShapes {
    std::map<int64_t, std::vector<int64_t>> shapes;
    std::vector<int64_t> Get(int64_t deviceId) const;
    bool IsEvenSplit() const;
};

// Bytes of the symmetric pool each new peer-mode group gets (0 = none): DTORCH_B200_POOL_MB, or the value set
// through SetPoolBytes, which wins for groups created after the call.
size_t PoolBytes();
void SetPoolBytes(size_t bytes);

// One dt_comm shared by the rank threads of a group, and the group's symmetric pool: the communicator's NVLS
// buffer when every device supports NVLink multicast, else its symmetric heap.
class SharedComm {
public:
    SharedComm(const std::vector<int>& cudaDevices, size_t poolBytes);
    ~SharedComm();
    SharedComm(const SharedComm&) = delete;
    SharedComm& operator=(const SharedComm&) = delete;
    dt_comm* get() const { return mComm; }
    int CudaDevice(int rank) const { return mDevices[static_cast<size_t>(rank)]; }
    int Size() const { return static_cast<int>(mDevices.size()); }
    SymmetricPool* Pool() const { return mPool.get(); }

private:
    dt_comm* mComm = nullptr;
    std::vector<int> mDevices;
    std::unique_ptr<SymmetricPool> mPool;
};

// Throws std::runtime_error carrying the status name and detail for a non-zero dt_status.
void Check(int status, const char* where);
int DTypeCode(at::ScalarType t);

// c10d backend whose collectives are the B200 kernels. Outputs are stream-ordered on the caller's current
// stream of the rank's device, so the returned Work is already complete.
class P2PBackend : public c10d::Backend {
public:
    P2PBackend(std::shared_ptr<SharedComm> comm, int rank, int size);
    const std::string getBackendName() const override { return "dtorch_b200"; }
    c10::intrusive_ptr<c10d::Work> allreduce(std::vector<at::Tensor>& tensors,
                                             const c10d::AllreduceOptions& opts = c10d::AllreduceOptions()) override;
    c10::intrusive_ptr<c10d::Work> _allgather_base(at::Tensor& output, at::Tensor& input,
                                                   const c10d::AllgatherOptions& opts = c10d::AllgatherOptions()) override;
    c10::intrusive_ptr<c10d::Work> allgather(std::vector<std::vector<at::Tensor>>& outputs, std::vector<at::Tensor>& inputs,
                                             const c10d::AllgatherOptions& opts = c10d::AllgatherOptions()) override;
    c10::intrusive_ptr<c10d::Work> _reduce_scatter_base(
        at::Tensor& output, at::Tensor& input, const c10d::ReduceScatterOptions& opts = c10d::ReduceScatterOptions()) override;
    c10::intrusive_ptr<c10d::Work> alltoall(std::vector<at::Tensor>& outputs, std::vector<at::Tensor>& inputs,
                                            const c10d::AllToAllOptions& opts = c10d::AllToAllOptions()) override;
    c10::intrusive_ptr<c10d::Work> barrier(const c10d::BarrierOptions& opts = c10d::BarrierOptions()) override;

    dt_comm* comm() const { return mComm->get(); }
    int cudaDevice() const { return mComm->CudaDevice(getRank()); }

private:
    std::shared_ptr<SharedComm> mComm;
};

class ThreadGroup {
public:
    ThreadGroup(std::shared_ptr<SharedComm> comm, const std::vector<int64_t>& allGlobalDeviceId, int rank, int size);
    ThreadGroup(const ThreadGroup&) = delete;
    ThreadGroup& operator=(const ThreadGroup&) = delete;

    int GetRank() const { return mRank; }
    int GetWorldSize() const { return mSize; }
    int64_t GetGlobalDeviceId() const { return mIds[static_cast<size_t>(mRank)]; }
    const std::vector<int64_t>& GetAllGlobalDeviceId() const { return mIds; }
    P2PBackend& Backend() { return *mBackend; }

    // A new tensor on this rank's device for a collective's output: from the group's symmetric pool when it has
    // one (every rank of the group must make the same sequence of these calls, with the same `bytesAllRanks`,
    // the largest of the ranks' sizes), else torch::empty.
    torch::Tensor NewOutput(at::IntArrayRef shape, const at::TensorOptions& opts, size_t bytesAllRanks);
    SymmetricPool* Pool() const { return mComm->Pool(); }

    void Barrier();

    // P -> R
    torch::Tensor AllReduce(const torch::Tensor& input, ReduceOpType op = ReduceOpType::kSum);
    // S0 -> R (even split: one fused buffer; uneven: AllGather along dim 0)
    torch::Tensor AllGatherIntoTensor(const torch::Tensor& input, const LocalShapes& operand);
    torch::Tensor EqualShapeAllGatherIntoTensor(const torch::Tensor& input);
    // S(shardIndex) -> R, uneven shards allowed; the concat along shardIndex happens inside the kernel
    torch::Tensor AllGather(const torch::Tensor& input, const LocalShapes& operand, int64_t shardIndex);
    // Shard(shardIndex, subSplit) -> R: every rank's front piece (of the first subSplit + 1 rows) in rank order,
    // then every rank's back piece, placed by the gather kernel itself
    torch::Tensor AllGatherSubSplit(const torch::Tensor& input, const LocalShapes& operand, int64_t shardIndex,
                                    int64_t subSplit);
    // every rank's tensor (views of one gathered buffer)
    std::vector<torch::Tensor> AllGatherIntoVec(const torch::Tensor& input, const LocalShapes& operand);
    // P -> S0, dim 0 divisible by the group size
    torch::Tensor ReduceScatterTensor(const torch::Tensor& input, ReduceOpType op = ReduceOpType::kSum);
    // S(srcDim) -> S(destDim); the split/contiguous pack and the concat happen inside the kernel
    torch::Tensor AllToAll(const torch::Tensor& input, size_t srcDim, size_t destDim, const LocalShapes& operand);
    // the same S(srcDim) -> S(destDim) for several tensors of one shape, in one launch
    std::vector<torch::Tensor> AllToAllMulti(const std::vector<torch::Tensor>& inputs, size_t srcDim, size_t destDim,
                                             const LocalShapes& operand);
    // R -> S(shardIdx); subSplitCoordinates < 0 means a plain shard
    torch::Tensor ReplicateToShard(const torch::Tensor& input, int64_t shardIdx, int64_t subSplitCoordinates = -1);

private:
    void CheckInput(const torch::Tensor& t) const;
    void* Stream() const;

    std::shared_ptr<SharedComm> mComm;
    std::vector<int64_t> mIds;
    int mRank;
    int mSize;
    c10::intrusive_ptr<P2PBackend> mBackend;
};

// Groups keyed by their ordered device list; one SharedComm per key, one ThreadGroup per rank.
class ThreadGroupManager {
public:
    static ThreadGroupManager& Global();
    ThreadGroup& GetThreadGroup(const std::vector<int64_t>& allDeviceId, int64_t currentDeviceId);
    void Clear();

private:
    struct Entry {
        std::shared_ptr<SharedComm> comm;
        std::vector<std::unique_ptr<ThreadGroup>> ranks;
    };
    std::mutex mMutex;
    std::map<std::vector<int64_t>, std::unique_ptr<Entry>> mGroups;
};

}  // namespace dtb
