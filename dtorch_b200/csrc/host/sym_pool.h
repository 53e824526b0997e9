// Peer-mapped symmetric buffer pool of one communicator: DTensor locals and ThreadGroup outputs allocated at the
// same offset in every rank's peer-mapped memory, so a collective on them needs no per-call pointer exchange and,
// when the memory is the communicator's NVLS buffer, an all-reduce on them can reduce inside the NVSwitch.
//
// The reference allocates every collective output with torch::empty on the rank's device
// (dtorch/core/communication/thread_group/thread_group.cc:155-156, :180-182, :198, :228-235); the peers only see
// it through the c10d backend's own exchange. Here the output lives in memory every peer already maps.
//
// Symmetry comes from the c10d contract that every rank of a group issues the same collectives in the same
// order: rank r's k-th allocation is the same block as every other rank's k-th allocation. The first rank to
// reach allocation k picks the block (first fit over the free ranges) for everyone; callers pass a size that is
// the same on every rank (the maximum over ranks, known from the operand's local shapes).
//
// Lifetime: a block returns to the free list once every rank's tensor is gone and the GPU has passed the
// points at which they were freed (events recorded on the freeing thread's current stream and on the rank's
// kernel stream, polled on the host), so memory is never reused while a kernel may still touch it. When no range
// fits, the first rank waits for the oldest released block's events with the pool unlocked (that GPU work may
// depend on kernels other rank threads still have to launch); if nothing is left to wait for, every rank gets
// an ordinary allocation instead. A tensor
// used on any other stream must be synchronized by its user before it is freed (the rule of torch's caching
// allocator without recordStream).
#pragma once

#include <cuda_runtime.h>

#include <condition_variable>
#include <cstdint>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <utility>
#include <vector>

#include <torch/torch.h>

namespace dtb {

class SymmetricPool {
public:
    // bases[r]: rank r's pool memory (as addressed by rank r's own device), `bytes` long on every rank;
    // nvls: the memory is the communicator's NVLS buffer.
    SymmetricPool(std::vector<int> devices, std::vector<char*> bases, size_t bytes, bool nvls);
    ~SymmetricPool();
    SymmetricPool(const SymmetricPool&) = delete;
    SymmetricPool& operator=(const SymmetricPool&) = delete;

    // Rank `rank`'s tensor of the next symmetric block of `bytes_all_ranks` bytes (the same value on every rank),
    // viewed with `shape` and `opts` (shape's bytes <= bytes_all_ranks). Returns an undefined tensor when the
    // pool has no room -- then for every rank, so callers fall back to torch::empty on all ranks alike.
    // `keepalive` is held by the tensor (the owner of the pool's memory must outlive it); `kernel_stream` is
    // the stream the rank's collectives run on.
    torch::Tensor Empty(int rank, at::IntArrayRef shape, const at::TensorOptions& opts, size_t bytes_all_ranks,
                        cudaStream_t kernel_stream, std::shared_ptr<void> keepalive);

    bool Owns(int rank, const void* p) const;
    bool nvls() const { return mNvls; }
    size_t bytes() const { return mBytes; }
    // bytes currently held by live or not-yet-released blocks (for tests)
    size_t InUse();

private:
    struct Block {
        size_t off = 0;
        size_t bytes = 0;
        int taken = 0;   // ranks that received their tensor
        int live = 0;    // ranks whose tensor is still alive
        bool failed = false;     // the pool had no room: every rank gets an undefined tensor
        bool resolving = false;  // the first rank is still finding room for it (others wait on mResolved)
        std::vector<std::pair<int, cudaEvent_t>> freed;  // (rank, event) recorded when a rank's tensor died
    };

    void Release(const std::shared_ptr<Block>& b, int rank, cudaStream_t kernel_stream);
    void Reclaim(bool wait);  // move released blocks whose GPU work has finished back to the free list
    bool Fit(size_t bytes, size_t* off);
    void Insert(size_t off, size_t bytes);
    cudaEvent_t NewEvent(int rank);

    std::vector<int> mDevices;
    std::vector<char*> mBases;
    size_t mBytes;
    bool mNvls;
    std::mutex mMutex;
    std::condition_variable mResolved;
    std::map<size_t, size_t> mFree;                      // offset -> length, coalesced
    std::vector<uint64_t> mSeq;                          // per rank: allocations made so far
    std::map<uint64_t, std::shared_ptr<Block>> mPending;  // allocation index -> block not yet taken by all ranks
    std::deque<std::shared_ptr<Block>> mReleased;        // dead on the host, maybe still in use on the GPU
    std::vector<std::vector<cudaEvent_t>> mEventPool;    // per rank, reusable events
    size_t mInUse = 0;
};

}  // namespace dtb
