// Symmetric buffer pool (see sym_pool.h).
#include "sym_pool.h"

#include <c10/cuda/CUDAStream.h>

#include <stdexcept>
#include <string>

namespace dtb {

namespace {

constexpr size_t kAlign = 256;  // block granularity (multicast and 16-byte vector accesses need far less)

struct CurrentDevice {
    int prev = -1;
    explicit CurrentDevice(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(dev);
    }
    ~CurrentDevice() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

SymmetricPool::SymmetricPool(std::vector<int> devices, std::vector<char*> bases, size_t bytes, bool nvls)
    : mDevices(std::move(devices)), mBases(std::move(bases)), mBytes(bytes / kAlign * kAlign), mNvls(nvls) {
    if (mDevices.size() != mBases.size() || mDevices.empty()) throw std::invalid_argument("SymmetricPool: bad ranks");
    mSeq.assign(mDevices.size(), 0);
    mEventPool.resize(mDevices.size());
    if (mBytes > 0) mFree[0] = mBytes;
}

SymmetricPool::~SymmetricPool() {
    // tensors hold the pool's owner alive, so no block is live here; wait for released ones, drop events
    Reclaim(true);
    for (size_t r = 0; r < mEventPool.size(); ++r) {
        CurrentDevice g(mDevices[r]);
        for (cudaEvent_t e : mEventPool[r]) cudaEventDestroy(e);
    }
}

bool SymmetricPool::Owns(int rank, const void* p) const {
    const char* q = static_cast<const char*>(p);
    const char* b = mBases[static_cast<size_t>(rank)];
    return q >= b && q < b + mBytes;
}

size_t SymmetricPool::InUse() {
    std::lock_guard<std::mutex> lock(mMutex);
    return mInUse;
}

bool SymmetricPool::Fit(size_t bytes, size_t* off) {
    for (auto it = mFree.begin(); it != mFree.end(); ++it) {
        if (it->second < bytes) continue;
        *off = it->first;
        const size_t rest = it->second - bytes;
        const size_t at = it->first + bytes;
        mFree.erase(it);
        if (rest > 0) mFree[at] = rest;
        return true;
    }
    return false;
}

void SymmetricPool::Insert(size_t off, size_t bytes) {
    auto it = mFree.emplace(off, bytes).first;
    auto next = std::next(it);
    if (next != mFree.end() && it->first + it->second == next->first) {
        it->second += next->second;
        mFree.erase(next);
    }
    if (it != mFree.begin()) {
        auto prev = std::prev(it);
        if (prev->first + prev->second == it->first) {
            prev->second += it->second;
            mFree.erase(it);
        }
    }
}

cudaEvent_t SymmetricPool::NewEvent(int rank) {
    auto& pool = mEventPool[static_cast<size_t>(rank)];
    if (!pool.empty()) {
        cudaEvent_t e = pool.back();
        pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    CurrentDevice g(mDevices[static_cast<size_t>(rank)]);
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return e;
}

// Called with mMutex held.
void SymmetricPool::Reclaim(bool wait) {
    while (!mReleased.empty()) {
        auto& b = mReleased.front();
        bool done = true;
        for (auto& re : b->freed) {
            if (re.second == nullptr) continue;
            cudaError_t q = wait ? cudaEventSynchronize(re.second) : cudaEventQuery(re.second);
            if (q == cudaErrorNotReady) {
                done = false;
                break;
            }
            cudaGetLastError();
        }
        if (!done) break;  // released in order: later blocks were freed later
        for (auto& re : b->freed)
            if (re.second != nullptr) mEventPool[static_cast<size_t>(re.first)].push_back(re.second);
        b->freed.clear();
        Insert(b->off, b->bytes);
        mInUse -= b->bytes;
        mReleased.pop_front();
    }
}

void SymmetricPool::Release(const std::shared_ptr<Block>& b, int rank, cudaStream_t kernel_stream) {
    const int dev = mDevices[static_cast<size_t>(rank)];
    std::lock_guard<std::mutex> lock(mMutex);
    // the GPU may still be using the memory on the freeing thread's current stream or on the kernel stream
    cudaStream_t current = c10::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(dev)).stream();
    {
        CurrentDevice g(dev);
        for (cudaStream_t s : {current, kernel_stream}) {
            cudaEvent_t e = NewEvent(rank);
            if (e != nullptr && cudaEventRecord(e, s) == cudaSuccess) {
                b->freed.emplace_back(rank, e);
            } else {
                cudaGetLastError();
                if (e != nullptr) mEventPool[static_cast<size_t>(rank)].push_back(e);
                cudaStreamSynchronize(s);  // no event: make sure the memory is idle the slow way
                cudaGetLastError();
            }
        }
    }
    if (--b->live == 0 && b->taken == static_cast<int>(mDevices.size())) mReleased.push_back(b);
}

torch::Tensor SymmetricPool::Empty(int rank, at::IntArrayRef shape, const at::TensorOptions& opts,
                                   size_t bytes_all_ranks, cudaStream_t kernel_stream, std::shared_ptr<void> keepalive) {
    const size_t n = mDevices.size();
    if (rank < 0 || static_cast<size_t>(rank) >= n) throw std::invalid_argument("SymmetricPool: rank out of range");
    int64_t numel = 1;
    for (auto s : shape) numel *= s;
    const size_t need = static_cast<size_t>(numel) * static_cast<size_t>(c10::elementSize(c10::typeMetaToScalarType(opts.dtype())));
    if (need > bytes_all_ranks) throw std::invalid_argument("SymmetricPool: tensor larger than its block");
    const size_t bytes = std::max<size_t>(kAlign, (bytes_all_ranks + kAlign - 1) / kAlign * kAlign);
    std::shared_ptr<Block> b;
    {
        std::unique_lock<std::mutex> lock(mMutex);
        const uint64_t k = mSeq[static_cast<size_t>(rank)]++;
        auto it = mPending.find(k);
        if (it == mPending.end()) {
            // first rank at allocation k: pick the block for every rank
            b = std::make_shared<Block>();
            b->bytes = bytes;
            b->resolving = true;
            mPending[k] = b;
            Reclaim(false);
            while (!Fit(bytes, &b->off)) {
                if (mReleased.empty()) {
                    b->failed = true;
                    break;
                }
                // wait for the oldest released block's GPU work WITHOUT holding the lock: that work may depend on
                // kernels other rank threads still have to launch, and they may need the lock to get there
                std::vector<std::pair<int, cudaEvent_t>> evs = mReleased.front()->freed;
                lock.unlock();
                for (auto& re : evs)
                    if (re.second != nullptr) cudaEventSynchronize(re.second);
                cudaGetLastError();
                lock.lock();
                Reclaim(false);
            }
            if (!b->failed) mInUse += bytes;
            b->resolving = false;
            mResolved.notify_all();
        } else {
            b = it->second;
            mResolved.wait(lock, [&] { return !b->resolving; });
            if (b->bytes != bytes)
                throw std::logic_error("SymmetricPool: ranks asked for different sizes at allocation " +
                                       std::to_string(k) + " (collectives issued out of order?)");
        }
        ++b->taken;
        if (!b->failed) ++b->live;
        if (b->taken == static_cast<int>(n)) {
            mPending.erase(k);
            if (!b->failed && b->live == 0) mReleased.push_back(b);
        }
    }
    if (b->failed) return torch::Tensor();
    char* p = mBases[static_cast<size_t>(rank)] + b->off;
    auto deleter = [this, b, rank, kernel_stream, keepalive](void*) { Release(b, rank, kernel_stream); };
    return torch::from_blob(p, shape, deleter, opts.device(torch::Device(torch::kCUDA, mDevices[static_cast<size_t>(rank)])));
}

}  // namespace dtb
