// Host side of the C ABI declared in include/dtorch_b200.h: communicators, peer mapping, per-call pointer
// rendezvous, kernel selection and launch.
//
// Reference interfaces replaced (tingkuanpei/dtorch):
//   ThreadGroup ctor / backend choice        dtorch/core/communication/thread_group/thread_group.cc:61-90
//   ThreadGroup::AllReduce                   thread_group.cc:127-141
//   ThreadGroup::EqualShapeAllGatherIntoTensor / AllGather / AllGatherIntoVec   thread_group.cc:151-190
//   ThreadGroup::ReduceScatterTensor         thread_group.cc:192-209
//   ThreadGroup::AllToAll                    thread_group.cc:211-241
//   ThreadGroup::Barrier                     thread_group.cc:118-125
//   ThreadGroupSameDeviceBackend             thread_group_same_device_backend.cc:71-360

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <memory>
#include <vector>

#include <dlfcn.h>

#include <cuda.h>
#include <cudaTypedefs.h>
#include <nccl.h>  // types only: the functions are looked up at run time (nccl_api)

#include "../../include/dtorch_b200.h"
#include "dt_kernels.cuh"

using namespace dtb;

namespace {

thread_local std::string g_err;
std::atomic<uint64_t> g_launches{0};

int fail(int status, const std::string& msg) {
    g_err = msg;
    return status;
}

#define DT_CUDA(call)                                                                          \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess) {                                                               \
            return fail(DT_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));      \
        }                                                                                      \
    } while (0)

// [kMaxBlocks][kMaxRanks] barrier flags, then kMaxBlocks per-block epoch counters
constexpr size_t kFlagBytes = static_cast<size_t>(kMaxBlocks) * (kMaxRanks + 1) * sizeof(uint32_t);
constexpr size_t kHeapOffset = 64 * 1024;  // heap starts 64 KiB into the slab (flags first)
constexpr uint32_t kHandleMagic = 0x44544232u;  // "DTB2"

// Restores the calling thread's current device on scope exit: the CUDA runtime shares the thread's current
// context with every other runtime in the process (torch included), so entry points must not leak a switch.
struct DeviceGuard {
    int prev = -1;
    DeviceGuard() {
        if (cudaGetDevice(&prev) != cudaSuccess) {
            prev = -1;
            cudaGetLastError();
        }
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

int elem_bytes(int dtype) {
    switch (dtype) {
        case DT_FLOAT32: return 4;
        case DT_BFLOAT16: return 2;
        case DT_FLOAT16: return 2;
        default: return 0;
    }
}

struct IpcHandle {
    uint32_t magic;
    int32_t rank;
    int32_t nranks;
    int32_t pad;
    uint64_t heap_bytes;
    cudaIpcMemHandle_t mem;
};

// Per-rank state. In a single-process communicator every rank's entry is filled; in a multi-process one only
// the local rank's entry owns memory and peer pointers come from IPC mappings.
struct RankState {
    int dev = -1;
    int num_sms = 148;
    char* slab = nullptr;         // cudaMalloc'd: [flags | pad | heap]
    uint32_t* flags = nullptr;    // this rank's flag array (on dev)
    char* heap = nullptr;
    int* err = nullptr;           // host-mapped error word
    uint64_t rv_gen = 0;          // rendezvous generations passed by this rank
    cudaEvent_t ready = nullptr;  // same-device mode
    uint32_t* peer_flags[kMaxRanks] = {};  // flags of rank r as addressed from this rank's device
    char* peer_heap[kMaxRanks] = {};       // heap of rank r as addressed from this rank's device
    bool imported[kMaxRanks] = {};         // peer slab opened through IPC (must be closed)
    // NVLS buffer: this rank's memory bound to the communicator's multicast object
    char* nvls_uc = nullptr;                     // unicast mapping (this rank's copy)
    char* nvls_mc = nullptr;                     // multicast mapping (every rank's copy at once)
    CUmemGenericAllocationHandle nvls_phys = 0;  // physical memory bound to the multicast object
    bool nvls_bound = false;
};

// What one rank publishes at a rendezvous.
struct Slot {
    const void* in;
    void* out;
    cudaStream_t stream;
    void* extra[kMaxRanks];  // further outputs of a multi-tensor call, copied by value
    // list forms (one buffer per peer): inputs, outputs and byte counts of the publishing rank
    const void* lin[kMaxRanks];
    void* lout[kMaxRanks];
    size_t lbytes[kMaxRanks];  // bytes sent to rank k
    size_t lcap[kMaxRanks];    // room in lout[k] for what rank k sends
};

}  // namespace

struct dt_comm {
    int n = 0;
    bool same_device = false;
    bool multiprocess = false;
    bool ready = false;
    std::atomic<bool> broken{false};
    int local_rank = -1;  // multi-process: the rank this process holds
    size_t heap_bytes = 0;
    int64_t timeout_ms = 600000;
    RankState r[kMaxRanks];
    // in-process rendezvous: double-buffered slots indexed by generation parity
    Slot slots[2][kMaxRanks];
    std::atomic<int> arrived[2];
    std::atomic<uint64_t> gen{0};
    // same-device mode: rank 0 launches, others wait for this generation and chain on `done`
    cudaEvent_t done = nullptr;
    std::atomic<uint64_t> launched_gen{0};
    std::atomic<int> launch_status{0};
    // NVLS (NVLink multicast) buffer
    CUmemGenericAllocationHandle nvls_mc_handle = 0;
    bool nvls_have_mc = false;
    size_t nvls_size = 0;
    CUdeviceptr nvls_mc_va = 0;  // single process: one multicast mapping shared by every rank
    // NCCL clique over the same devices (single-process peer mode), made by the first call routed to NCCL
    std::mutex nccl_mu;
    std::atomic<int> nccl_state{0};  // 0: not tried, 1: ready, -1: unavailable (nccl_err says why)
    std::string nccl_err;
    ncclComm_t nccl[kMaxRanks] = {};
    bool nccl_route = true;   // DTORCH_B200_NCCL != 0: DT_ALGO_AUTO may route to NCCL where it measured faster
    bool rank_order = false;  // DTORCH_B200_RANK_ORDER=1: every call behaves as if DT_RANK_ORDER were set
};

namespace {

int64_t env_timeout_ms() {
    const char* s = std::getenv("DTORCH_COMM_TIMEOUT_SECOND");
    if (s != nullptr && *s != '\0') {
        long long v = std::atoll(s);
        if (v > 0) return static_cast<int64_t>(v) * 1000;
    }
    return 600 * 1000;  // the reference's default (global_option.cc:20)
}

bool env_flag(const char* name, bool dflt) {
    const char* s = std::getenv(name);
    if (s == nullptr || *s == '\0') return dflt;
    return !(s[0] == '0' && s[1] == '\0');
}

// ---- NCCL, for the messages where it measured faster -------------------------------------------------------
// Looked up at run time -- the copy the process already loaded (torch's), else libnccl.so.2 from the library
// path -- so the library has no link-time dependency on it and a process without NCCL never routes there.
struct NcclApi {
    bool ok = false;
    int version = 0;
    ncclResult_t (*init_all)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl_api() {
    static const NcclApi api = [] {
        NcclApi a;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (h == nullptr) return a;
        a.init_all = reinterpret_cast<decltype(a.init_all)>(dlsym(h, "ncclCommInitAll"));
        a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
        a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(h, "ncclCommDestroy"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
        auto get_version = reinterpret_cast<ncclResult_t (*)(int*)>(dlsym(h, "ncclGetVersion"));
        if (get_version != nullptr) get_version(&a.version);
        a.ok = a.init_all && a.all_reduce && a.destroy && a.error_string;
        return a;
    }();
    return api;
}

bool check_rank(const dt_comm* c, int rank) {
    if (c == nullptr || rank < 0 || rank >= c->n) return false;
    if (c->multiprocess && rank != c->local_rank) return false;
    return true;
}

int alloc_rank(dt_comm* c, int rank, int dev, size_t heap_bytes) {
    RankState& s = c->r[rank];
    s.dev = dev;
    DT_CUDA(cudaSetDevice(dev));
    DT_CUDA(cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev));
    const size_t bytes = kHeapOffset + heap_bytes;
    DT_CUDA(cudaMalloc(&s.slab, bytes));
    DT_CUDA(cudaMemset(s.slab, 0, kFlagBytes));
    s.flags = reinterpret_cast<uint32_t*>(s.slab);
    s.heap = s.slab + kHeapOffset;
    DT_CUDA(cudaHostAlloc(&s.err, sizeof(int) * 4, cudaHostAllocMapped | cudaHostAllocPortable));
    *reinterpret_cast<volatile int*>(s.err) = 0;
    DT_CUDA(cudaEventCreateWithFlags(&s.ready, cudaEventDisableTiming));
    DT_CUDA(cudaDeviceSynchronize());
    return DT_OK;
}

// Largest grid whose blocks are all resident at once (every block of a barrier kernel waits for the block
// with the same index on every peer, so all of them must be running).
template <typename K>
int resident_grid(K kernel, int dev, int num_sms) {
    static std::mutex m;
    static std::unordered_map<uint64_t, int> cache;
    const uint64_t key = (reinterpret_cast<uint64_t>(reinterpret_cast<const void*>(kernel)) << 4) ^ static_cast<uint64_t>(dev);
    {
        std::lock_guard<std::mutex> g(m);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0) != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        per_sm = 1;
    }
    const int g = std::min(per_sm * num_sms, kMaxBlocks);
    std::lock_guard<std::mutex> lk(m);
    cache[key] = g;
    return g;
}

SignalCtx make_sig(dt_comm* c, int rank) {
    SignalCtx s{};
    for (int i = 0; i < kMaxRanks; ++i) s.flags[i] = c->r[rank].peer_flags[i];
    s.epochs = c->r[rank].flags + kMaxBlocks * kMaxRanks;
    s.err = c->r[rank].err;
    s.rank = rank;
    s.n = c->n;
    s.timeout_ns = static_cast<uint64_t>(c->timeout_ms) * 1000000ull;
    return s;
}

// In-process rendezvous of all ranks of a single-process communicator: every rank publishes its Slot and
// receives everyone's. Spins (yielding) with the communicator timeout; a timeout marks the communicator
// broken because the generation count can no longer agree across ranks.
int rendezvous(dt_comm* c, int rank, const Slot& mine, Slot* all) {
    RankState& s = c->r[rank];
    const uint64_t my_gen = s.rv_gen;
    const int buf = static_cast<int>(my_gen & 1);
    c->slots[buf][rank] = mine;
    if (c->arrived[buf].fetch_add(1, std::memory_order_acq_rel) + 1 == c->n) {
        c->arrived[buf].store(0, std::memory_order_relaxed);
        c->gen.store(my_gen + 1, std::memory_order_release);
    } else {
        const auto t0 = std::chrono::steady_clock::now();
        uint32_t spins = 0;
        while (c->gen.load(std::memory_order_acquire) <= my_gen) {
            if (++spins > 256) {
                std::this_thread::yield();
                if ((spins & 1023) == 0) {
                    const auto dt = std::chrono::steady_clock::now() - t0;
                    if (std::chrono::duration_cast<std::chrono::milliseconds>(dt).count() > c->timeout_ms) {
                        c->broken = true;
                        return fail(DT_ERR_TIMEOUT, "rendezvous: a rank did not arrive within the timeout");
                    }
                }
            }
        }
    }
    for (int i = 0; i < c->n; ++i) all[i] = c->slots[buf][i];
    s.rv_gen = my_gen + 1;
    return DT_OK;
}

bool in_heap(const dt_comm* c, int rank, const void* p, size_t bytes) {
    const RankState& s = c->r[rank];
    if (s.heap == nullptr || c->heap_bytes == 0) return false;
    const char* q = static_cast<const char*>(p);
    return q >= s.heap && q + bytes <= s.heap + c->heap_bytes;
}

// Every rank's copy of a buffer that sits at the same offset of symmetric memory on every rank, as addressed
// from `rank`'s device: the symmetric heap (both modes), or the NVLS buffer's unicast mappings (single process,
// where every rank's mapping is open to every device). False if `p` is in neither.
bool symmetric_peers(const dt_comm* c, int rank, const void* p, size_t bytes, const char** peers) {
    const RankState& s = c->r[rank];
    const char* q = static_cast<const char*>(p);
    if (bytes == 0) {
        for (int r = 0; r < c->n; ++r) peers[r] = q;
        return true;
    }
    if (in_heap(c, rank, p, bytes)) {
        for (int r = 0; r < c->n; ++r) peers[r] = s.peer_heap[r] + (q - s.heap);
        return true;
    }
    if (!c->multiprocess && s.nvls_uc != nullptr && q >= s.nvls_uc && q + bytes <= s.nvls_uc + c->nvls_size) {
        for (int r = 0; r < c->n; ++r) peers[r] = c->r[r].nvls_uc + (q - s.nvls_uc);
        return true;
    }
    return false;
}

// Resolve every rank's in/out pointer as addressed from `rank`'s device: symmetric offsets when both buffers
// live in symmetric memory (heap or NVLS buffer), otherwise (single process only) the per-call rendezvous.
int resolve_peers(dt_comm* c, int rank, const void* in, size_t in_bytes, void* out, size_t out_bytes,
                  const char** ins, char** outs) {
    const char* sym_out[kMaxRanks];
    if (symmetric_peers(c, rank, in, in_bytes, ins) && symmetric_peers(c, rank, out, out_bytes, sym_out)) {
        for (int r = 0; r < c->n; ++r) outs[r] = const_cast<char*>(sym_out[r]);
        return DT_OK;
    }
    if (c->multiprocess) {
        return fail(DT_ERR_INVALID, "multi-process communicator: buffers must live in the symmetric heap");
    }
    Slot all[kMaxRanks];
    int st = rendezvous(c, rank, Slot{in, out, nullptr}, all);
    if (st != DT_OK) return st;
    for (int r = 0; r < c->n; ++r) {
        ins[r] = static_cast<const char*>(all[r].in);
        outs[r] = static_cast<char*>(all[r].out);
    }
    return DT_OK;
}

int launch_check(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(DT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return DT_OK;
}

// ---------------------------------------------------------------------------------------------------------
// Reduction launches
// ---------------------------------------------------------------------------------------------------------
// Grid of a launch. Barrier kernels pair block b of every rank with block b of every peer, so (1) every rank
// must launch the same grid -- callers pass `want_blocks` computed from sizes every rank knows -- and (2) all
// blocks must be resident at once, which the per-SM cap guarantees (checked against the occupancy of the
// variant; variants are chosen from rank-independent parameters).
template <typename K>
int pick_grid(K kernel, int dev, int num_sms, int64_t want_blocks, int per_sm_cap, int* grid) {
    const int occ = resident_grid(kernel, dev, num_sms) / std::max(num_sms, 1);
    const int per_sm = std::min(per_sm_cap, std::max(occ, 1));
    const int64_t cap = std::min<int64_t>(static_cast<int64_t>(per_sm) * num_sms, kMaxBlocks);
    *grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want_blocks, cap)));
    return DT_OK;
}

constexpr int kReduceBlocksPerSM = 2;
constexpr int kMultiSegs = 3 * kMaxRanks * kMaxRanks;  // same-device fused all-to-all: q, k, v at 8 ranks
constexpr int kCopyBlocksPerSM = 2;

// Upper bound on the CTAs of a peer (cross-GPU) launch; DTORCH_B200_P2P_CTAS overrides the default (no cap
// beyond the residency limit). Every rank must use the same value.
int64_t p2p_ctas() {
    static const int64_t v = [] {
        const char* s = std::getenv("DTORCH_B200_P2P_CTAS");
        const long long x = (s != nullptr && *s != '\0') ? std::atoll(s) : 0;
        return x > 0 ? static_cast<int64_t>(std::min<long long>(x, kMaxBlocks)) : static_cast<int64_t>(kMaxBlocks);
    }();
    return v;
}

template <int NR>
constexpr int reduce_unroll() { return NR <= 2 ? 4 : 2; }

int64_t reduce_want_blocks(int64_t vectors, int64_t scalars, int nr) {
    const int64_t u = nr <= 2 ? 4 : 2;
    const int64_t vb = (vectors + kThreads * u - 1) / (kThreads * u);
    const int64_t sb = (scalars + kThreads - 1) / kThreads;
    return std::max<int64_t>(1, std::max(vb, sb));
}

template <int DT, int NR, bool ST, bool BAR>
int launch_reduce_t(const ReduceArgs& a, int dev, int num_sms, cudaStream_t stream, int64_t want_blocks) {
    auto k = k_reduce<DT, NR, ST, BAR>;
    if (want_blocks <= 0) want_blocks = reduce_want_blocks(a.vhi - a.vlo, a.shi - a.slo, NR);
    if (BAR) want_blocks = std::min(want_blocks, p2p_ctas());
    int grid = 1;
    pick_grid(k, dev, num_sms, want_blocks, kReduceBlocksPerSM, &grid);
    k<<<grid, kThreads, 0, stream>>>(a);
    return launch_check("k_reduce");
}

template <int DT, bool ST, bool BAR>
int launch_reduce_nr(const ReduceArgs& a, int dev, int num_sms, cudaStream_t stream, int64_t want) {
    if (a.n <= 2) return launch_reduce_t<DT, 2, ST, BAR>(a, dev, num_sms, stream, want);
    if (a.n <= 4) return launch_reduce_t<DT, 4, ST, BAR>(a, dev, num_sms, stream, want);
    return launch_reduce_t<DT, 8, ST, BAR>(a, dev, num_sms, stream, want);
}

// want_blocks <= 0: size the grid from this launch's own ranges (same-device kernels, no barrier).
template <bool BAR>
int launch_reduce(const ReduceArgs& a, int dtype, bool storage, int dev, int num_sms, cudaStream_t stream,
                  int64_t want_blocks = 0) {
    switch (dtype) {
        case DT_FLOAT32:
            return launch_reduce_nr<0, false, BAR>(a, dev, num_sms, stream, want_blocks);
        case DT_BFLOAT16:
            return storage ? launch_reduce_nr<1, true, BAR>(a, dev, num_sms, stream, want_blocks)
                           : launch_reduce_nr<1, false, BAR>(a, dev, num_sms, stream, want_blocks);
        case DT_FLOAT16:
            return storage ? launch_reduce_nr<2, true, BAR>(a, dev, num_sms, stream, want_blocks)
                           : launch_reduce_nr<2, false, BAR>(a, dev, num_sms, stream, want_blocks);
        default:
            return fail(DT_ERR_INVALID, "unsupported dtype");
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Fill the vector / scalar ranges for reducing elements [lo, hi) of the inputs. Vectors are used when every
// input and output base is 16-byte aligned and the range starts on a vector boundary; the remainder is scalar.
void set_ranges(ReduceArgs& a, int64_t lo, int64_t hi, int per_vec, bool vec_ok) {
    if (!vec_ok || lo % per_vec != 0) {
        a.vlo = a.vhi = 0;
        a.slo = lo;
        a.shi = hi;
        return;
    }
    a.vlo = lo / per_vec;
    a.vhi = hi / per_vec;
    a.slo = a.vhi * per_vec;
    a.shi = hi;
    if (a.vhi < a.vlo) a.vhi = a.vlo;
}

// ---------------------------------------------------------------------------------------------------------
// Copy launches
// ---------------------------------------------------------------------------------------------------------
uint64_t gcd_u64(uint64_t a, uint64_t b) {
    while (b != 0) {
        const uint64_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

void finish_seg(Seg& s, int vw_unused) {
    (void)vw_unused;
    // Merge adjacent row dims that are contiguous on both sides, then fold contiguous rows into the run.
    for (int pass = 0; pass < 2; ++pass) {
        for (int d = 1; d >= 0; --d) {
            if (s.cnt[d] > 1 && s.cnt[d + 1] > 1 && s.ss[d] == s.cnt[d + 1] * s.ss[d + 1] &&
                s.ds[d] == s.cnt[d + 1] * s.ds[d + 1]) {
                s.cnt[d + 1] *= s.cnt[d];
                s.cnt[d] = 1;
                s.ss[d] = s.ds[d] = 0;
            }
        }
        // move a lone row dim to slot 2 (fast path in the kernel)
        if (s.cnt[2] == 1) {
            for (int d = 1; d >= 0; --d) {
                if (s.cnt[d] > 1) {
                    std::swap(s.cnt[d], s.cnt[2]);
                    std::swap(s.ss[d], s.ss[2]);
                    std::swap(s.ds[d], s.ds[2]);
                    break;
                }
            }
        }
    }
    if (s.cnt[0] == 1 && s.cnt[1] == 1 && s.cnt[2] > 1 && s.ss[2] == s.run && s.ds[2] == s.run) {
        s.run *= s.cnt[2];
        s.cnt[2] = 1;
        s.ss[2] = s.ds[2] = 0;
    }
}

uint64_t seg_align(const Seg& s) {
    uint64_t g = reinterpret_cast<uint64_t>(s.src) | reinterpret_cast<uint64_t>(s.dst);
    g = gcd_u64(g == 0 ? 16 : g, static_cast<uint64_t>(s.run));
    for (int d = 0; d < 3; ++d) {
        if (s.cnt[d] > 1) {
            g = gcd_u64(g, static_cast<uint64_t>(s.ss[d]));
            g = gcd_u64(g, static_cast<uint64_t>(s.ds[d]));
        }
    }
    return g;
}

// Items of a segment set counted with 2 KiB items (the 16-byte geometry) -- the rank-independent size
// measure barrier launches use for their grid.
int64_t copy_want_blocks(int64_t max_row_bytes, int64_t rows, int nseg) {
    constexpr int64_t seg = CopyGeom<16>::kSegBytes;
    const int64_t items = rows * ((max_row_bytes + seg - 1) / seg);
    const int64_t warps = kThreads / 32;
    return std::max<int64_t>(1, (items * nseg + warps - 1) / warps);
}

constexpr int64_t kShortRowSlots = 4 * 32;  // accesses per short-row item: 4 per lane (copy_rows_v)

template <int VW>
void set_geom(Seg& s) {
    s.vw = VW;
    s.seg_bytes = CopyGeom<VW>::kSegBytes;
}

// Per segment: merge contiguous row dims, pick the widest access its pointers, strides and run allow, and
// count its pieces. Then one launch for the whole set.
template <int MAXSEG, bool BAR>
int launch_copy(CopyArgs<MAXSEG>& a, int dev, int num_sms, cudaStream_t stream, int64_t want_blocks = 0) {
    a.max_items = 0;
    for (int i = 0; i < a.nseg; ++i) {
        Seg& s = a.seg[i];
        finish_seg(s, 0);
        const uint64_t g = s.run > 0 ? seg_align(s) : 16;
        if (g % 16 == 0) set_geom<16>(s);
        else if (g % 8 == 0) set_geom<8>(s);
        else if (g % 4 == 0) set_geom<4>(s);
        else if (g % 2 == 0) set_geom<2>(s);
        else set_geom<1>(s);
        const int64_t rows = s.cnt[0] * s.cnt[1] * s.cnt[2];
        s.spr = s.run > 0 ? (s.run + s.seg_bytes - 1) / s.seg_bytes : 0;
        s.items = rows * s.spr;
        s.rpi = 0;
        s.vpr = 0;
        // short rows (at most a quarter of the lane slots each): several whole rows per item
        const int64_t vpr = (s.run + s.vw - 1) / s.vw;
        if (s.run > 0 && rows > 1 && vpr * 4 <= kShortRowSlots) {
            s.vpr = static_cast<int32_t>(vpr);
            s.rpi = static_cast<int32_t>(kShortRowSlots / vpr);
            s.spr = 1;
            s.items = (rows + s.rpi - 1) / s.rpi;
        }
        a.max_items = std::max(a.max_items, s.items);
    }
    auto k = k_copy<MAXSEG, BAR>;
    int per_sm = kCopyBlocksPerSM;
    if (BAR && want_blocks > 0) {
        // peer copies, measured at 8 GPUs: one CTA per SM keeps the fabric less congested up to ~256 MiB
        // per rank; two per SM win a few percent above (the size measure is the same on every rank)
        if (want_blocks < 16384) per_sm = 1;
        want_blocks = std::min(want_blocks, p2p_ctas());
    }
    if (want_blocks <= 0) {
        const int64_t warps_per_block = kThreads / 32;
        want_blocks = std::max<int64_t>((a.max_items * a.nseg + warps_per_block - 1) / warps_per_block, 1);
    }
    int grid = 1;
    pick_grid(k, dev, num_sms, want_blocks, per_sm, &grid);
    k<<<grid, kThreads, 0, stream>>>(a);
    return launch_check("k_copy");
}

// Shard sizes: the first L % n ranks get one more (Placement::GetShardSizeForAllRank,
// dtorch/api/cpp/distributed_spec.cc:202-213).
void shard_sizes(int64_t L, int n, int64_t* out) {
    for (int i = 0; i < n; ++i) out[i] = L / n + (i < L % n ? 1 : 0);
}

// All-to-all segment from source rank i (input base `src`) to destination rank k (output base `dst`).
// The tensor is viewed as [d0, X, dmid, Y, d2] with X/Y the src/dst dims in their order in the shape.
struct A2AGeom {
    int64_t d0, dmid, d2;
    int64_t D;      // dst-dim extent (same on every rank of the group)
    int64_t A;      // src-dim extent of the output (sum of src_lens)
    bool src_first; // src_dim < dst_dim
    int64_t es;
};

Seg a2a_seg(const A2AGeom& g, const char* src, char* dst, int64_t L_i, int64_t soff_i, int64_t len_k, int64_t off_k) {
    Seg s{};
    s.src = src;
    s.dst = dst;
    const int64_t es = g.es;
    if (g.src_first) {
        // in: [d0, L_i, dmid, D, d2]  -> rows (p, x, q), run = len_k*d2
        // out: [d0, A, dmid, len_k, d2]
        s.run = len_k * g.d2 * es;
        s.cnt[0] = g.d0;
        s.cnt[1] = L_i;
        s.cnt[2] = g.dmid;
        s.ss[2] = g.D * g.d2 * es;
        s.ss[1] = g.dmid * s.ss[2];
        s.ss[0] = L_i * s.ss[1];
        s.ds[2] = len_k * g.d2 * es;
        s.ds[1] = g.dmid * s.ds[2];
        s.ds[0] = g.A * s.ds[1];
        s.src += off_k * g.d2 * es;
        s.dst += soff_i * s.ds[1];
    } else {
        // in: [d0, D, dmid, L_i, d2]  -> rows (p, y, q), run = L_i*d2
        // out: [d0, len_k, dmid, A, d2]
        s.run = L_i * g.d2 * es;
        s.cnt[0] = g.d0;
        s.cnt[1] = len_k;
        s.cnt[2] = g.dmid;
        s.ss[2] = L_i * g.d2 * es;
        s.ss[1] = g.dmid * s.ss[2];
        s.ss[0] = g.D * s.ss[1];
        s.ds[2] = g.A * g.d2 * es;
        s.ds[1] = g.dmid * s.ds[2];
        s.ds[0] = len_k * s.ds[1];
        s.src += off_k * s.ss[1];
        s.dst += soff_i * g.d2 * es;
    }
    if (s.run == 0 || s.cnt[0] == 0 || s.cnt[1] == 0 || s.cnt[2] == 0) {
        s.run = 0;
        s.cnt[0] = s.cnt[1] = s.cnt[2] = 1;
    }
    return s;
}

int a2a_geom(int n, int ndim, const int64_t* in_shape, int src_dim, int dst_dim, const int64_t* src_lens,
             size_t elem_b, A2AGeom* g) {
    if (ndim < 2 || ndim > 16 || in_shape == nullptr || src_lens == nullptr) return fail(DT_ERR_INVALID, "a2a: bad shape");
    if (src_dim < 0 || src_dim >= ndim || dst_dim < 0 || dst_dim >= ndim || src_dim == dst_dim)
        return fail(DT_ERR_INVALID, "a2a: src_dim/dst_dim out of range or equal");
    if (elem_b == 0) return fail(DT_ERR_INVALID, "a2a: elem_bytes == 0");
    for (int d = 0; d < ndim; ++d)
        if (in_shape[d] < 0) return fail(DT_ERR_INVALID, "a2a: negative extent");
    const int lo = std::min(src_dim, dst_dim), hi = std::max(src_dim, dst_dim);
    g->d0 = 1;
    g->dmid = 1;
    g->d2 = 1;
    for (int d = 0; d < lo; ++d) g->d0 *= in_shape[d];
    for (int d = lo + 1; d < hi; ++d) g->dmid *= in_shape[d];
    for (int d = hi + 1; d < ndim; ++d) g->d2 *= in_shape[d];
    g->D = in_shape[dst_dim];
    g->A = 0;
    for (int r = 0; r < n; ++r) {
        if (src_lens[r] < 0) return fail(DT_ERR_INVALID, "a2a: negative src_lens");
        g->A += src_lens[r];
    }
    g->src_first = src_dim < dst_dim;
    g->es = static_cast<int64_t>(elem_b);
    if (g->D < n) return fail(DT_ERR_INVALID, "a2a: dst dim smaller than the group (reference asserts size >= n)");
    return DT_OK;
}

// Same-device mode: rank 0 launches one kernel for the whole group after every rank's stream reached the
// call (its `ready` event); the others chain their streams on `done`. `body` issues the kernel on rank 0's
// stream given every rank's Slot.
template <typename Body>
int same_device_call(dt_comm* c, int rank, Slot mine, cudaStream_t stream, Body body) {
    RankState& s = c->r[rank];
    DT_CUDA(cudaSetDevice(s.dev));
    DT_CUDA(cudaEventRecord(s.ready, stream));
    const uint64_t my_gen = s.rv_gen;
    Slot all[kMaxRanks];
    mine.stream = stream;
    int st = rendezvous(c, rank, mine, all);
    if (st != DT_OK) return st;
    if (rank == 0) {
        int rc = DT_OK;
        for (int r = 1; r < c->n && rc == DT_OK; ++r)
            if (cudaStreamWaitEvent(stream, c->r[r].ready, 0) != cudaSuccess) rc = fail(DT_ERR_CUDA, "cudaStreamWaitEvent");
        if (rc == DT_OK) rc = body(all, stream);
        if (rc == DT_OK && cudaEventRecord(c->done, stream) != cudaSuccess) rc = fail(DT_ERR_CUDA, "cudaEventRecord");
        c->launch_status.store(rc, std::memory_order_relaxed);
        c->launched_gen.store(my_gen + 1, std::memory_order_release);
        return rc;
    }
    const auto t0 = std::chrono::steady_clock::now();
    uint32_t spins = 0;
    while (c->launched_gen.load(std::memory_order_acquire) <= my_gen) {
        if (++spins > 256) {
            std::this_thread::yield();
            if ((spins & 1023) == 0 &&
                std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() >
                    c->timeout_ms) {
                c->broken = true;
                return fail(DT_ERR_TIMEOUT, "same-device: launch by rank 0 not seen within the timeout");
            }
        }
    }
    const int rc = c->launch_status.load(std::memory_order_relaxed);
    if (rc != DT_OK) return fail(rc, "same-device: rank 0 failed to launch the collective");
    DT_CUDA(cudaStreamWaitEvent(stream, c->done, 0));
    return DT_OK;
}

template <typename Body>
int same_device_call(dt_comm* c, int rank, const void* in, void* out, cudaStream_t stream, Body body) {
    Slot mine{};
    mine.in = in;
    mine.out = out;
    return same_device_call(c, rank, mine, stream, body);
}

// ---------------------------------------------------------------------------------------------------------
// CUDA driver entry points for NVLink multicast (looked up at run time through the runtime, so the library
// has no link-time dependency on libcuda)
// ---------------------------------------------------------------------------------------------------------
struct Driver {
    PFN_cuDeviceGet deviceGet = nullptr;
    PFN_cuDeviceGetAttribute deviceGetAttribute = nullptr;
    PFN_cuMulticastCreate mcCreate = nullptr;
    PFN_cuMulticastAddDevice mcAddDevice = nullptr;
    PFN_cuMulticastBindMem mcBindMem = nullptr;
    PFN_cuMulticastUnbind mcUnbind = nullptr;
    PFN_cuMulticastGetGranularity mcGranularity = nullptr;
    PFN_cuMemCreate memCreate = nullptr;
    PFN_cuMemRelease memRelease = nullptr;
    PFN_cuMemAddressReserve addressReserve = nullptr;
    PFN_cuMemAddressFree addressFree = nullptr;
    PFN_cuMemMap memMap = nullptr;
    PFN_cuMemUnmap memUnmap = nullptr;
    PFN_cuMemSetAccess memSetAccess = nullptr;
    PFN_cuMemGetAllocationGranularity allocGranularity = nullptr;
    PFN_cuMemExportToShareableHandle exportHandle = nullptr;
    PFN_cuMemImportFromShareableHandle importHandle = nullptr;
    bool ok = false;
    std::string missing;
};

const Driver& driver() {
    static Driver d = [] {
        Driver r;
        auto get = [&r](const char* name, void** fn) {
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
                *fn == nullptr) {
                cudaGetLastError();
                if (r.missing.empty()) r.missing = name;
                *fn = nullptr;
            }
        };
        get("cuDeviceGet", reinterpret_cast<void**>(&r.deviceGet));
        get("cuDeviceGetAttribute", reinterpret_cast<void**>(&r.deviceGetAttribute));
        get("cuMulticastCreate", reinterpret_cast<void**>(&r.mcCreate));
        get("cuMulticastAddDevice", reinterpret_cast<void**>(&r.mcAddDevice));
        get("cuMulticastBindMem", reinterpret_cast<void**>(&r.mcBindMem));
        get("cuMulticastUnbind", reinterpret_cast<void**>(&r.mcUnbind));
        get("cuMulticastGetGranularity", reinterpret_cast<void**>(&r.mcGranularity));
        get("cuMemCreate", reinterpret_cast<void**>(&r.memCreate));
        get("cuMemRelease", reinterpret_cast<void**>(&r.memRelease));
        get("cuMemAddressReserve", reinterpret_cast<void**>(&r.addressReserve));
        get("cuMemAddressFree", reinterpret_cast<void**>(&r.addressFree));
        get("cuMemMap", reinterpret_cast<void**>(&r.memMap));
        get("cuMemUnmap", reinterpret_cast<void**>(&r.memUnmap));
        get("cuMemSetAccess", reinterpret_cast<void**>(&r.memSetAccess));
        get("cuMemGetAllocationGranularity", reinterpret_cast<void**>(&r.allocGranularity));
        get("cuMemExportToShareableHandle", reinterpret_cast<void**>(&r.exportHandle));
        get("cuMemImportFromShareableHandle", reinterpret_cast<void**>(&r.importHandle));
        r.ok = r.missing.empty();
        return r;
    }();
    return d;
}

#define DT_CU(call)                                                                                     \
    do {                                                                                                \
        CUresult r_ = (call);                                                                           \
        if (r_ != CUDA_SUCCESS) return fail(DT_ERR_CUDA, std::string(#call) + ": CUresult " + std::to_string(r_)); \
    } while (0)

int nvls_device_supported(int dev, bool* yes) {
    const Driver& D = driver();
    if (!D.ok) return fail(DT_ERR_UNSUPPORTED, "CUDA driver entry point missing: " + D.missing);
    CUdevice cu = 0;
    DT_CU(D.deviceGet(&cu, dev));
    int v = 0;
    DT_CU(D.deviceGetAttribute(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, cu));
    *yes = v != 0;
    return DT_OK;
}

// Multicast and allocation granularity of `dev` for `n` devices; the buffer size is a multiple of both.
int nvls_granularity(int dev, int n, size_t* gran) {
    const Driver& D = driver();
    CUmulticastObjectProp mp{};
    mp.numDevices = static_cast<unsigned int>(n);
    mp.size = 1;
    mp.handleTypes = 0;
    size_t g_mc = 0, g_alloc = 0;
    DT_CU(D.mcGranularity(&g_mc, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED));
    CUmemAllocationProp ap{};
    ap.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    ap.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    ap.location.id = dev;
    DT_CU(D.allocGranularity(&g_alloc, &ap, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED));
    *gran = std::max(g_mc, g_alloc);
    return DT_OK;
}

// Physical memory of `rank` on its device, bound to the multicast object, mapped at a unicast address that
// the listed devices may access.
int nvls_bind_rank(dt_comm* c, int rank, const int* access_devs, int n_access) {
    const Driver& D = driver();
    RankState& s = c->r[rank];
    CUmemAllocationProp ap{};
    ap.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    ap.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    ap.location.id = s.dev;
    // memory bound to a multicast object requests the object's shareable handle type
    if (c->multiprocess) ap.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    DT_CU(D.memCreate(&s.nvls_phys, c->nvls_size, &ap, 0));
    DT_CU(D.mcBindMem(c->nvls_mc_handle, 0, s.nvls_phys, 0, c->nvls_size, 0));
    s.nvls_bound = true;
    CUdeviceptr va = 0;
    DT_CU(D.addressReserve(&va, c->nvls_size, 0, 0, 0));
    DT_CU(D.memMap(va, c->nvls_size, 0, s.nvls_phys, 0));
    s.nvls_uc = reinterpret_cast<char*>(va);
    std::vector<CUmemAccessDesc> acc(static_cast<size_t>(n_access));
    for (int i = 0; i < n_access; ++i) {
        acc[i].location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        acc[i].location.id = access_devs[i];
        acc[i].flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    }
    DT_CU(D.memSetAccess(va, c->nvls_size, acc.data(), acc.size()));
    return DT_OK;
}

// Multicast mapping accessible from the listed devices.
int nvls_map_multicast(dt_comm* c, const int* access_devs, int n_access, CUdeviceptr* out) {
    const Driver& D = driver();
    CUdeviceptr va = 0;
    DT_CU(D.addressReserve(&va, c->nvls_size, 0, 0, 0));
    DT_CU(D.memMap(va, c->nvls_size, 0, c->nvls_mc_handle, 0));
    std::vector<CUmemAccessDesc> acc(static_cast<size_t>(n_access));
    for (int i = 0; i < n_access; ++i) {
        acc[i].location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        acc[i].location.id = access_devs[i];
        acc[i].flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    }
    DT_CU(D.memSetAccess(va, c->nvls_size, acc.data(), acc.size()));
    *out = va;
    return DT_OK;
}

// Release every NVLS resource of the communicator (after its devices were synchronized).
void nvls_release(dt_comm* c) {
    if (!c->nvls_have_mc) return;
    const Driver& D = driver();
    for (int i = 0; i < kMaxRanks; ++i) {
        RankState& s = c->r[i];
        if (s.dev < 0) continue;
        cudaSetDevice(s.dev);
        if (s.nvls_mc != nullptr && c->nvls_mc_va == 0) {
            D.memUnmap(reinterpret_cast<CUdeviceptr>(s.nvls_mc), c->nvls_size);
            D.addressFree(reinterpret_cast<CUdeviceptr>(s.nvls_mc), c->nvls_size);
        }
        if (s.nvls_uc != nullptr) {
            D.memUnmap(reinterpret_cast<CUdeviceptr>(s.nvls_uc), c->nvls_size);
            D.addressFree(reinterpret_cast<CUdeviceptr>(s.nvls_uc), c->nvls_size);
        }
        if (s.nvls_bound) {
            CUdevice cu = 0;
            if (D.deviceGet(&cu, s.dev) == CUDA_SUCCESS) D.mcUnbind(c->nvls_mc_handle, cu, 0, c->nvls_size);
        }
        if (s.nvls_phys != 0) D.memRelease(s.nvls_phys);
        s.nvls_uc = s.nvls_mc = nullptr;
        s.nvls_phys = 0;
        s.nvls_bound = false;
    }
    if (c->nvls_mc_va != 0) {
        D.memUnmap(c->nvls_mc_va, c->nvls_size);
        D.addressFree(c->nvls_mc_va, c->nvls_size);
        c->nvls_mc_va = 0;
    }
    D.memRelease(c->nvls_mc_handle);
    c->nvls_have_mc = false;
    c->nvls_size = 0;
}

// CTAs issuing multimem traffic per rank. The switch serves a bounded number of in-flight reductions; more
// CTAs than that only queue up (measured: fewer CTAs keep NVLS throughput steady as messages grow).
// DTORCH_B200_NVLS_CTAS overrides the default; every rank must use the same value.
int64_t nvls_ctas() {
    static const int64_t v = [] {
        const char* s = std::getenv("DTORCH_B200_NVLS_CTAS");
        const long long x = (s != nullptr && *s != '\0') ? std::atoll(s) : 0;
        return x > 0 ? static_cast<int64_t>(std::min<long long>(x, kMaxBlocks)) : static_cast<int64_t>(16);
    }();
    return v;
}

template <int DT>
int launch_nvls_t(const NvlsArgs& a, int dev, int num_sms, cudaStream_t stream, int64_t want) {
    want = std::min(want, nvls_ctas());
    auto k = k_allreduce_nvls<DT>;
    int grid = 1;
    pick_grid(k, dev, num_sms, want, kReduceBlocksPerSM, &grid);
    k<<<grid, kThreads, 0, stream>>>(a);
    return launch_check("k_allreduce_nvls");
}

int common_checks(dt_comm* c, int rank) {
    if (c == nullptr) return fail(DT_ERR_INVALID, "null communicator");
    if (!check_rank(c, rank)) return fail(DT_ERR_INVALID, "rank out of range for this communicator");
    if (c->broken) return fail(DT_ERR_STATE, "communicator is broken by an earlier timeout");
    if (!c->ready) return fail(DT_ERR_STATE, "communicator not ready (import peers first)");
    return DT_OK;
}

// Local reduce-scatter in one launch: inputs of n * out_count elements, chunk k of the rank-order sum into
// outs[k].
int local_reduce_scatter(int n, const char* const* ins, char* const* outs, size_t out_count, int dtype, int flags,
                         cudaStream_t stream, int dev, int num_sms) {
    ReduceArgs a{};
    const int pv = 16 / elem_bytes(dtype);
    bool vec_ok = static_cast<int64_t>(out_count) % pv == 0;
    for (int r = 0; r < n; ++r) {
        a.in[r] = ins[r];
        a.out[r] = outs[r];
        vec_ok = vec_ok && aligned16(ins[r]) && aligned16(outs[r]);
    }
    a.n = n;
    a.nout = 0;
    a.out_shift = 0;
    a.chunk = static_cast<int64_t>(out_count);
    set_ranges(a, 0, static_cast<int64_t>(out_count) * n, pv, vec_ok);
    return launch_reduce<false>(a, dtype, (flags & DT_ACCUM_STORAGE) != 0, dev, num_sms, stream);
}

// Local (single-device) reduce with `nout` outputs, elements [0, count).
int local_reduce(int n, const char* const* ins, char* const* outs, int nout, size_t count, int dtype, int flags,
                 cudaStream_t stream, int dev, int num_sms) {
    ReduceArgs a{};
    const int pv = 16 / elem_bytes(dtype);
    bool vec_ok = true;
    for (int r = 0; r < n; ++r) {
        a.in[r] = ins[r];
        vec_ok = vec_ok && aligned16(ins[r]);
    }
    for (int j = 0; j < nout; ++j) {
        a.out[j] = outs[j];
        vec_ok = vec_ok && aligned16(outs[j]);
    }
    a.n = n;
    a.nout = nout;
    a.out_shift = 0;
    set_ranges(a, 0, static_cast<int64_t>(count), pv, vec_ok);
    return launch_reduce<false>(a, dtype, (flags & DT_ACCUM_STORAGE) != 0, dev, num_sms, stream);
}

// Copy streams and events of the host-buffer all-reduce, one set per device; the mutex serialises the
// enqueueing of concurrent calls on one device. Every event is waited on right after it is recorded, and
// cudaStreamWaitEvent captures the record it sees at that moment, so one event per hand-off direction is
// reused for every chunk of every call.
struct Staging {
    std::mutex mu;
    cudaStream_t h2d = nullptr;
    cudaStream_t d2h = nullptr;
    cudaEvent_t start = nullptr;
    cudaEvent_t end_h2d = nullptr;
    cudaEvent_t end_d2h = nullptr;
    cudaEvent_t arrived = nullptr;  // a chunk's inputs are on the device (h2d -> caller's stream)
    cudaEvent_t reduced = nullptr;  // a chunk's sum is ready (caller's stream -> d2h)
};

Staging& staging_of(int dev) {
    static std::mutex m;
    static std::unordered_map<int, std::unique_ptr<Staging>> all;
    std::lock_guard<std::mutex> g(m);
    auto& p = all[dev];
    if (!p) p = std::make_unique<Staging>();
    return *p;
}

int current_device_sms(int* dev, int* sms) {
    DT_CUDA(cudaGetDevice(dev));
    DT_CUDA(cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, *dev));
    return DT_OK;
}

// The communicator's NCCL clique, made once by whichever rank thread gets here first (ncclCommInitAll over the
// communicator's devices, in rank order) while the other rank threads wait; every rank thread then sees the
// same outcome, so all ranks route a call the same way. Single-process peer mode only: a multi-process
// communicator has no host channel of its own for NCCL's unique id. Returns true when the clique is usable.
bool nccl_ready(dt_comm* c) {
    if (c->multiprocess || c->same_device || c->n < 2) return false;
    const int state = c->nccl_state.load(std::memory_order_acquire);
    if (state != 0) return state > 0;
    std::lock_guard<std::mutex> g(c->nccl_mu);
    if (c->nccl_state.load(std::memory_order_relaxed) == 0) {
        const NcclApi& api = nccl_api();
        int st = -1;
        if (!api.ok) {
            c->nccl_err = "libnccl.so.2 could not be loaded";
        } else {
            int devs[kMaxRanks];
            for (int r = 0; r < c->n; ++r) devs[r] = c->r[r].dev;
            DeviceGuard device_guard;
            const ncclResult_t e = api.init_all(c->nccl, c->n, devs);
            if (e == ncclSuccess) {
                st = 1;
            } else {
                c->nccl_err = std::string("ncclCommInitAll: ") + api.error_string(e);
                for (int r = 0; r < c->n; ++r) c->nccl[r] = nullptr;
            }
        }
        c->nccl_state.store(st, std::memory_order_release);
    }
    return c->nccl_state.load(std::memory_order_relaxed) > 0;
}

int nccl_all_reduce(dt_comm* c, int rank, const void* in, void* out, size_t count, int dtype, cudaStream_t stream) {
    if (!nccl_ready(c)) {
        if (c->multiprocess || c->same_device)
            return fail(DT_ERR_UNSUPPORTED, "DT_ALGO_NCCL: only for a single-process communicator in peer mode");
        return fail(DT_ERR_UNSUPPORTED, "DT_ALGO_NCCL: " + c->nccl_err);
    }
    const ncclDataType_t t = dtype == DT_FLOAT32 ? ncclFloat32 : dtype == DT_BFLOAT16 ? ncclBfloat16 : ncclFloat16;
    const NcclApi& api = nccl_api();
    const ncclResult_t e = api.all_reduce(in, out, count, t, ncclSum, c->nccl[rank], stream);
    if (e != ncclSuccess) return fail(DT_ERR_CUDA, std::string("ncclAllReduce: ") + api.error_string(e));
    return DT_OK;
}

}  // namespace

// =============================================================================================================
// C ABI
// =============================================================================================================
extern "C" {

const char* dt_status_string(int status) {
    switch (status) {
        case DT_OK: return "ok";
        case DT_ERR_INVALID: return "invalid argument";
        case DT_ERR_CUDA: return "CUDA error";
        case DT_ERR_TIMEOUT: return "timeout waiting for a peer";
        case DT_ERR_PEER: return "peer access unavailable";
        case DT_ERR_UNSUPPORTED: return "unsupported";
        case DT_ERR_STATE: return "communicator not usable";
        default: return "unknown status";
    }
}

const char* dt_last_error_message(void) { return g_err.c_str(); }

int dt_version(void) { return (1 << 16) | 1; }

uint64_t dt_kernel_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int dt_comm_create(int nranks, const int* cuda_devices, size_t heap_bytes, dt_comm** out) {
    DeviceGuard device_guard;
    if (out == nullptr) return fail(DT_ERR_INVALID, "null out");
    *out = nullptr;
    if (nranks < 1 || nranks > kMaxRanks || cuda_devices == nullptr) return fail(DT_ERR_INVALID, "nranks must be 1..8");
    int ndev = 0;
    DT_CUDA(cudaGetDeviceCount(&ndev));
    bool same = true;
    for (int i = 0; i < nranks; ++i) {
        if (cuda_devices[i] < 0 || cuda_devices[i] >= ndev) return fail(DT_ERR_INVALID, "device id out of range");
        if (cuda_devices[i] != cuda_devices[0]) same = false;
        for (int j = 0; j < i; ++j)
            if (!same && cuda_devices[j] == cuda_devices[i])
                return fail(DT_ERR_INVALID, "devices must be all equal (same-device mode) or all distinct");
    }
    if (!same) {
        for (int i = 0; i < nranks; ++i)
            for (int j = 0; j < i; ++j)
                if (cuda_devices[j] == cuda_devices[i])
                    return fail(DT_ERR_INVALID, "devices must be all equal (same-device mode) or all distinct");
    }
    dt_comm* c = new dt_comm();
    c->n = nranks;
    c->same_device = same && nranks > 1;
    c->heap_bytes = heap_bytes;
    c->timeout_ms = env_timeout_ms();
    c->nccl_route = env_flag("DTORCH_B200_NCCL", true);
    c->rank_order = env_flag("DTORCH_B200_RANK_ORDER", false);
    c->arrived[0] = 0;
    c->arrived[1] = 0;
    int st = DT_OK;
    for (int i = 0; i < nranks && st == DT_OK; ++i) st = alloc_rank(c, i, cuda_devices[i], c->same_device ? 0 : heap_bytes);
    if (st == DT_OK && c->same_device) {
        cudaSetDevice(cuda_devices[0]);
        if (cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming) != cudaSuccess) st = fail(DT_ERR_CUDA, "event");
    }
    if (st == DT_OK && !c->same_device) {
        for (int i = 0; i < nranks && st == DT_OK; ++i) {
            cudaSetDevice(cuda_devices[i]);
            for (int j = 0; j < nranks; ++j) {
                if (i == j) continue;
                int can = 0;
                cudaDeviceCanAccessPeer(&can, cuda_devices[i], cuda_devices[j]);
                if (!can) {
                    st = fail(DT_ERR_PEER, "cudaDeviceCanAccessPeer = 0");
                    break;
                }
                cudaError_t e = cudaDeviceEnablePeerAccess(cuda_devices[j], 0);
                if (e == cudaErrorPeerAccessAlreadyEnabled) {
                    cudaGetLastError();
                } else if (e != cudaSuccess) {
                    st = fail(DT_ERR_PEER, std::string("cudaDeviceEnablePeerAccess: ") + cudaGetErrorString(e));
                    break;
                }
            }
        }
        for (int i = 0; i < nranks; ++i)
            for (int j = 0; j < nranks; ++j) {
                c->r[i].peer_flags[j] = c->r[j].flags;
                c->r[i].peer_heap[j] = c->r[j].heap;
            }
    }
    if (st != DT_OK) {
        std::string msg = g_err;
        dt_comm_destroy(c);
        g_err = msg;
        return st;
    }
    c->ready = true;
    *out = c;
    return DT_OK;
}

int dt_comm_create_rank(int nranks, int rank, int cuda_device, size_t heap_bytes, dt_comm** out) {
    DeviceGuard device_guard;
    if (out == nullptr) return fail(DT_ERR_INVALID, "null out");
    *out = nullptr;
    if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks) return fail(DT_ERR_INVALID, "bad rank/nranks");
    dt_comm* c = new dt_comm();
    c->n = nranks;
    c->multiprocess = true;
    c->local_rank = rank;
    c->heap_bytes = heap_bytes;
    c->timeout_ms = env_timeout_ms();
    c->rank_order = env_flag("DTORCH_B200_RANK_ORDER", false);
    int st = alloc_rank(c, rank, cuda_device, heap_bytes);
    if (st != DT_OK) {
        std::string msg = g_err;
        dt_comm_destroy(c);
        g_err = msg;
        return st;
    }
    c->r[rank].peer_flags[rank] = c->r[rank].flags;
    c->r[rank].peer_heap[rank] = c->r[rank].heap;
    c->ready = nranks == 1;
    *out = c;
    return DT_OK;
}

size_t dt_comm_handle_bytes(void) { return sizeof(IpcHandle); }

int dt_comm_export(dt_comm* c, void* handle) {
    DeviceGuard device_guard;
    if (c == nullptr || handle == nullptr || !c->multiprocess) return fail(DT_ERR_INVALID, "export needs a multi-process communicator");
    RankState& s = c->r[c->local_rank];
    IpcHandle h{};
    h.magic = kHandleMagic;
    h.rank = c->local_rank;
    h.nranks = c->n;
    h.heap_bytes = c->heap_bytes;
    DT_CUDA(cudaSetDevice(s.dev));
    DT_CUDA(cudaIpcGetMemHandle(&h.mem, s.slab));
    std::memcpy(handle, &h, sizeof(h));
    return DT_OK;
}

int dt_comm_import(dt_comm* c, const void* handles) {
    DeviceGuard device_guard;
    if (c == nullptr || handles == nullptr || !c->multiprocess) return fail(DT_ERR_INVALID, "import needs a multi-process communicator");
    const int me = c->local_rank;
    RankState& s = c->r[me];
    DT_CUDA(cudaSetDevice(s.dev));
    const IpcHandle* hs = static_cast<const IpcHandle*>(handles);
    for (int r = 0; r < c->n; ++r) {
        if (r == me) continue;
        const IpcHandle& h = hs[r];
        if (h.magic != kHandleMagic || h.rank != r || h.nranks != c->n || h.heap_bytes != c->heap_bytes)
            return fail(DT_ERR_INVALID, "import: handle does not match this communicator");
        if (s.imported[r]) continue;
        void* p = nullptr;
        DT_CUDA(cudaIpcOpenMemHandle(&p, h.mem, cudaIpcMemLazyEnablePeerAccess));
        s.imported[r] = true;
        s.peer_flags[r] = reinterpret_cast<uint32_t*>(p);
        s.peer_heap[r] = static_cast<char*>(p) + kHeapOffset;
    }
    c->ready = true;
    return DT_OK;
}

int dt_comm_destroy(dt_comm* c) {
    DeviceGuard device_guard;
    if (c == nullptr) return DT_OK;
    for (int i = 0; i < kMaxRanks; ++i) {
        if (c->r[i].dev < 0) continue;
        cudaSetDevice(c->r[i].dev);
        cudaDeviceSynchronize();
    }
    if (c->nccl_state.load() > 0) {
        // one thread destroys the whole clique, as it was made (NCCL frees the shared parts with the last one)
        for (int i = 0; i < c->n; ++i)
            if (c->nccl[i] != nullptr) nccl_api().destroy(c->nccl[i]);
    }
    nvls_release(c);
    for (int i = 0; i < kMaxRanks; ++i) {
        RankState& s = c->r[i];
        if (s.dev < 0) continue;
        cudaSetDevice(s.dev);
        for (int j = 0; j < kMaxRanks; ++j)
            if (s.imported[j]) cudaIpcCloseMemHandle(s.peer_flags[j]);
        if (s.ready) cudaEventDestroy(s.ready);
        if (s.slab) cudaFree(s.slab);
        if (s.err) cudaFreeHost(s.err);
    }
    if (c->done) cudaEventDestroy(c->done);
    cudaGetLastError();
    delete c;
    return DT_OK;
}

int dt_comm_size(const dt_comm* c) { return c ? c->n : 0; }

int dt_comm_same_device(const dt_comm* c) { return (c && c->same_device) ? 1 : 0; }

int dt_comm_heap(dt_comm* c, int rank, void** base, size_t* bytes) {
    if (c == nullptr || !check_rank(c, rank) || base == nullptr || bytes == nullptr) return fail(DT_ERR_INVALID, "bad args");
    *base = c->r[rank].heap;
    *bytes = c->same_device ? 0 : c->heap_bytes;
    return DT_OK;
}

int dt_comm_set_timeout_ms(dt_comm* c, int64_t ms) {
    if (c == nullptr || ms <= 0) return fail(DT_ERR_INVALID, "timeout must be > 0");
    c->timeout_ms = ms;
    return DT_OK;
}

int dt_comm_error(dt_comm* c, int rank) {
    if (c == nullptr || !check_rank(c, rank)) return DT_ERR_INVALID;
    return *reinterpret_cast<volatile int*>(c->r[rank].err);
}

int dt_comm_clear_error(dt_comm* c, int rank) {
    if (c == nullptr || !check_rank(c, rank)) return fail(DT_ERR_INVALID, "bad rank");
    *reinterpret_cast<volatile int*>(c->r[rank].err) = 0;
    return DT_OK;
}

// ---- all-reduce / reduce-scatter ---------------------------------------------------------------------------

int dt_all_reduce(dt_comm* c, int rank, const void* in, void* out, size_t count, int dtype, int op, int flags,
                  void* stream_v) {
    int st = common_checks(c, rank);
    DeviceGuard device_guard;
    if (st != DT_OK) return st;
    const int es = elem_bytes(dtype);
    if (es == 0) return fail(DT_ERR_INVALID, "unsupported dtype");
    if (op != DT_SUM) return fail(DT_ERR_UNSUPPORTED, "only SUM is supported (as in the reference)");
    if (count > 0 && (in == nullptr || out == nullptr)) return fail(DT_ERR_INVALID, "null buffer");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
    RankState& s = c->r[rank];
    const bool storage = (flags & DT_ACCUM_STORAGE) != 0;
    const bool rank_order = (flags & DT_RANK_ORDER) != 0 || c->rank_order;
    constexpr int kAlgoBits = DT_ALGO_ONESHOT | DT_ALGO_TWOSHOT | DT_ALGO_NVLS | DT_ALGO_NCCL;
    if ((flags & DT_ALGO_NCCL) != 0) {
        if ((flags & kAlgoBits) != DT_ALGO_NCCL) return fail(DT_ERR_INVALID, "DT_ALGO_NCCL with another DT_ALGO_* flag");
        if (storage || rank_order)
            return fail(DT_ERR_UNSUPPORTED, "DT_ALGO_NCCL sums in NCCL's order and precision; DT_ACCUM_STORAGE and "
                                            "DT_RANK_ORDER are not available with it");
        if (c->same_device || c->multiprocess)
            return fail(DT_ERR_UNSUPPORTED, "DT_ALGO_NCCL: only for a single-process communicator in peer mode");
    }
    if (c->same_device) {
        return same_device_call(c, rank, in, out, stream, [&](const Slot* all, cudaStream_t st0) -> int {
            const char* ins[kMaxRanks];
            char* outs[kMaxRanks];
            int nout = 0;
            for (int r = 0; r < c->n; ++r) {
                ins[r] = static_cast<const char*>(all[r].in);
                bool dup = false;
                for (int j = 0; j < nout; ++j) dup = dup || outs[j] == all[r].out;
                if (!dup) outs[nout++] = static_cast<char*>(all[r].out);
            }
            if (count == 0) return DT_OK;
            return local_reduce(c->n, ins, outs, nout, count, dtype, flags, st0, s.dev, s.num_sms);
        });
    }
    DT_CUDA(cudaSetDevice(s.dev));
    if (c->n == 1) {
        if (count > 0 && in != out) DT_CUDA(cudaMemcpyAsync(out, in, count * es, cudaMemcpyDeviceToDevice, stream));
        return DT_OK;
    }
    if ((flags & DT_ALGO_NCCL) != 0) return nccl_all_reduce(c, rank, in, out, count, dtype, stream);
    // NVLS: input and output inside the communicator's NVLS buffer (same offsets on every rank)
    {
        int64_t nv_in = -1, nv_out = -1;
        const size_t bytes = count * es;
        if (s.nvls_uc != nullptr && s.nvls_mc != nullptr && count > 0) {
            const char* lo = s.nvls_uc;
            const char* pi = static_cast<const char*>(in);
            const char* po = static_cast<const char*>(out);
            if (pi >= lo && pi + bytes <= lo + c->nvls_size && po >= lo && po + bytes <= lo + c->nvls_size) {
                nv_in = pi - lo;
                nv_out = po - lo;
            }
        }
        const bool nvls_ok = nv_in >= 0 && nv_in % 16 == 0 && nv_out % 16 == 0 && bytes % 16 == 0;
        const bool want_nvls = (flags & DT_ALGO_NVLS) != 0;
        if (want_nvls && !nvls_ok)
            return fail(DT_ERR_INVALID, "DT_ALGO_NVLS needs 16-byte aligned input and output inside the communicator's "
                                        "NVLS buffer and a size that is a multiple of 16 bytes");
        if (want_nvls && (storage || rank_order))
            return fail(DT_ERR_UNSUPPORTED, "DT_ALGO_NVLS reduces in the switch's order with fp32 accumulation; "
                                            "DT_ACCUM_STORAGE and DT_RANK_ORDER are not available with it");
        // measured: at 8 ranks NVLS is ahead of the two-shot kernel from 8-16 MiB (781 vs 633 GB/s at 128 MiB);
        // at 4 ranks the two are level within 2 % either way from 16 MiB to 1 GiB (128 MiB: 645 vs 653), so
        // the rank-order fold stays; at 2 ranks NVLS is behind (it moves (1+1/n)S per GPU against 2(n-1)/n S)
        const size_t nvls_min = static_cast<size_t>(8) << 20;
        const bool auto_nvls = (flags & kAlgoBits) == 0 && nvls_ok && !storage && !rank_order && c->n >= 6 &&
                               bytes >= nvls_min;
        if (want_nvls || auto_nvls) {
            NvlsArgs na{};
            na.sig = make_sig(c, rank);
            na.mc_in = s.nvls_mc + nv_in;
            na.mc_out = s.nvls_mc + nv_out;
            const int64_t nvec = static_cast<int64_t>(bytes / 16);
            na.vlo = nvec * rank / c->n;
            na.vhi = nvec * (rank + 1) / c->n;
            const int64_t per_rank = (nvec + c->n - 1) / c->n;
            const int64_t want = std::max<int64_t>(1, (per_rank + kThreads * 4 - 1) / (kThreads * 4));
            switch (dtype) {
                case DT_FLOAT32: return launch_nvls_t<0>(na, s.dev, s.num_sms, stream, want);
                case DT_BFLOAT16: return launch_nvls_t<1>(na, s.dev, s.num_sms, stream, want);
                default: return launch_nvls_t<2>(na, s.dev, s.num_sms, stream, want);
            }
        }
    }
    // NCCL where it measured faster: at 8 GPUs on ordinary buffers from 256 MiB (per-rank bus 657 vs 646 GB/s
    // at 256 MiB, 704 vs 655 at 512 MiB, 726 vs 662 at 1 GiB); at 2 and 4 ranks the rank-order two-shot kernel is
    // ahead at every size from 2 MiB up, and below 256 MiB at 8 ranks too. Every input of the decision is the
    // same on every rank (flags, count, the communicator's shared clique state).
    const size_t nccl_min = static_cast<size_t>(256) << 20;
    if ((flags & kAlgoBits) == 0 && !storage && !rank_order && c->nccl_route && c->n >= 8 &&
        count * es >= nccl_min && nccl_ready(c))
        return nccl_all_reduce(c, rank, in, out, count, dtype, stream);
    ReduceArgs a{};
    const char* ins[kMaxRanks];
    char* outs[kMaxRanks];
    st = resolve_peers(c, rank, in, count * es, out, count * es, ins, outs);
    if (st != DT_OK) return st;
    a.sig = make_sig(c, rank);
    a.n = c->n;
    const int pv = 16 / es;
    bool vec_ok = true;
    for (int r = 0; r < c->n; ++r) {
        a.in[r] = ins[r];
        vec_ok = vec_ok && aligned16(ins[r]) && aligned16(outs[r]);
    }
    int algo = flags & (DT_ALGO_ONESHOT | DT_ALGO_TWOSHOT);
    if (algo == 0) algo = (count * es <= static_cast<size_t>(256) * 1024) ? DT_ALGO_ONESHOT : DT_ALGO_TWOSHOT;
    // one-shot would overwrite an input that peers still read; decided from every rank's pointers so that all
    // ranks pick the same kernel even when only some of them reduce in place
    for (int r = 0; r < c->n; ++r)
        if (ins[r] == outs[r]) algo = DT_ALGO_TWOSHOT;
    if (algo == DT_ALGO_ONESHOT) {
        a.out[0] = outs[rank];
        a.nout = 1;
        set_ranges(a, 0, static_cast<int64_t>(count), pv, vec_ok);
    } else {
        // chunk c of the vectors belongs to rank c; the element tail belongs to the last rank
        const int64_t nvec = vec_ok ? static_cast<int64_t>(count) / pv : 0;
        a.nout = c->n;
        for (int j = 0; j < c->n; ++j) a.out[j] = outs[(rank + 1 + j) % c->n];
        if (vec_ok) {
            a.vlo = nvec * rank / c->n;
            a.vhi = nvec * (rank + 1) / c->n;
            a.slo = a.shi = 0;
            if (rank == c->n - 1) {
                a.slo = nvec * pv;
                a.shi = static_cast<int64_t>(count);
            }
        } else {
            a.vlo = a.vhi = 0;
            a.slo = static_cast<int64_t>(count) * rank / c->n;
            a.shi = static_cast<int64_t>(count) * (rank + 1) / c->n;
        }
    }
    // grid from sizes every rank shares (vec_ok is computed from every rank's pointers)
    int64_t want;
    if (algo == DT_ALGO_ONESHOT) {
        want = vec_ok ? reduce_want_blocks(static_cast<int64_t>(count) / pv, pv, c->n)
                      : reduce_want_blocks(0, static_cast<int64_t>(count), c->n);
    } else {
        const int64_t nvec = static_cast<int64_t>(count) / pv;
        want = vec_ok ? reduce_want_blocks((nvec + c->n - 1) / c->n, pv, c->n)
                      : reduce_want_blocks(0, (static_cast<int64_t>(count) + c->n - 1) / c->n, c->n);
    }
    return launch_reduce<true>(a, dtype, storage, s.dev, s.num_sms, stream, want);
}

int dt_reduce_scatter(dt_comm* c, int rank, const void* in, void* out, size_t out_count, int dtype, int op, int flags,
                      void* stream_v) {
    int st = common_checks(c, rank);
    DeviceGuard device_guard;
    if (st != DT_OK) return st;
    const int es = elem_bytes(dtype);
    if (es == 0) return fail(DT_ERR_INVALID, "unsupported dtype");
    if (op != DT_SUM) return fail(DT_ERR_UNSUPPORTED, "only SUM is supported (as in the reference)");
    if (out_count > 0 && (in == nullptr || out == nullptr)) return fail(DT_ERR_INVALID, "null buffer");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
    RankState& s = c->r[rank];
    const size_t in_count = out_count * static_cast<size_t>(c->n);
    if (c->same_device) {
        return same_device_call(c, rank, in, out, stream, [&](const Slot* all, cudaStream_t st0) -> int {
            if (out_count == 0) return DT_OK;
            const char* ins[kMaxRanks];
            char* outs[kMaxRanks];
            for (int r = 0; r < c->n; ++r) {
                ins[r] = static_cast<const char*>(all[r].in);
                outs[r] = static_cast<char*>(all[r].out);
            }
            return local_reduce_scatter(c->n, ins, outs, out_count, dtype, flags, st0, s.dev, s.num_sms);
        });
    }
    DT_CUDA(cudaSetDevice(s.dev));
    if (c->n == 1) {
        if (out_count > 0 && in != out) DT_CUDA(cudaMemcpyAsync(out, in, out_count * es, cudaMemcpyDeviceToDevice, stream));
        return DT_OK;
    }
    const char* ins[kMaxRanks];
    char* outs[kMaxRanks];
    st = resolve_peers(c, rank, in, in_count * es, out, out_count * es, ins, outs);
    if (st != DT_OK) return st;
    ReduceArgs a{};
    a.sig = make_sig(c, rank);
    a.n = c->n;
    const int pv = 16 / es;
    // vector path decided from every rank's pointers and the shared chunk size, so all ranks agree
    bool vec_ok = static_cast<int64_t>(out_count) % pv == 0;
    for (int r = 0; r < c->n; ++r) {
        a.in[r] = ins[r];
        vec_ok = vec_ok && aligned16(ins[r]) && aligned16(outs[r]);
    }
    a.out[0] = outs[rank];
    a.nout = 1;
    const int64_t lo = static_cast<int64_t>(out_count) * rank;
    a.out_shift = lo;
    set_ranges(a, lo, lo + static_cast<int64_t>(out_count), pv, vec_ok);
    const int64_t want = vec_ok ? reduce_want_blocks(static_cast<int64_t>(out_count) / pv, 0, c->n)
                                : reduce_want_blocks(0, static_cast<int64_t>(out_count), c->n);
    return launch_reduce<true>(a, dtype, (flags & DT_ACCUM_STORAGE) != 0, s.dev, s.num_sms, stream, want);
}

// ---- all-gather -------------------------------------------------------------------------------------------

}  // extern "C"

namespace {

// Placement of rank r's shard in the gathered tensor, as 1 or 2 segments from `src` to `dst` (the output base):
// without sub-split, rows [0, lens[r]) land at the concat offset of rank r; with sub-split (fronts != nullptr)
// the first fronts[r] rows land among the front parts (all ranks' fronts first, in rank order) and the rest
// among the back parts after them -- DistributeGather::GatherShardWithSubSplit,
// dtorch/core/kernel/kernel_implement/distributed_scather_and_gather.cc:147-183.
int gather_segs(int n, int r, const int64_t* lens, const int64_t* fronts, size_t outer, size_t inner_bytes,
                const char* src, char* dst, Seg* out) {
    int64_t total = 0, off = 0, ftotal = 0, foff = 0, boff = 0;
    for (int i = 0; i < n; ++i) {
        total += lens[i];
        if (i < r) off += lens[i];
        if (fronts != nullptr) {
            ftotal += fronts[i];
            if (i < r) {
                foff += fronts[i];
                boff += lens[i] - fronts[i];
            }
        }
    }
    const int64_t inner = static_cast<int64_t>(inner_bytes);
    auto seg = [&](int64_t row0, int64_t rows, int64_t at) {
        Seg g{};
        g.src = src + row0 * inner;
        g.dst = dst + at * inner;
        g.run = rows * inner;
        g.cnt[0] = g.cnt[1] = 1;
        g.cnt[2] = static_cast<int64_t>(outer);
        g.ss[2] = lens[r] * inner;
        g.ds[2] = total * inner;
        if (g.run == 0 || outer == 0) {
            g.run = 0;
            g.cnt[2] = 1;
        }
        return g;
    };
    if (fronts == nullptr) {
        out[0] = seg(0, lens[r], off);
        return 1;
    }
    out[0] = seg(0, fronts[r], foff);
    out[1] = seg(fronts[r], lens[r] - fronts[r], ftotal + boff);
    return 2;
}

int check_gather(int n, const int64_t* lens, const int64_t* fronts) {
    if (lens == nullptr) return fail(DT_ERR_INVALID, "null lens");
    for (int r = 0; r < n; ++r) {
        if (lens[r] < 0) return fail(DT_ERR_INVALID, "negative shard length");
        if (fronts != nullptr && (fronts[r] < 0 || fronts[r] > lens[r]))
            return fail(DT_ERR_INVALID, "sub-split front part outside its shard");
    }
    return DT_OK;
}

// Every rank's shard (all on this device) into one output.
int local_gather(int n, const void* const* ins, void* out, size_t outer, const int64_t* lens, const int64_t* fronts,
                 size_t inner_bytes, cudaStream_t stream, int dev, int sms) {
    CopyArgs<2 * kMaxRanks> a{};
    a.nseg = 0;
    for (int r = 0; r < n; ++r) {
        if (ins[r] == nullptr && lens[r] > 0 && outer > 0 && inner_bytes > 0) return fail(DT_ERR_INVALID, "null input");
        a.nseg += gather_segs(n, r, lens, fronts, outer, inner_bytes, static_cast<const char*>(ins[r]),
                              static_cast<char*>(out), &a.seg[a.nseg]);
    }
    return launch_copy<2 * kMaxRanks, false>(a, dev, sms, stream);
}

int all_gather_impl(dt_comm* c, int rank, const void* in, void* out, size_t outer, const int64_t* lens,
                    const int64_t* fronts, size_t inner_bytes, void* stream_v) {
    DeviceGuard device_guard;
    int st = common_checks(c, rank);
    if (st != DT_OK) return st;
    st = check_gather(c->n, lens, fronts);
    if (st != DT_OK) return st;
    int64_t total = 0;
    for (int r = 0; r < c->n; ++r) total += lens[r];
    const size_t in_bytes = outer * static_cast<size_t>(lens[rank]) * inner_bytes;
    const size_t out_bytes = outer * static_cast<size_t>(total) * inner_bytes;
    if ((in_bytes > 0 && in == nullptr) || (out_bytes > 0 && out == nullptr)) return fail(DT_ERR_INVALID, "null buffer");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
    RankState& s = c->r[rank];
    if (c->same_device) {
        std::vector<int64_t> lv(lens, lens + c->n), fv;
        if (fronts != nullptr) fv.assign(fronts, fronts + c->n);
        return same_device_call(c, rank, in, out, stream, [&](const Slot* all, cudaStream_t st0) -> int {
            const void* ins[kMaxRanks];
            void* outs[kMaxRanks];
            int nout = 0;
            for (int r = 0; r < c->n; ++r) {
                ins[r] = all[r].in;
                bool dup = false;
                for (int j = 0; j < nout; ++j) dup = dup || outs[j] == all[r].out;
                if (!dup) outs[nout++] = all[r].out;
            }
            if (out_bytes == 0) return DT_OK;
            for (int j = 0; j < nout; ++j) {
                const int rc = local_gather(c->n, ins, outs[j], outer, lv.data(), fv.empty() ? nullptr : fv.data(),
                                            inner_bytes, st0, s.dev, s.num_sms);
                if (rc != DT_OK) return rc;
            }
            return DT_OK;
        });
    }
    DT_CUDA(cudaSetDevice(s.dev));
    if (c->n == 1) {
        if (out_bytes > 0 && in != out) DT_CUDA(cudaMemcpyAsync(out, in, out_bytes, cudaMemcpyDeviceToDevice, stream));
        return DT_OK;
    }
    const char* ins[kMaxRanks];
    char* outs[kMaxRanks];
    st = resolve_peers(c, rank, in, in_bytes, out, out_bytes, ins, outs);
    if (st != DT_OK) return st;
    CopyArgs<2 * kMaxRanks> a{};
    a.sig = make_sig(c, rank);
    a.nseg = 0;
    for (int j = 0; j < c->n; ++j) {
        const int k = (rank + 1 + j) % c->n;  // destinations in rotated order, own output last
        a.nseg += gather_segs(c->n, rank, lens, fronts, outer, inner_bytes, static_cast<const char*>(in), outs[k],
                              &a.seg[a.nseg]);
    }
    int64_t max_len = 0;
    for (int r = 0; r < c->n; ++r) max_len = std::max(max_len, lens[r]);
    // the grid depends only on sizes every rank shares
    const int64_t want = copy_want_blocks(max_len * static_cast<int64_t>(inner_bytes), static_cast<int64_t>(outer), c->n);
    return launch_copy<2 * kMaxRanks, true>(a, s.dev, s.num_sms, stream, want);
}

}  // namespace

extern "C" {

int dt_all_gather(dt_comm* c, int rank, const void* in, void* out, size_t outer, const int64_t* lens,
                  size_t inner_bytes, void* stream_v) {
    return all_gather_impl(c, rank, in, out, outer, lens, nullptr, inner_bytes, stream_v);
}

int dt_all_gather_sub_split(dt_comm* c, int rank, const void* in, void* out, size_t outer, const int64_t* lens,
                            const int64_t* fronts, size_t inner_bytes, void* stream_v) {
    if (fronts == nullptr) return fail(DT_ERR_INVALID, "dt_all_gather_sub_split: null fronts");
    return all_gather_impl(c, rank, in, out, outer, lens, fronts, inner_bytes, stream_v);
}

// ---- all-to-all -------------------------------------------------------------------------------------------

int dt_all_to_all(dt_comm* c, int rank, const void* in, void* out, int ndim, const int64_t* in_shape, int src_dim,
                  int dst_dim, const int64_t* src_lens, size_t elem_b, void* stream_v) {
    DeviceGuard device_guard;
    int st = common_checks(c, rank);
    if (st != DT_OK) return st;
    A2AGeom g{};
    st = a2a_geom(c->n, ndim, in_shape, src_dim, dst_dim, src_lens, elem_b, &g);
    if (st != DT_OK) return st;
    if (in_shape[src_dim] != src_lens[rank]) return fail(DT_ERR_INVALID, "a2a: in_shape[src_dim] != src_lens[rank]");
    int64_t split[kMaxRanks], doff[kMaxRanks], soff[kMaxRanks];
    shard_sizes(g.D, c->n, split);
    int64_t acc = 0;
    for (int k = 0; k < c->n; ++k) {
        doff[k] = acc;
        acc += split[k];
    }
    acc = 0;
    for (int r = 0; r < c->n; ++r) {
        soff[r] = acc;
        acc += src_lens[r];
    }
    const int64_t in_elems = g.d0 * g.dmid * g.d2 * g.D * src_lens[rank];
    const int64_t out_elems = g.d0 * g.dmid * g.d2 * g.A * split[rank];
    if ((in_elems > 0 && in == nullptr) || (out_elems > 0 && out == nullptr)) return fail(DT_ERR_INVALID, "null buffer");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
    RankState& s = c->r[rank];
    if (c->same_device) {
        std::vector<int64_t> shape(in_shape, in_shape + ndim);
        std::vector<int64_t> lens(src_lens, src_lens + c->n);
        return same_device_call(c, rank, in, out, stream, [&](const Slot* all, cudaStream_t st0) -> int {
            const void* ins[kMaxRanks];
            void* outs[kMaxRanks];
            for (int r = 0; r < c->n; ++r) {
                ins[r] = all[r].in;
                outs[r] = all[r].out;
            }
            return dt_local_all_to_all(c->n, ins, outs, ndim, shape.data(), src_dim, dst_dim, lens.data(), elem_b, st0);
        });
    }
    DT_CUDA(cudaSetDevice(s.dev));
    if (c->n == 1) {
        if (in_elems > 0 && in != out) DT_CUDA(cudaMemcpyAsync(out, in, in_elems * elem_b, cudaMemcpyDeviceToDevice, stream));
        return DT_OK;
    }
    const char* ins[kMaxRanks];
    char* outs[kMaxRanks];
    st = resolve_peers(c, rank, in, in_elems * elem_b, out, out_elems * elem_b, ins, outs);
    if (st != DT_OK) return st;
    CopyArgs<kMaxRanks> a{};
    a.sig = make_sig(c, rank);
    a.nseg = c->n;
    for (int j = 0; j < c->n; ++j) {
        const int k = (rank + 1 + j) % c->n;
        a.seg[j] = a2a_seg(g, static_cast<const char*>(in), outs[k], src_lens[rank], soff[rank], split[k], doff[k]);
    }
    int64_t max_l = 0;
    for (int r = 0; r < c->n; ++r) max_l = std::max(max_l, src_lens[r]);
    const int64_t max_k = split[0];
    const int64_t run = (g.src_first ? max_k : max_l) * g.d2 * g.es;
    const int64_t rows = g.d0 * g.dmid * (g.src_first ? max_l : max_k);
    const int64_t want = copy_want_blocks(run, rows, c->n);
    return launch_copy<kMaxRanks, true>(a, s.dev, s.num_sms, stream, want);
}

int dt_all_to_all_multi(dt_comm* c, int rank, int ntensors, const void* const* ins_v, void* const* outs_v, int ndim,
                        const int64_t* in_shape, int src_dim, int dst_dim, const int64_t* src_lens, size_t elem_b,
                        void* stream_v) {
    DeviceGuard device_guard;
    int st = common_checks(c, rank);
    if (st != DT_OK) return st;
    if (ntensors < 1 || ntensors > kMaxRanks || ins_v == nullptr || outs_v == nullptr)
        return fail(DT_ERR_INVALID, "dt_all_to_all_multi: ntensors must be 1..8");
    if (ntensors == 1)
        return dt_all_to_all(c, rank, ins_v[0], outs_v[0], ndim, in_shape, src_dim, dst_dim, src_lens, elem_b, stream_v);
    A2AGeom g{};
    st = a2a_geom(c->n, ndim, in_shape, src_dim, dst_dim, src_lens, elem_b, &g);
    if (st != DT_OK) return st;
    if (in_shape[src_dim] != src_lens[rank]) return fail(DT_ERR_INVALID, "a2a: in_shape[src_dim] != src_lens[rank]");
    int64_t split[kMaxRanks], doff[kMaxRanks], soff[kMaxRanks];
    shard_sizes(g.D, c->n, split);
    int64_t acc = 0;
    for (int k = 0; k < c->n; ++k) {
        doff[k] = acc;
        acc += split[k];
    }
    acc = 0;
    for (int r = 0; r < c->n; ++r) {
        soff[r] = acc;
        acc += src_lens[r];
    }
    const int64_t in_elems = g.d0 * g.dmid * g.d2 * g.D * src_lens[rank];
    const int64_t out_elems = g.d0 * g.dmid * g.d2 * g.A * split[rank];
    for (int t = 0; t < ntensors; ++t)
        if ((in_elems > 0 && ins_v[t] == nullptr) || (out_elems > 0 && outs_v[t] == nullptr))
            return fail(DT_ERR_INVALID, "null buffer");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
    RankState& s = c->r[rank];
    if (c->n == 1) {
        for (int t = 0; t < ntensors; ++t) {
            st = dt_all_to_all(c, rank, ins_v[t], outs_v[t], ndim, in_shape, src_dim, dst_dim, src_lens, elem_b, stream_v);
            if (st != DT_OK) return st;
        }
        return DT_OK;
    }
    if (c->same_device) {
        // one launch for every tensor of every rank: ntensors * n * n segments (at most 3 tensors at 8 ranks fit
        // one launch's parameters; more run as one launch per tensor)
        Slot mine{};
        for (int t = 0; t < ntensors; ++t) {
            mine.lin[t] = ins_v[t];
            mine.extra[t] = outs_v[t];
        }
        return same_device_call(c, rank, mine, stream, [&](const Slot* all, cudaStream_t st0) -> int {
            const int per = c->n * c->n;
            for (int t0 = 0; t0 < ntensors;) {
                const int nt = std::min(ntensors - t0, std::max(1, kMultiSegs / per));
                CopyArgs<kMultiSegs> a{};
                a.nseg = 0;
                // interleaved: destination shift j, then tensor, then source rank
                for (int j = 0; j < c->n; ++j)
                    for (int t = t0; t < t0 + nt; ++t)
                        for (int i = 0; i < c->n; ++i) {
                            const int k = (i + j) % c->n;
                            a.seg[a.nseg++] = a2a_seg(g, static_cast<const char*>(all[i].lin[t]),
                                                      static_cast<char*>(all[k].extra[t]), src_lens[i], soff[i],
                                                      split[k], doff[k]);
                        }
                const int rc = launch_copy<kMultiSegs, false>(a, s.dev, s.num_sms, st0);
                if (rc != DT_OK) return rc;
                t0 += nt;
            }
            return DT_OK;
        });
    }
    DT_CUDA(cudaSetDevice(s.dev));
    // every rank's output pointers of every tensor, as addressed from this device
    char* outs[kMaxRanks][kMaxRanks];  // [tensor][rank]
    bool sym = true;
    for (int t = 0; t < ntensors && sym; ++t) {
        const char* peers[kMaxRanks];
        sym = symmetric_peers(c, rank, outs_v[t], static_cast<size_t>(out_elems) * elem_b, peers);
        for (int r = 0; sym && r < c->n; ++r) outs[t][r] = const_cast<char*>(peers[r]);
    }
    if (sym) {
        // every output is in symmetric memory: nothing to exchange
    } else if (c->multiprocess) {
        return fail(DT_ERR_INVALID, "multi-process communicator: buffers must live in the symmetric heap");
    } else {
        Slot mine{};
        mine.in = ins_v[0];
        mine.out = outs_v[0];
        for (int t = 0; t < ntensors; ++t) mine.extra[t] = outs_v[t];
        Slot all[kMaxRanks];
        st = rendezvous(c, rank, mine, all);
        if (st != DT_OK) return st;
        for (int t = 0; t < ntensors; ++t)
            for (int r = 0; r < c->n; ++r) outs[t][r] = static_cast<char*>(all[r].extra[t]);
    }
    CopyArgs<kMaxRanks * kMaxRanks> a{};
    a.sig = make_sig(c, rank);
    a.nseg = ntensors * c->n;
    // segment (j * ntensors + t): tensor t to destination (rank + 1 + j) % n -- destinations interleaved
    for (int j = 0; j < c->n; ++j) {
        const int k = (rank + 1 + j) % c->n;
        for (int t = 0; t < ntensors; ++t)
            a.seg[j * ntensors + t] = a2a_seg(g, static_cast<const char*>(ins_v[t]), outs[t][k], src_lens[rank],
                                              soff[rank], split[k], doff[k]);
    }
    int64_t max_l = 0;
    for (int r = 0; r < c->n; ++r) max_l = std::max(max_l, src_lens[r]);
    const int64_t max_k = split[0];
    const int64_t run = (g.src_first ? max_k : max_l) * g.d2 * g.es;
    const int64_t rows = g.d0 * g.dmid * (g.src_first ? max_l : max_k);
    const int64_t want = copy_want_blocks(run, rows, c->n * ntensors);
    return launch_copy<kMaxRanks * kMaxRanks, true>(a, s.dev, s.num_sms, stream, want);
}

// ---- list forms (c10d's allgather / alltoall with one tensor per rank) ------------------------------------

}  // extern "C"

namespace {

// Launch one segment per (source, destination) pair: rank i's ins[k] -> rank k's outs[i], `bytes[i][k]`.
// Peer mode: this rank's row only, every rank the same grid (sized from every rank's sizes).
int list_copy(dt_comm* c, int rank, const Slot* all, cudaStream_t stream, bool same_device) {
    RankState& s = c->r[rank];
    int64_t max_bytes = 0;
    for (int i = 0; i < c->n; ++i)
        for (int k = 0; k < c->n; ++k) max_bytes = std::max<int64_t>(max_bytes, static_cast<int64_t>(all[i].lbytes[k]));
    if (same_device) {
        CopyArgs<kMaxRanks * kMaxRanks> a{};
        a.nseg = c->n * c->n;
        for (int j = 0; j < c->n; ++j)
            for (int i = 0; i < c->n; ++i) {
                const int k = (i + j) % c->n;
                Seg& g = a.seg[j * c->n + i];
                g = Seg{};
                g.src = static_cast<const char*>(all[i].lin[k]);
                g.dst = static_cast<char*>(all[k].lout[i]);
                g.run = static_cast<int64_t>(all[i].lbytes[k]);
                g.cnt[0] = g.cnt[1] = g.cnt[2] = 1;
            }
        return launch_copy<kMaxRanks * kMaxRanks, false>(a, s.dev, s.num_sms, stream);
    }
    CopyArgs<kMaxRanks> a{};
    a.sig = make_sig(c, rank);
    a.nseg = c->n;
    for (int j = 0; j < c->n; ++j) {
        const int k = (rank + 1 + j) % c->n;  // destinations in rotated order, own copy last
        Seg& g = a.seg[j];
        g = Seg{};
        g.src = static_cast<const char*>(all[rank].lin[k]);
        g.dst = static_cast<char*>(all[k].lout[rank]);
        g.run = static_cast<int64_t>(all[rank].lbytes[k]);
        g.cnt[0] = g.cnt[1] = g.cnt[2] = 1;
    }
    const int64_t want = copy_want_blocks(max_bytes, 1, c->n);
    return launch_copy<kMaxRanks, true>(a, s.dev, s.num_sms, stream, want);
}

// Arguments of every rank, checked together so that every rank reaches the same verdict (a rank that launched
// alone would wait for its peers until the timeout): buffers present, and what rank i sends to rank k fits
// the room rank k gave for it.
int list_check(const dt_comm* c, const Slot* all, const char* what) {
    for (int i = 0; i < c->n; ++i)
        for (int k = 0; k < c->n; ++k) {
            if ((all[i].lbytes[k] > 0 && all[i].lin[k] == nullptr) || (all[k].lcap[i] > 0 && all[k].lout[i] == nullptr))
                return fail(DT_ERR_INVALID, std::string(what) + ": null buffer");
            if (all[i].lbytes[k] > all[k].lcap[i])
                return fail(DT_ERR_INVALID, std::string(what) + ": rank " + std::to_string(i) + " sends " +
                                                std::to_string(all[i].lbytes[k]) + " bytes to rank " +
                                                std::to_string(k) + ", which has room for " +
                                                std::to_string(all[k].lcap[i]));
        }
    return DT_OK;
}

int list_call(dt_comm* c, int rank, const Slot& mine, void* stream_v, const char* what) {
    int st = common_checks(c, rank);
    if (st != DT_OK) return st;
    if (c->multiprocess)
        return fail(DT_ERR_UNSUPPORTED, std::string(what) + ": the list forms exchange buffer lists in process; "
                                        "use a single-process communicator");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
    RankState& s = c->r[rank];
    if (c->same_device) {
        return same_device_call(c, rank, mine, stream, [&](const Slot* all, cudaStream_t st0) -> int {
            const int rc = list_check(c, all, what);
            return rc != DT_OK ? rc : list_copy(c, rank, all, st0, true);
        });
    }
    DT_CUDA(cudaSetDevice(s.dev));
    Slot all[kMaxRanks];
    st = rendezvous(c, rank, mine, all);
    if (st != DT_OK) return st;
    st = list_check(c, all, what);
    if (st != DT_OK) return st;
    if (c->n == 1) {
        if (mine.lbytes[0] > 0 && mine.lin[0] != mine.lout[0])
            DT_CUDA(cudaMemcpyAsync(mine.lout[0], mine.lin[0], mine.lbytes[0], cudaMemcpyDeviceToDevice, stream));
        return DT_OK;
    }
    return list_copy(c, rank, all, stream, false);
}

}  // namespace

extern "C" {

int dt_all_to_all_list(dt_comm* c, int rank, const void* const* ins, const size_t* in_bytes, void* const* outs,
                       const size_t* out_bytes, void* stream) {
    DeviceGuard device_guard;
    if (c == nullptr || ins == nullptr || outs == nullptr || in_bytes == nullptr || out_bytes == nullptr)
        return fail(DT_ERR_INVALID, "dt_all_to_all_list: null argument");
    Slot mine{};
    for (int k = 0; k < c->n && k < kMaxRanks; ++k) {
        mine.lin[k] = ins[k];
        mine.lbytes[k] = in_bytes[k];
        mine.lout[k] = outs[k];
        mine.lcap[k] = out_bytes[k];
    }
    return list_call(c, rank, mine, stream, "dt_all_to_all_list");
}

int dt_all_gather_list(dt_comm* c, int rank, const void* in, size_t in_bytes, void* const* outs,
                       const size_t* out_bytes, void* stream) {
    DeviceGuard device_guard;
    if (c == nullptr || outs == nullptr || out_bytes == nullptr)
        return fail(DT_ERR_INVALID, "dt_all_gather_list: null argument");
    Slot mine{};
    for (int k = 0; k < c->n && k < kMaxRanks; ++k) {
        mine.lin[k] = in;  // the same input goes to every rank
        mine.lbytes[k] = in_bytes;
        mine.lout[k] = outs[k];
        mine.lcap[k] = out_bytes[k];
    }
    return list_call(c, rank, mine, stream, "dt_all_gather_list");
}

int dt_barrier(dt_comm* c, int rank, void* stream_v) {
    DeviceGuard device_guard;
    int st = common_checks(c, rank);
    if (st != DT_OK) return st;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
    RankState& s = c->r[rank];
    if (c->same_device) {
        return same_device_call(c, rank, nullptr, nullptr, stream, [](const Slot*, cudaStream_t) { return DT_OK; });
    }
    if (c->n == 1) return DT_OK;
    DT_CUDA(cudaSetDevice(s.dev));
    k_barrier<<<1, 32, 0, stream>>>(make_sig(c, rank));
    return launch_check("k_barrier");
}

// ---- NVLS buffer ------------------------------------------------------------------------------------------

int dt_comm_nvls_supported(dt_comm* c, int* supported) {
    DeviceGuard device_guard;
    if (c == nullptr || supported == nullptr) return fail(DT_ERR_INVALID, "null argument");
    *supported = 0;
    if (c->same_device || c->n < 2) return DT_OK;
    for (int r = 0; r < c->n; ++r) {
        if (c->multiprocess && r != c->local_rank) continue;
        bool yes = false;
        const int st = nvls_device_supported(c->r[r].dev, &yes);
        if (st != DT_OK) return st == DT_ERR_UNSUPPORTED ? DT_OK : st;
        if (!yes) return DT_OK;
    }
    *supported = 1;
    return DT_OK;
}

int dt_comm_nvls_alloc(dt_comm* c, size_t bytes) {
    DeviceGuard device_guard;
    if (c == nullptr || bytes == 0) return fail(DT_ERR_INVALID, "null communicator or zero size");
    if (c->multiprocess || c->same_device || c->n < 2)
        return fail(DT_ERR_INVALID, "dt_comm_nvls_alloc needs a single-process peer communicator of >= 2 ranks");
    if (c->nvls_have_mc) return fail(DT_ERR_STATE, "the communicator already has an NVLS buffer");
    int supported = 0;
    int st = dt_comm_nvls_supported(c, &supported);
    if (st != DT_OK) return st;
    if (!supported) return fail(DT_ERR_UNSUPPORTED, "NVLink multicast is not supported on these devices");
    const Driver& D = driver();
    size_t gran = 0;
    DT_CUDA(cudaSetDevice(c->r[0].dev));
    st = nvls_granularity(c->r[0].dev, c->n, &gran);
    if (st != DT_OK) return st;
    c->nvls_size = (bytes + gran - 1) / gran * gran;
    CUmulticastObjectProp mp{};
    mp.numDevices = static_cast<unsigned int>(c->n);
    mp.size = c->nvls_size;
    mp.handleTypes = 0;
    DT_CU(D.mcCreate(&c->nvls_mc_handle, &mp));
    c->nvls_have_mc = true;
    int devs[kMaxRanks];
    for (int r = 0; r < c->n; ++r) {
        devs[r] = c->r[r].dev;
        CUdevice cu = 0;
        DT_CU(D.deviceGet(&cu, devs[r]));
        DT_CU(D.mcAddDevice(c->nvls_mc_handle, cu));
    }
    for (int r = 0; r < c->n && st == DT_OK; ++r) {
        DT_CUDA(cudaSetDevice(devs[r]));
        st = nvls_bind_rank(c, r, devs, c->n);
    }
    if (st == DT_OK) st = nvls_map_multicast(c, devs, c->n, &c->nvls_mc_va);
    if (st != DT_OK) {
        const std::string msg = g_err;
        nvls_release(c);
        g_err = msg;
        return st;
    }
    for (int r = 0; r < c->n; ++r) {
        c->r[r].nvls_mc = reinterpret_cast<char*>(c->nvls_mc_va);
        DT_CUDA(cudaSetDevice(devs[r]));
        DT_CUDA(cudaMemset(c->r[r].nvls_uc, 0, c->nvls_size));
        DT_CUDA(cudaDeviceSynchronize());
    }
    return DT_OK;
}

int dt_comm_nvls_create(dt_comm* c, size_t bytes, int* fd) {
    DeviceGuard device_guard;
    if (c == nullptr || fd == nullptr || bytes == 0 || !c->multiprocess)
        return fail(DT_ERR_INVALID, "dt_comm_nvls_create needs a multi-process communicator, a size and an fd pointer");
    if (c->nvls_have_mc) return fail(DT_ERR_STATE, "the communicator already has an NVLS buffer");
    int supported = 0;
    int st = dt_comm_nvls_supported(c, &supported);
    if (st != DT_OK) return st;
    if (!supported) return fail(DT_ERR_UNSUPPORTED, "NVLink multicast is not supported on this device");
    const Driver& D = driver();
    RankState& s = c->r[c->local_rank];
    DT_CUDA(cudaSetDevice(s.dev));
    size_t gran = 0;
    st = nvls_granularity(s.dev, c->n, &gran);
    if (st != DT_OK) return st;
    c->nvls_size = (bytes + gran - 1) / gran * gran;
    CUmulticastObjectProp mp{};
    mp.numDevices = static_cast<unsigned int>(c->n);
    mp.size = c->nvls_size;
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    DT_CU(D.mcCreate(&c->nvls_mc_handle, &mp));
    c->nvls_have_mc = true;
    int h = -1;
    DT_CU(D.exportHandle(&h, c->nvls_mc_handle, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0));
    *fd = h;
    return DT_OK;
}

int dt_comm_nvls_attach(dt_comm* c, int fd, size_t bytes) {
    DeviceGuard device_guard;
    if (c == nullptr || bytes == 0 || !c->multiprocess) return fail(DT_ERR_INVALID, "dt_comm_nvls_attach: bad arguments");
    const Driver& D = driver();
    if (!D.ok) return fail(DT_ERR_UNSUPPORTED, "CUDA driver entry point missing: " + D.missing);
    RankState& s = c->r[c->local_rank];
    DT_CUDA(cudaSetDevice(s.dev));
    size_t gran = 0;
    int st = nvls_granularity(s.dev, c->n, &gran);
    if (st != DT_OK) return st;
    const size_t size = (bytes + gran - 1) / gran * gran;
    if (!c->nvls_have_mc) {
        if (fd < 0) return fail(DT_ERR_INVALID, "dt_comm_nvls_attach: invalid file descriptor");
        DT_CU(D.importHandle(&c->nvls_mc_handle, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                             CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR));
        c->nvls_have_mc = true;
        c->nvls_size = size;
    } else if (c->nvls_size != size) {
        return fail(DT_ERR_INVALID, "dt_comm_nvls_attach: size differs from the creator's");
    }
    CUdevice cu = 0;
    DT_CU(D.deviceGet(&cu, s.dev));
    DT_CU(D.mcAddDevice(c->nvls_mc_handle, cu));
    return DT_OK;
}

int dt_comm_nvls_bind(dt_comm* c) {
    DeviceGuard device_guard;
    if (c == nullptr || !c->multiprocess || !c->nvls_have_mc)
        return fail(DT_ERR_STATE, "dt_comm_nvls_bind: attach the multicast object first");
    RankState& s = c->r[c->local_rank];
    DT_CUDA(cudaSetDevice(s.dev));
    const int dev = s.dev;
    int st = nvls_bind_rank(c, c->local_rank, &dev, 1);
    CUdeviceptr mc = 0;
    if (st == DT_OK) st = nvls_map_multicast(c, &dev, 1, &mc);
    if (st != DT_OK) return st;
    s.nvls_mc = reinterpret_cast<char*>(mc);
    DT_CUDA(cudaMemset(s.nvls_uc, 0, c->nvls_size));
    DT_CUDA(cudaDeviceSynchronize());
    return DT_OK;
}

int dt_comm_nvls_buffer(dt_comm* c, int rank, void** ptr, size_t* bytes) {
    if (c == nullptr || !check_rank(c, rank) || ptr == nullptr || bytes == nullptr) return fail(DT_ERR_INVALID, "bad args");
    *ptr = c->r[rank].nvls_uc;
    *bytes = c->r[rank].nvls_uc != nullptr ? c->nvls_size : 0;
    return DT_OK;
}

// ---- point-to-point move between two GPUs ---------------------------------------------------------------

}  // extern "C"

namespace {

// Peer access from `from` to `to`, enabled once per ordered pair for the whole process.
int ensure_peer_access(int from, int to) {
    static std::mutex mu;
    static std::vector<std::pair<int, int>> done;
    std::lock_guard<std::mutex> lock(mu);
    for (auto& p : done)
        if (p.first == from && p.second == to) return DT_OK;
    int can = 0;
    DT_CUDA(cudaDeviceCanAccessPeer(&can, from, to));
    if (!can) return fail(DT_ERR_PEER, "cudaDeviceCanAccessPeer = 0 for the two devices");
    DT_CUDA(cudaSetDevice(from));
    const cudaError_t e = cudaDeviceEnablePeerAccess(to, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
    } else if (e != cudaSuccess) {
        return fail(DT_ERR_PEER, std::string("cudaDeviceEnablePeerAccess: ") + cudaGetErrorString(e));
    }
    done.emplace_back(from, to);
    return DT_OK;
}

}  // namespace

extern "C" {

int dt_peer_copy(void* dst, int dst_device, const void* src, int src_device, size_t bytes, void* stream) {
    DeviceGuard device_guard;
    if (bytes == 0) return DT_OK;
    if (dst == nullptr || src == nullptr) return fail(DT_ERR_INVALID, "dt_peer_copy: null buffer");
    int ndev = 0;
    DT_CUDA(cudaGetDeviceCount(&ndev));
    if (src_device < 0 || src_device >= ndev || dst_device < 0 || dst_device >= ndev)
        return fail(DT_ERR_INVALID, "dt_peer_copy: device id out of range");
    if (src_device != dst_device) {
        const int st = ensure_peer_access(src_device, dst_device);
        if (st != DT_OK) return st;
    }
    DT_CUDA(cudaSetDevice(src_device));
    int sms = 0;
    DT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, src_device));
    CopyArgs<1> a{};
    a.nseg = 1;
    Seg& g = a.seg[0];
    g.src = static_cast<const char*>(src);
    g.dst = static_cast<char*>(dst);
    g.run = static_cast<int64_t>(bytes);
    g.cnt[0] = g.cnt[1] = g.cnt[2] = 1;
    return launch_copy<1, false>(a, src_device, sms, static_cast<cudaStream_t>(stream));
}

// ---- same-device kernels ----------------------------------------------------------------------------------

int dt_local_all_reduce(int n, const void* const* ins, void* out, size_t count, int dtype, int flags, void* stream) {
    if (n < 1 || n > kMaxRanks || ins == nullptr) return fail(DT_ERR_INVALID, "n must be 1..8");
    if (elem_bytes(dtype) == 0) return fail(DT_ERR_INVALID, "unsupported dtype");
    if (count == 0) return DT_OK;
    if (out == nullptr) return fail(DT_ERR_INVALID, "null out");
    for (int r = 0; r < n; ++r)
        if (ins[r] == nullptr) return fail(DT_ERR_INVALID, "null input");
    int dev = 0, sms = 0;
    int st = current_device_sms(&dev, &sms);
    if (st != DT_OK) return st;
    const char* in_c[kMaxRanks];
    for (int r = 0; r < n; ++r) in_c[r] = static_cast<const char*>(ins[r]);
    char* o = static_cast<char*>(out);
    return local_reduce(n, in_c, &o, 1, count, dtype, flags, static_cast<cudaStream_t>(stream), dev, sms);
}

int dt_local_all_reduce_host(int n, const void* const* host_ins, void* const* dev_ins, void* dev_out, void* host_out,
                             size_t count, int dtype, int flags, size_t chunk_bytes, void* stream_v) {
    if (n < 1 || n > kMaxRanks || host_ins == nullptr || dev_ins == nullptr) return fail(DT_ERR_INVALID, "n must be 1..8");
    const int es = elem_bytes(dtype);
    if (es == 0) return fail(DT_ERR_INVALID, "unsupported dtype");
    if (count == 0) return DT_OK;
    if (dev_out == nullptr || host_out == nullptr) return fail(DT_ERR_INVALID, "null output");
    for (int r = 0; r < n; ++r)
        if (host_ins[r] == nullptr || dev_ins[r] == nullptr) return fail(DT_ERR_INVALID, "null input");
    int dev = 0, sms = 0;
    int st = current_device_sms(&dev, &sms);
    if (st != DT_OK) return st;
    cudaStream_t user = static_cast<cudaStream_t>(stream_v);
    // 16 MiB per rank measured best for 8 x 128 MiB bf16 partials (4 MiB: per-copy overheads eat the overlap;
    // 64 MiB and up: the last chunk's reduce and D2H no longer hide behind the inputs)
    if (chunk_bytes == 0) chunk_bytes = static_cast<size_t>(16) << 20;
    size_t chunk = std::max<size_t>(16, chunk_bytes / 16 * 16) / static_cast<size_t>(es);
    const size_t nchunks = (count + chunk - 1) / chunk;
    Staging& sg = staging_of(dev);
    std::lock_guard<std::mutex> lock(sg.mu);
    if (sg.h2d == nullptr) {
        DT_CUDA(cudaStreamCreateWithFlags(&sg.h2d, cudaStreamNonBlocking));
        DT_CUDA(cudaStreamCreateWithFlags(&sg.d2h, cudaStreamNonBlocking));
        for (cudaEvent_t* e : {&sg.start, &sg.end_h2d, &sg.end_d2h, &sg.arrived, &sg.reduced})
            DT_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    }
    // the staging buffers are free once the work already on `stream` (earlier calls included) has finished
    DT_CUDA(cudaEventRecord(sg.start, user));
    DT_CUDA(cudaStreamWaitEvent(sg.h2d, sg.start, 0));
    DT_CUDA(cudaStreamWaitEvent(sg.d2h, sg.start, 0));
    int rc = DT_OK;
    auto cuda_ok = [&rc](cudaError_t e, const char* what) {
        if (e != cudaSuccess && rc == DT_OK) rc = fail(DT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
        return rc == DT_OK;
    };
    for (size_t c = 0; c < nchunks && rc == DT_OK; ++c) {
        const size_t off = c * chunk * es;
        const size_t len = std::min(chunk, count - c * chunk);
        const char* ins_c[kMaxRanks];
        for (int r = 0; r < n && rc == DT_OK; ++r) {
            cuda_ok(cudaMemcpyAsync(static_cast<char*>(dev_ins[r]) + off, static_cast<const char*>(host_ins[r]) + off,
                                    len * es, cudaMemcpyHostToDevice, sg.h2d),
                    "cudaMemcpyAsync H2D");
            ins_c[r] = static_cast<const char*>(dev_ins[r]) + off;
        }
        if (!cuda_ok(cudaEventRecord(sg.arrived, sg.h2d), "cudaEventRecord")) break;
        if (!cuda_ok(cudaStreamWaitEvent(user, sg.arrived, 0), "cudaStreamWaitEvent")) break;
        char* o = static_cast<char*>(dev_out) + off;
        rc = local_reduce(n, ins_c, &o, 1, len, dtype, flags, user, dev, sms);
        if (rc != DT_OK) break;
        if (!cuda_ok(cudaEventRecord(sg.reduced, user), "cudaEventRecord")) break;
        if (!cuda_ok(cudaStreamWaitEvent(sg.d2h, sg.reduced, 0), "cudaStreamWaitEvent")) break;
        cuda_ok(cudaMemcpyAsync(static_cast<char*>(host_out) + off, o, len * es, cudaMemcpyDeviceToHost, sg.d2h),
                "cudaMemcpyAsync D2H");
    }
    // whether or not every chunk was enqueued, `stream` ends after every copy this call put in flight, so a
    // caller that synchronizes `stream` after an error may free or reuse the buffers
    const std::string msg = g_err;
    const bool ends_ok = cudaEventRecord(sg.end_h2d, sg.h2d) == cudaSuccess &&
                         cudaEventRecord(sg.end_d2h, sg.d2h) == cudaSuccess &&
                         cudaStreamWaitEvent(user, sg.end_h2d, 0) == cudaSuccess &&
                         cudaStreamWaitEvent(user, sg.end_d2h, 0) == cudaSuccess;
    if (rc != DT_OK) {
        g_err = msg;
        return rc;
    }
    if (!ends_ok) return fail(DT_ERR_CUDA, "dt_local_all_reduce_host: ordering the caller's stream after the copies");
    return DT_OK;
}

int dt_local_reduce_scatter(int n, const void* const* ins, void* const* outs, size_t out_count, int dtype, int flags,
                            void* stream) {
    if (n < 1 || n > kMaxRanks || ins == nullptr || outs == nullptr) return fail(DT_ERR_INVALID, "n must be 1..8");
    const int es = elem_bytes(dtype);
    if (es == 0) return fail(DT_ERR_INVALID, "unsupported dtype");
    if (out_count == 0) return DT_OK;
    for (int r = 0; r < n; ++r)
        if (ins[r] == nullptr || outs[r] == nullptr) return fail(DT_ERR_INVALID, "null buffer");
    int dev = 0, sms = 0;
    int st = current_device_sms(&dev, &sms);
    if (st != DT_OK) return st;
    const char* in_c[kMaxRanks];
    char* out_c[kMaxRanks];
    for (int r = 0; r < n; ++r) {
        in_c[r] = static_cast<const char*>(ins[r]);
        out_c[r] = static_cast<char*>(outs[r]);
    }
    return local_reduce_scatter(n, in_c, out_c, out_count, dtype, flags, static_cast<cudaStream_t>(stream), dev, sms);
}

int dt_local_all_gather(int n, const void* const* ins, void* out, size_t outer, const int64_t* lens, size_t inner_bytes,
                        void* stream) {
    if (n < 1 || n > kMaxRanks || ins == nullptr) return fail(DT_ERR_INVALID, "n must be 1..8");
    int st = check_gather(n, lens, nullptr);
    if (st != DT_OK) return st;
    int64_t total = 0;
    for (int r = 0; r < n; ++r) total += lens[r];
    if (outer * static_cast<size_t>(total) * inner_bytes == 0) return DT_OK;
    if (out == nullptr) return fail(DT_ERR_INVALID, "null out");
    int dev = 0, sms = 0;
    st = current_device_sms(&dev, &sms);
    if (st != DT_OK) return st;
    return local_gather(n, ins, out, outer, lens, nullptr, inner_bytes, static_cast<cudaStream_t>(stream), dev, sms);
}

int dt_local_all_to_all(int n, const void* const* ins, void* const* outs, int ndim, const int64_t* in_shape,
                        int src_dim, int dst_dim, const int64_t* src_lens, size_t elem_b, void* stream) {
    if (n < 1 || n > kMaxRanks || ins == nullptr || outs == nullptr) return fail(DT_ERR_INVALID, "n must be 1..8");
    A2AGeom g{};
    int st = a2a_geom(n, ndim, in_shape, src_dim, dst_dim, src_lens, elem_b, &g);
    if (st != DT_OK) return st;
    int64_t split[kMaxRanks], doff[kMaxRanks], soff[kMaxRanks];
    shard_sizes(g.D, n, split);
    int64_t acc = 0;
    for (int k = 0; k < n; ++k) {
        doff[k] = acc;
        acc += split[k];
    }
    acc = 0;
    for (int r = 0; r < n; ++r) {
        soff[r] = acc;
        acc += src_lens[r];
    }
    for (int r = 0; r < n; ++r)
        if ((src_lens[r] > 0 && ins[r] == nullptr) || outs[r] == nullptr) return fail(DT_ERR_INVALID, "null buffer");
    int dev = 0, sms = 0;
    st = current_device_sms(&dev, &sms);
    if (st != DT_OK) return st;
    CopyArgs<kMaxRanks * kMaxRanks> a{};
    a.nseg = n * n;
    // interleave destinations: segment index j*n + i moves source i -> destination (i + j) % n
    for (int j = 0; j < n; ++j)
        for (int i = 0; i < n; ++i) {
            const int k = (i + j) % n;
            a.seg[j * n + i] = a2a_seg(g, static_cast<const char*>(ins[i]), static_cast<char*>(outs[k]), src_lens[i],
                                       soff[i], split[k], doff[k]);
        }
    return launch_copy<kMaxRanks * kMaxRanks, false>(a, dev, sms, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// =============================================================================================================
// Host-partials all-reduce that allocates nothing on the device
// =============================================================================================================
// Staging memory of dt_local_all_reduce_host_noalloc: a fixed array in the library's own device image. Every
// GPU on which the library's kernels are loaded holds these DT_NOALLOC_SCRATCH_BYTES until the process exits.
// In host code this name is a host-side stand-in, not a device address: only the address that
// cudaGetSymbolAddress returns for the current device may be handed to a kernel or a copy.
static __device__ __align__(256) unsigned char dt_noalloc_scratch[DT_NOALLOC_SCRATCH_BYTES];

namespace {

// Device address of dt_noalloc_scratch on `dev` (which must be current), looked up once per device.
int noalloc_scratch(int dev, char** out) {
    static std::mutex mu;
    static std::unordered_map<int, char*> addr;
    std::lock_guard<std::mutex> lock(mu);
    auto it = addr.find(dev);
    if (it == addr.end()) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, dt_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            return fail(DT_ERR_CUDA, std::string("cudaGetSymbolAddress(dt_noalloc_scratch): ") + cudaGetErrorString(e));
        }
        it = addr.emplace(dev, static_cast<char*>(p)).first;
    }
    *out = it->second;
    return DT_OK;
}

size_t round256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

extern "C" int dt_local_all_reduce_host_noalloc(int n, const void* const* host_ins, void* host_out, size_t count,
                                                int dtype, int flags, void* stream_v) {
    if (n < 1 || n > kMaxRanks || host_ins == nullptr) return fail(DT_ERR_INVALID, "n must be 1..8");
    const int es = elem_bytes(dtype);
    if (es == 0) return fail(DT_ERR_INVALID, "unsupported dtype");
    if (count == 0) return DT_OK;
    if (host_out == nullptr) return fail(DT_ERR_INVALID, "null output");
    for (int r = 0; r < n; ++r)
        if (host_ins[r] == nullptr) return fail(DT_ERR_INVALID, "null input");
    // n input slots and one output slot, each 256-byte aligned; checked before anything touches the device
    const size_t slot = round256(count * static_cast<size_t>(es));
    if (count > (static_cast<size_t>(DT_NOALLOC_SCRATCH_BYTES) / static_cast<size_t>(es)) ||
        slot * static_cast<size_t>(n + 1) > static_cast<size_t>(DT_NOALLOC_SCRATCH_BYTES)) {
        return fail(DT_ERR_INVALID, "dt_local_all_reduce_host_noalloc: " + std::to_string(n) + " partials of " +
                                        std::to_string(count * static_cast<size_t>(es)) + " bytes need " +
                                        std::to_string(n + 1) + " staging slots of " + std::to_string(slot) +
                                        " bytes; the static scratch holds " +
                                        std::to_string(static_cast<size_t>(DT_NOALLOC_SCRATCH_BYTES)) +
                                        " bytes (use dt_local_all_reduce_host with caller-provided buffers)");
    }
    int dev = 0, sms = 0;
    int st = current_device_sms(&dev, &sms);
    if (st != DT_OK) return st;
    char* scratch = nullptr;
    st = noalloc_scratch(dev, &scratch);
    if (st != DT_OK) return st;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
    // Everything on the caller's stream: the inputs' copies, one rank-order reduction, the result's copy.
    // Every scratch byte the reduction reads was written by this call's own copies, so nothing needs clearing.
    const char* ins[kMaxRanks];
    for (int r = 0; r < n; ++r) {
        char* d = scratch + static_cast<size_t>(r) * slot;
        DT_CUDA(cudaMemcpyAsync(d, host_ins[r], count * es, cudaMemcpyHostToDevice, stream));
        ins[r] = d;
    }
    char* out = scratch + static_cast<size_t>(n) * slot;
    st = local_reduce(n, ins, &out, 1, count, dtype, flags, stream, dev, sms);
    if (st != DT_OK) return st;
    DT_CUDA(cudaMemcpyAsync(host_out, out, count * es, cudaMemcpyDeviceToHost, stream));
    return DT_OK;
}
