/*
 * dtorch_b200 — C ABI of the B200-native thread-group collectives that execute DTensor redistribution.
 *
 * The reference (DTorch) runs every rank of a mesh-dim group as one host thread inside one process and reaches
 * its collectives through `ThreadGroup` (dtorch/core/communication/thread_group/thread_group.h:29-78), which
 * forwards to a c10d::Backend picked in the ThreadGroup constructor (thread_group.cc:61-90): ProcessGroupNCCL for
 * distinct GPUs, ThreadGroupSameDeviceBackend when every rank shares one device. This library is the third
 * branch: distinct local GPUs in one process (or one process per GPU with IPC-mapped peers), moved by
 * hand-written sm_100a kernels that load and store peer HBM directly over NVLink / NVSwitch.
 *
 * Conventions
 *   - Every entry point returns dt_status (0 = success) and never aborts the process.
 *   - Pointers are device pointers on the rank's own GPU unless stated otherwise. `stream` is a cudaStream_t
 *     passed as void* (NULL = legacy default stream of the rank's device).
 *   - Collectives are stream-ordered and asynchronous: they enqueue work on `stream` and return.
 *   - All ranks of a communicator must call the same collectives in the same order (the contract of c10d and
 *     of the reference's ThreadGroup).
 *   - Sizes are in elements unless the name ends in _bytes.
 */
#ifndef DTORCH_B200_H
#define DTORCH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DT_MAX_RANKS 8

typedef enum dt_status {
    DT_OK = 0,
    DT_ERR_INVALID = 1,     /* bad argument: null pointer, rank out of range, size mismatch, unsupported dtype */
    DT_ERR_CUDA = 2,        /* a CUDA runtime call failed (message in dt_last_error_message) */
    DT_ERR_TIMEOUT = 3,     /* a host rendezvous or a device-side wait on a peer exceeded the timeout */
    DT_ERR_PEER = 4,        /* peer access between two devices is unavailable */
    DT_ERR_UNSUPPORTED = 5, /* valid request this build does not implement (e.g. a non-SUM reduction) */
    DT_ERR_STATE = 6        /* communicator not ready (multi-process communicator not yet imported) */
} dt_status;

typedef enum dt_dtype {
    DT_FLOAT32 = 0,
    DT_BFLOAT16 = 1,
    DT_FLOAT16 = 2
} dt_dtype;

typedef enum dt_redop {
    DT_SUM = 0 /* c10d::ReduceOp::SUM; the only op the reference asserts (thread_group.cc:130, :201) */
} dt_redop;

/* Reduction flags (bitwise OR).
 *   DT_ACCUM_FP32     accumulate in fp32 in rank order 0..n-1, round to the storage type once (default).
 *   DT_ACCUM_STORAGE  round to the storage type after every add, which is what the reference's CPU fold
 *                     `result += x_r` does in bf16/fp16 (thread_group_same_device_backend.cc:123-130);
 *                     bit-identical to it. For fp32 both modes are the same left fold.
 *   DT_RANK_ORDER     keep the rank-order fold whatever the size: DT_ALGO_AUTO then never picks NVLS or NCCL,
 *                     and forcing either is rejected (DT_ERR_UNSUPPORTED); the environment variable
 *                     DTORCH_B200_RANK_ORDER=1 sets it for every call.
 *   DT_ALGO_ONESHOT / DT_ALGO_TWOSHOT force the all-reduce algorithm; default picks by message size.
 *   DT_ALGO_NVLS      reduce inside the NVSwitch (NVLink SHARP): needs input and output in the communicator's
 *                     NVLS buffer (dt_comm_nvls_*); fp32 accumulation in the switch's order, not rank order.
 *                     Picked by default for such buffers at >= 6 ranks from 8 MiB (where it measured faster
 *                     than the rank-order kernels; at 4 ranks they are level, so the rank-order fold stays).
 *   DT_ALGO_NCCL      ncclAllReduce on a clique of NCCL communicators over the same devices (the reference's
 *                     own GPU backend, thread_group.cc:75-88), made by the first such call (ncclCommInitAll;
 *                     that call must not be captured in a CUDA graph). NCCL's summation order, and for
 *                     bf16/fp16 its precision (partial sums in the storage type); identical on every rank;
 *                     its waits are NCCL's, not bounded by the communicator's timeout.
 *                     Single-process peer mode only; libnccl.so.2 is looked up at run time (the copy the
 *                     process already loaded first). Picked by default for ordinary buffers at 8 ranks from
 *                     256 MiB, where it measured faster than the two-shot kernel (unless DT_RANK_ORDER,
 *                     DT_ACCUM_STORAGE or DTORCH_B200_NCCL=0). */
#define DT_ACCUM_FP32 0x0
#define DT_ACCUM_STORAGE 0x1
#define DT_RANK_ORDER 0x2
#define DT_ALGO_AUTO 0x00
#define DT_ALGO_ONESHOT 0x10
#define DT_ALGO_TWOSHOT 0x20
#define DT_ALGO_NVLS 0x40
#define DT_ALGO_NCCL 0x80

typedef struct dt_comm dt_comm;

/* ---- library ---------------------------------------------------------------------------------------------- */

/* Human-readable name of a status code. */
const char* dt_status_string(int status);

/* Detail of the last failure on the calling host thread ("" if none). */
const char* dt_last_error_message(void);

/* ABI version, (major << 16) | minor. */
int dt_version(void);

/* ---- communicator ------------------------------------------------------------------------------------------ */

/* Single-process communicator over `nranks` ranks, rank r on CUDA device cuda_devices[r].
 * Replaces the c10d backend construction in ThreadGroup::ThreadGroup (thread_group.cc:61-90) for kGpu with
 * distinct devices; all ranks of the group live in this process, as in DTorch's single-controller runtime.
 * Enables peer access between every ordered pair of distinct devices and allocates, per rank, a signal slab
 * (epoch flags for device-side barriers) plus `heap_bytes` of symmetric heap.
 * If every rank names the same device, the communicator runs in same-device mode: the equivalent of
 * ThreadGroupSameDeviceBackend (thread_group_same_device_backend.cc:71-360) — each collective rendezvouses the
 * rank threads on the host and one kernel does the whole collective on that device. */
int dt_comm_create(int nranks, const int* cuda_devices, size_t heap_bytes, dt_comm** out);

/* Multi-process communicator: this process holds rank `rank` only, on device `cuda_device`.
 * Peers become reachable after dt_comm_export on every rank and dt_comm_import of all handles. */
int dt_comm_create_rank(int nranks, int rank, int cuda_device, size_t heap_bytes, dt_comm** out);

/* Size of the opaque handle dt_comm_export writes. */
size_t dt_comm_handle_bytes(void);

/* Write this rank's IPC handle (signal slab + heap) into `handle` (dt_comm_handle_bytes() bytes). */
int dt_comm_export(dt_comm* comm, void* handle);

/* Map every peer's slab: `handles` holds nranks handles in rank order (this rank's own entry is ignored). */
int dt_comm_import(dt_comm* comm, const void* handles);

/* Release slabs, mappings and events. Waits for the communicator's outstanding work on its devices. */
int dt_comm_destroy(dt_comm* comm);

/* Number of ranks, and whether the communicator is in same-device mode (1) or peer mode (0). */
int dt_comm_size(const dt_comm* comm);
int dt_comm_same_device(const dt_comm* comm);

/* Base and size of rank `rank`'s symmetric heap. Buffers placed at the same offset on every rank are reached
 * by peers without a host rendezvous; in a multi-process communicator every buffer a collective reads or
 * writes on a peer must live in the heap. */
int dt_comm_heap(dt_comm* comm, int rank, void** base, size_t* bytes);

/* Device-side wait limit for peers, in milliseconds. Default: DTORCH_COMM_TIMEOUT_SECOND * 1000 (the
 * reference's knob, global_option.cc:20-27, default 600 s). A wait that runs out records DT_ERR_TIMEOUT, the
 * kernel returns, and dt_comm_error reports it; the GPU context stays usable. */
int dt_comm_set_timeout_ms(dt_comm* comm, int64_t ms);

/* Sticky device-side error of rank `rank` (DT_OK or DT_ERR_TIMEOUT). Reads host-mapped memory and does not
 * synchronize; call after the stream has been synchronized to see errors from finished work.
 * dt_comm_clear_error resets it. */
int dt_comm_error(dt_comm* comm, int rank);
int dt_comm_clear_error(dt_comm* comm, int rank);

/* ---- collectives (called by each rank with its own rank index) ---------------------------------------------- */

/* Partial -> Replicate. out[i] = sum over ranks r = 0..n-1 (in that order) of in_r[i], `count` elements.
 * Replaces ThreadGroup::AllReduce (thread_group.cc:127-141); `in` is not modified (the reference clones it
 * first, :136). in == out is allowed. The rank order holds for every call with DT_RANK_ORDER or
 * DT_ACCUM_STORAGE; without them DT_ALGO_AUTO may pick NVLS or NCCL where those measured faster (flags). */
int dt_all_reduce(dt_comm* comm, int rank, const void* in, void* out, size_t count, int dtype, int op, int flags,
                  void* stream);

/* Partial -> Shard(0). out = rows [rank*out_count, (rank+1)*out_count) of the rank-order sum of every rank's
 * `in` (nranks * out_count elements). Replaces ThreadGroup::ReduceScatterTensor (thread_group.cc:192-209),
 * which requires dim 0 divisible by the group size (:195). Out of place: no input is modified. */
int dt_reduce_scatter(dt_comm* comm, int rank, const void* in, void* out, size_t out_count, int dtype, int op,
                      int flags, void* stream);

/* Shard(d) -> Replicate. Every rank's input is [outer, lens[rank], inner] (inner in bytes: product of the
 * dims after d times the element size); out is [outer, sum(lens), inner], shards concatenated in rank order
 * along d. Covers ThreadGroup::EqualShapeAllGatherIntoTensor (:151-166, d = 0, even), AllGather (:168-171,
 * any d, uneven lens) and AllGatherIntoVec + concat; the concat is fused into the peer stores. */
int dt_all_gather(dt_comm* comm, int rank, const void* in, void* out, size_t outer, const int64_t* lens,
                  size_t inner_bytes, void* stream);

/* Shard(d, s) -> Replicate for the sub-split placement (the causal load-balancing layout of context
 * parallelism): rank r's shard [outer, lens[r], inner] is its piece of the first s + 1 rows (fronts[r] rows)
 * followed by its piece of the rest. out is [outer, sum(lens), inner] with every rank's front part first, in
 * rank order, then every rank's back part. Replaces ThreadGroup::AllGatherIntoVec followed by
 * DistributeGather::GatherShardWithSubSplit (convert_kernel.cc:164-166,
 * distributed_scather_and_gather.cc:147-183) -- a gather and two concatenations -- with one launch of peer
 * stores straight into place. */
int dt_all_gather_sub_split(dt_comm* comm, int rank, const void* in, void* out, size_t outer, const int64_t* lens,
                            const int64_t* fronts, size_t inner_bytes, void* stream);

/* Shard(src_dim) -> Shard(dst_dim). `in` is this rank's contiguous local tensor of shape in_shape[0..ndim-1]
 * (in_shape[src_dim] == src_lens[rank]); src_lens[r] is rank r's extent along src_dim. The dst_dim extent D is
 * split with the reference's rule (first D % n ranks get one more), chunk k goes to rank k, and `out` is
 * rank's chunk from every peer concatenated along src_dim in rank order: shape in_shape with
 * [src_dim] = sum(src_lens) and [dst_dim] = split(D)[rank]. Replaces ThreadGroup::AllToAll
 * (thread_group.cc:211-241): the per-chunk .contiguous() pack and the final concat are fused into the peer
 * stores. */
int dt_all_to_all(dt_comm* comm, int rank, const void* in, void* out, int ndim, const int64_t* in_shape,
                  int src_dim, int dst_dim, const int64_t* src_lens, size_t elem_bytes, void* stream);

/* Several tensors of one local shape swapped Shard(src_dim) -> Shard(dst_dim) in one launch: ins[t] -> outs[t],
 * t < ntensors <= 8, each with the layout rules of dt_all_to_all. The q, k and v swaps of Ulysses context
 * parallelism (python/dtorch/nn/scaled_dot_product_attention_with_cp.py:73-85, three ThreadGroup::AllToAll calls)
 * become one kernel whose peer stores interleave all three tensors. */
int dt_all_to_all_multi(dt_comm* comm, int rank, int ntensors, const void* const* ins, void* const* outs, int ndim,
                        const int64_t* in_shape, int src_dim, int dst_dim, const int64_t* src_lens, size_t elem_bytes,
                        void* stream);

/* The list form of c10d's alltoall (the virtual ThreadGroup::AllToAll calls, thread_group.cc:236, and the
 * same-device backend's alltoall, thread_group_same_device_backend.cc:276-302): ins[k] (in_bytes[k] bytes) is
 * this rank's buffer for rank k, outs[k] (room for out_bytes[k] bytes) receives rank k's buffer for this rank.
 * One launch moves every pair with peer stores; no concatenation or staging copy. Single-process
 * communicators (peer or same-device mode): the ranks exchange their buffer lists in process. Every rank checks
 * every pair (a send larger than its destination's room is DT_ERR_INVALID on all ranks). */
int dt_all_to_all_list(dt_comm* comm, int rank, const void* const* ins, const size_t* in_bytes, void* const* outs,
                       const size_t* out_bytes, void* stream);

/* The list form of c10d's allgather (ThreadGroup::AllGatherIntoVec, thread_group.cc:173-190; same-device
 * allgather, thread_group_same_device_backend.cc:177-201): `in` (in_bytes) goes to every rank; outs[k] (room for
 * out_bytes[k] bytes) receives rank k's input. Shards of different sizes are fine. Single-process
 * communicators, checked like dt_all_to_all_list. */
int dt_all_gather_list(dt_comm* comm, int rank, const void* in, size_t in_bytes, void* const* outs,
                       const size_t* out_bytes, void* stream);

/* Device-side barrier of all ranks on their streams. Replaces ThreadGroup::Barrier (thread_group.cc:118-125). */
int dt_barrier(dt_comm* comm, int rank, void* stream);

/* ---- point-to-point ----------------------------------------------------------------------------------- */

/* Copy `bytes` from src (on src_device) to dst (on dst_device) with a kernel on src_device that stores straight
 * into the destination GPU's memory over NVLink (peer access between the two devices is enabled on first use).
 * `stream` belongs to src_device; the copy is ordered after earlier work on it and complete when it gets past
 * the call -- a consumer on the destination device must wait for that (e.g. an event). Replaces the tensor-store
 * hand-off of a mesh-to-mesh move, ConvertKernel::ConvertDeviceMesh (convert_kernel.cc:79-102) ->
 * TensorStore::DestGetAndToDevice (tensor_store.cc:40-62), and the per-device pieces of gathering a DTensor onto
 * one GPU. src_device == dst_device is a local copy. */
int dt_peer_copy(void* dst, int dst_device, const void* src, int src_device, size_t bytes, void* stream);

/* ---- NVLS buffer (NVLink SHARP) ------------------------------------------------------------------------- */
/* Memory of every rank bound to one NVLink multicast object, so an all-reduce can reduce inside the NVSwitch
 * (dt_all_reduce with DT_ALGO_NVLS). Buffers at the same offset on every rank form one operand. No
 * counterpart in the reference, whose GPU collectives are NCCL's. */

/* *supported = 1 if every local device of the communicator supports NVLink multicast. */
int dt_comm_nvls_supported(dt_comm* comm, int* supported);

/* Single-process peer communicator: allocate `bytes` (rounded up to the multicast granularity) per rank. */
int dt_comm_nvls_alloc(dt_comm* comm, size_t bytes);

/* Multi-process communicator, three steps: one rank creates the multicast object and exports it as a POSIX
 * file descriptor (*fd) that the caller hands to the other processes (e.g. SCM_RIGHTS); then every rank
 * calls dt_comm_nvls_attach (the creator with any fd) to add its device; after every rank has attached,
 * every rank calls dt_comm_nvls_bind to bind and map its memory. The caller closes received descriptors. */
int dt_comm_nvls_create(dt_comm* comm, size_t bytes, int* fd);
int dt_comm_nvls_attach(dt_comm* comm, int fd, size_t bytes);
int dt_comm_nvls_bind(dt_comm* comm);

/* Rank `rank`'s pointer to its NVLS buffer and the buffer size (NULL / 0 if none). */
int dt_comm_nvls_buffer(dt_comm* comm, int rank, void** ptr, size_t* bytes);

/* ---- same-device kernels: all n ranks' buffers on the current device, one launch ------------------------- */
/* These are the kernels a same-device communicator launches; they are exported so a caller that already holds
 * every rank's buffer (the 1-GPU emulation mode, DTORCH_DTENSOR_IN_SAME_DEVICE in the reference) can use them
 * directly. `ins`/`outs` are host arrays of n device pointers. */

/* out = rank-order sum of ins[0..n-1] (the fold of thread_group_same_device_backend.cc:123-130). */
int dt_local_all_reduce(int n, const void* const* ins, void* out, size_t count, int dtype, int flags, void* stream);

/* The same all-reduce for partials that live in host memory (the reference's CPU-mesh all-reduce,
 * ThreadGroup::AllReduce on kCpu tensors, thread_group.cc:127-141, run on one GPU): host_ins[r] (pinned) are
 * copied in chunks into the device staging buffers dev_ins[r]; each chunk is reduced into dev_out as soon as
 * all of its inputs have arrived and copied back into host_out (pinned) while later chunks are still on the
 * way in, so both copy directions and the reduction overlap. Enqueued after the work already on `stream`;
 * host_out is complete once `stream` reaches the end of the call. chunk_bytes: per-rank chunk size (0 = 16 MiB,
 * rounded to 16 bytes; chunks are 16 bytes at least).
 * In place is allowed on both sides: dev_out may equal one of dev_ins[r] and host_out one of host_ins[r] (a
 * chunk's result is written only after all of that chunk's inputs were read). Calls that share staging buffers
 * must be issued on the same stream: a call waits only for earlier work on its own stream. If the call fails
 * part way, `stream` still ends after every copy it had put in flight, so synchronizing `stream` makes the
 * buffers safe to free or reuse. */
int dt_local_all_reduce_host(int n, const void* const* host_ins, void* const* dev_ins, void* dev_out,
                             void* host_out, size_t count, int dtype, int flags, size_t chunk_bytes, void* stream);

/* Size of the device scratch that dt_local_all_reduce_host_noalloc stages through (32 MiB). */
#define DT_NOALLOC_SCRATCH_BYTES (32u << 20)

/* The host-partials all-reduce of dt_local_all_reduce_host for callers that cannot allocate device memory,
 * with no staging buffers to pass in. No counterpart in the reference. It serves callers that hold host tensors
 * only -- the CPU-mesh side of a ThreadGroup has no device buffers of its own to stage through -- and callers
 * whose device memory is owned by another allocator (a serving process that reserved the GPU's memory up front)
 * or that cannot afford cudaMalloc / cudaFree, which may synchronize the whole device.
 * The n partials and the sum are staged in a fixed array inside this library's device image: every GPU on
 * which the library's kernels are loaded holds DT_NOALLOC_SCRATCH_BYTES until the process exits, and the call
 * itself calls no cudaMalloc, cudaFree or other allocating routine. The staging needs n + 1 slots of
 * count * element size bytes, each rounded up to 256 bytes; anything larger is rejected with DT_ERR_INVALID
 * before the device is touched. Runs on the current device; the first call on a device looks up the array's
 * device address, so make that first call before any stream capture. Everything is enqueued on `stream` in
 * order (copies in, one rank-order reduction, copy out; no overlap), and host_out is complete once `stream`
 * reaches the end of the call. host_ins[r] and host_out should be pinned for asynchronous copies. Every call
 * on a device shares the one array, which keeps the last call's contents: calls on one stream are ordered,
 * but calls that overlap on the GPU (different streams, or different host threads) race on it.
 * flags: DT_ACCUM_FP32 or DT_ACCUM_STORAGE, as for dt_local_all_reduce. */
int dt_local_all_reduce_host_noalloc(int n, const void* const* host_ins, void* host_out, size_t count, int dtype,
                                     int flags, void* stream);

/* outs[r] = rows [r*out_count, (r+1)*out_count) of the rank-order sum (same-device _reduce_scatter_base,
 * thread_group_same_device_backend.cc:238-274, without its in-place write into rank 0's input). */
int dt_local_reduce_scatter(int n, const void* const* ins, void* const* outs, size_t out_count, int dtype, int flags,
                            void* stream);

/* out = concat of ins[r] ([outer, lens[r], inner_bytes]) along the middle dim in rank order. */
int dt_local_all_gather(int n, const void* const* ins, void* out, size_t outer, const int64_t* lens,
                        size_t inner_bytes, void* stream);

/* outs[k] = concat over r of chunk k (along dst_dim) of ins[r], along src_dim. Shapes as dt_all_to_all, with
 * ins[r] of shape in_shape except [src_dim] = src_lens[r]. */
int dt_local_all_to_all(int n, const void* const* ins, void* const* outs, int ndim, const int64_t* in_shape,
                        int src_dim, int dst_dim, const int64_t* src_lens, size_t elem_bytes, void* stream);

/* ---- instrumentation -------------------------------------------------------------------------------------- */

/* Number of kernels this library has launched on the calling process since load (all threads). */
uint64_t dt_kernel_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* DTORCH_B200_H */
