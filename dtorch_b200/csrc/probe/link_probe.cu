// Link probe: peer-copy throughput of the transfer mechanisms a collective can use over NVLink -- SM 16-byte
// vector copies and TMA bulk copies (cp.async.bulk global -> shared -> global), run on the source GPU (remote
// stores, "push") or on the destination GPU (remote loads, "pull"). A diagnostic for `bench.py --link-probe`,
// not part of the collective path; it tells what per-direction bandwidth the fabric sustains, which bounds
// the bus bandwidth of every P2P collective.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

extern "C" {

__global__ void k_lsu_copy(const uint4* __restrict__ src, uint4* __restrict__ dst, long long nvec) {
    const long long stride = (long long)gridDim.x * blockDim.x * 4;
    for (long long base = (long long)blockIdx.x * blockDim.x * 4; base < nvec; base += stride) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            long long i = base + u * blockDim.x + threadIdx.x;
            if (i < nvec) v[u] = src[i];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            long long i = base + u * blockDim.x + threadIdx.x;
            if (i < nvec) dst[i] = v[u];
        }
    }
}

}  // extern "C"

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// TMA bulk copy through shared memory: chunks of CHUNK bytes, STAGES buffers, one thread drives.
// bytes must be a multiple of 16 and pointers 16-byte aligned (checked by the host).
template <int CHUNK, int STAGES>
__global__ void k_tma_copy(const char* __restrict__ src, char* __restrict__ dst, long long bytes, int* err) {
    extern __shared__ __align__(128) char smem[];
    __shared__ __align__(8) uint64_t mbar[STAGES];
    if (threadIdx.x != 0) return;
    for (int s = 0; s < STAGES; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&mbar[s])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const long long nchunks = (bytes + CHUNK - 1) / CHUNK;
    // my chunks: blockIdx.x, blockIdx.x + gridDim.x, ...
    long long my_n = 0;
    if (blockIdx.x < nchunks) my_n = (nchunks - 1 - blockIdx.x) / gridDim.x + 1;
    auto chunk_off = [&](long long i) { return (blockIdx.x + i * gridDim.x) * (long long)CHUNK; };
    auto chunk_len = [&](long long i) {
        long long o = chunk_off(i);
        long long l = bytes - o;
        return (uint32_t)(l < CHUNK ? l : CHUNK);
    };
    auto issue_load = [&](long long i) {
        const int s = (int)(i % STAGES);
        const uint32_t len = chunk_len(i);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&mbar[s])), "r"(len) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         smem_u32(smem + s * CHUNK)),
                     "l"(src + chunk_off(i)), "r"(len), "r"(smem_u32(&mbar[s]))
                     : "memory");
    };
    for (long long i = 0; i < my_n && i < STAGES; ++i) issue_load(i);
    for (long long i = 0; i < my_n; ++i) {
        const int s = (int)(i % STAGES);
        const uint32_t parity = (uint32_t)((i / STAGES) & 1);
        uint32_t done = 0;
        long long spins = 0;
        while (!done) {
            asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                         : "=r"(done)
                         : "r"(smem_u32(&mbar[s])), "r"(parity)
                         : "memory");
            if (!done && ++spins > (1ll << 26)) {
                *err = 1;
                asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
                return;
            }
        }
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst + chunk_off(i)),
                     "r"(smem_u32(smem + s * CHUNK)), "r"(chunk_len(i))
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        // reload the stage of chunk i-1 once its store has finished reading shared memory
        if (i >= 1 && i - 1 + STAGES < my_n) {
            asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
            issue_load(i - 1 + STAGES);
        }
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

extern "C" {

int probe_lsu(const void* src, void* dst, long long bytes, int grid, int block, void* stream) {
    k_lsu_copy<<<grid, block, 0, (cudaStream_t)stream>>>((const uint4*)src, (uint4*)dst, bytes / 16);
    return (int)cudaGetLastError();
}

#define TMA_VARIANT(CH, ST)                                                                                    \
    if (chunk == CH && stages == ST) {                                                                         \
        k_tma_copy<CH, ST><<<grid, 32, CH * ST, (cudaStream_t)stream>>>((const char*)src, (char*)dst, bytes, err); \
        return (int)cudaGetLastError();                                                                        \
    }

int probe_tma(const void* src, void* dst, long long bytes, int grid, int chunk, int stages, int* err, void* stream) {
    if (((uintptr_t)src | (uintptr_t)dst | (uintptr_t)bytes) & 15) return -1;
    TMA_VARIANT(16384, 4)
    TMA_VARIANT(32768, 4)
    TMA_VARIANT(32768, 6)
    TMA_VARIANT(65536, 3)
    TMA_VARIANT(8192, 8)
    return -2;
}

// cudaFuncSetAttribute is per device: call on every device before use
int probe_prepare(void) {
    cudaFuncSetAttribute(k_tma_copy<16384, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 16384 * 4);
    cudaFuncSetAttribute(k_tma_copy<32768, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 32768 * 4);
    cudaFuncSetAttribute(k_tma_copy<32768, 6>, cudaFuncAttributeMaxDynamicSharedMemorySize, 32768 * 6);
    cudaFuncSetAttribute(k_tma_copy<65536, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, 65536 * 3);
    cudaFuncSetAttribute(k_tma_copy<8192, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8192 * 8);
    return (int)cudaGetLastError();
}

int probe_enable_peer(int a, int b) {
    int prev;
    cudaGetDevice(&prev);
    cudaSetDevice(a);
    cudaError_t e = cudaDeviceEnablePeerAccess(b, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        e = cudaSuccess;
    }
    cudaSetDevice(prev);
    return (int)e;
}

int probe_set_device(int d) { return (int)cudaSetDevice(d); }
}
