// Device code of the redistribute collectives: cross-GPU block barriers, the rank-ordered reduction family
// (one-shot / two-shot all-reduce, reduce-scatter, same-device reduce) and the segment-copy engine (all-gather
// with the concat fused, all-to-all with the shard-dim pack fused).
//
// Everything here is data movement plus an elementwise add, so it is bound by HBM (local buffers) or by
// NVLink (peer buffers): 16-byte vector loads and stores, several independent vectors in flight per thread,
// grids sized to the SM count. Tensor cores are not involved.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dtb {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 1024;  // rows of the per-rank flag array: one row of kMaxRanks flags per block index
constexpr int kThreads = 512;     // threads per block of every kernel
constexpr int kErrTimeout = 3;    // == DT_ERR_TIMEOUT

// ------------------------------------------------------------------------------------------------------------
// Memory-model primitives (PTX ISA: st.release / ld.acquire at system scope, %globaltimer).
// ------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Signals of one rank: flags[r] is rank r's flag array as addressed from this GPU (a peer pointer for r !=
// rank). Row b, column s of rank r's array holds the last barrier value block b of rank s announced to r.
struct SignalCtx {
    uint32_t* flags[kMaxRanks];
    uint32_t* epochs;  // this rank's per-block collective counters (local memory, one per block index)
    int* err;          // this rank's error word (host-mapped)
    int rank;
    int n;
    uint64_t timeout_ns;
};

// Epoch of this launch for block blockIdx.x: the block's own counter in device memory, advanced once per
// launch. Every rank launches the same grid for the same collective, so block b has seen the same number of
// collectives on every rank and agrees with its peers; nothing comes from the host, which keeps a captured
// CUDA graph correct on replay. Barrier values are 2e-1 (start) and 2e (end).
__device__ __forceinline__ uint32_t block_epoch(const SignalCtx& s) {
    __shared__ uint32_t e;
    if (threadIdx.x == 0) {
        e = s.epochs[blockIdx.x] + 1;
        s.epochs[blockIdx.x] = e;
    }
    __syncthreads();
    return e;
}

// Barrier of block blockIdx.x across all ranks: nothing after the barrier starts before every rank's block
// blockIdx.x has announced `value`. Values only grow (two per collective: odd on entry, even on exit), so
// flags are never reset; comparisons are wrap-safe. A wait that outlives timeout_ns records kErrTimeout in the
// error word and the block gives up (returns false) instead of spinning on.
// The exit announcement is a release at system scope after __syncthreads: by cumulativity every store of the
// block into peer outputs (and every load of peer inputs) is ordered before it, with no separate fence. The
// entry announcement is relaxed: what it publishes -- this rank's inputs, written by earlier work on its
// stream, and its outputs, free since that work completed -- is ordered by stream order on this GPU already,
// and a peer reaches that memory through this GPU's L2. (Dropping the fences cut the per-call overhead of a
// 2-rank all-gather from ~19 to ~12.5 us at 1 MiB.)
__device__ __forceinline__ bool block_barrier(const SignalCtx& s, uint32_t value) {
    __syncthreads();
    bool ok = true;
    if (threadIdx.x < s.n) {
        uint32_t* flag = s.flags[threadIdx.x] + blockIdx.x * kMaxRanks + s.rank;
        if (value & 1u) {
            st_relaxed_sys(flag, value);
        } else {
            st_release_sys(flag, value);
        }
        const uint32_t* mine = s.flags[s.rank] + blockIdx.x * kMaxRanks + threadIdx.x;
        uint64_t start = 0;
        uint32_t spins = 0;
        while (static_cast<int32_t>(ld_acquire_sys(mine) - value) < 0) {
            if ((++spins & 31u) == 0) {
                const uint64_t now = global_timer_ns();
                if (start == 0) {
                    start = now;
                } else if (now - start > s.timeout_ns) {
                    *reinterpret_cast<volatile int*>(s.err) = kErrTimeout;
                    ok = false;
                    break;
                }
            }
        }
    }
    return __syncthreads_and(ok) != 0;
}

// ------------------------------------------------------------------------------------------------------------
// Element types. A 16-byte vector holds kPerVec elements; arithmetic is fp32.
// ------------------------------------------------------------------------------------------------------------
template <int DT>
struct Elem;

template <>
struct Elem<0> {  // fp32
    static constexpr int kPerVec = 4;
    static constexpr int kBytes = 4;
    __device__ static __forceinline__ void unpack(const uint4& v, float (&f)[4]) {
        f[0] = __uint_as_float(v.x);
        f[1] = __uint_as_float(v.y);
        f[2] = __uint_as_float(v.z);
        f[3] = __uint_as_float(v.w);
    }
    __device__ static __forceinline__ uint4 pack(const float (&f)[4]) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
    }
    __device__ static __forceinline__ float round_storage(float x) { return x; }
    __device__ static __forceinline__ float load1(const char* p) { return *reinterpret_cast<const float*>(p); }
    __device__ static __forceinline__ void store1(char* p, float x) { *reinterpret_cast<float*>(p) = x; }
};

__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

__device__ __forceinline__ uint32_t float_to_bf16_bits(float x) {
    return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(x)));
}

template <>
struct Elem<1> {  // bf16
    static constexpr int kPerVec = 8;
    static constexpr int kBytes = 2;
    __device__ static __forceinline__ void unpack(const uint4& v, float (&f)[8]) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    __device__ static __forceinline__ uint4 pack(const float (&f)[8]) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = float_to_bf16_bits(f[2 * i]) | (float_to_bf16_bits(f[2 * i + 1]) << 16);
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
    __device__ static __forceinline__ float round_storage(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
    __device__ static __forceinline__ float load1(const char* p) {
        return bf16_bits_to_float(*reinterpret_cast<const uint16_t*>(p));
    }
    __device__ static __forceinline__ void store1(char* p, float x) {
        *reinterpret_cast<uint16_t*>(p) = static_cast<uint16_t>(float_to_bf16_bits(x));
    }
};

template <>
struct Elem<2> {  // fp16
    static constexpr int kPerVec = 8;
    static constexpr int kBytes = 2;
    __device__ static __forceinline__ void unpack(const uint4& v, float (&f)[8]) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[2 * i] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] & 0xffffu)));
            f[2 * i + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[i] >> 16)));
        }
    }
    __device__ static __forceinline__ uint4 pack(const float (&f)[8]) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = __half_as_ushort(__float2half_rn(f[2 * i]));
            const uint32_t hi = __half_as_ushort(__float2half_rn(f[2 * i + 1]));
            w[i] = lo | (hi << 16);
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
    __device__ static __forceinline__ float round_storage(float x) { return __half2float(__float2half_rn(x)); }
    __device__ static __forceinline__ float load1(const char* p) {
        return __half2float(*reinterpret_cast<const __half*>(p));
    }
    __device__ static __forceinline__ void store1(char* p, float x) {
        *reinterpret_cast<__half*>(p) = __float2half_rn(x);
    }
};

// ------------------------------------------------------------------------------------------------------------
// Rank-ordered reduction.
//   acc = x_0; acc = acc + x_1; ...; acc = acc + x_{n-1}     (fp32 adds in this order; STORAGE rounds each
//   partial sum to the storage type, reproducing the reference's in-dtype CPU fold bit for bit)
// One kernel covers: two-shot all-reduce (this rank's chunk, result pushed to every rank's output),
// one-shot all-reduce (whole buffer, own output), reduce-scatter (own chunk, own output, shifted index),
// and the same-device reduce (no barrier, all inputs local).
// ------------------------------------------------------------------------------------------------------------
struct ReduceArgs {
    const char* in[kMaxRanks];  // input of rank r (rank order = summation order)
    char* out[kMaxRanks];       // outputs written with the result, in store order
    SignalCtx sig;
    int64_t vlo, vhi;     // 16-byte vector range of the input this launch reduces
    int64_t slo, shi;     // element range reduced one element at a time (misaligned buffers, tails)
    int64_t out_shift;    // output element index = input element index - out_shift
    int64_t chunk;        // > 0: scatter mode -- element i goes to out[i / chunk] at i % chunk (elements; a
                          // multiple of the vector width when vectors are used), nout unused
    int n;                // number of inputs
    int nout;             // number of outputs
};

template <int DT, int NRMAX, bool STORAGE>
__device__ __forceinline__ void reduce_vectors(const ReduceArgs& a) {
    using E = Elem<DT>;
    constexpr int P = E::kPerVec;
    constexpr int U = NRMAX <= 2 ? 4 : 2;  // independent vectors per thread per iteration
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x * U;
    const uint4* in[NRMAX];
#pragma unroll
    for (int r = 0; r < NRMAX; ++r) in[r] = reinterpret_cast<const uint4*>(a.in[r < a.n ? r : 0]);
    const int64_t vshift = a.out_shift / P;  // host guarantees out_shift % P == 0 on the vector path
    for (int64_t base = a.vlo + static_cast<int64_t>(blockIdx.x) * blockDim.x * U; base < a.vhi; base += step) {
        uint4 x[NRMAX][U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t v = base + u * blockDim.x + threadIdx.x;
            if (v < a.vhi) {
#pragma unroll
                for (int r = 0; r < NRMAX; ++r)
                    if (r < a.n) x[r][u] = in[r][v];
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t v = base + u * blockDim.x + threadIdx.x;
            if (v < a.vhi) {
                float acc[P];
                E::unpack(x[0][u], acc);
#pragma unroll
                for (int r = 1; r < NRMAX; ++r) {
                    if (r < a.n) {
                        float t[P];
                        E::unpack(x[r][u], t);
#pragma unroll
                        for (int e = 0; e < P; ++e) acc[e] = STORAGE ? E::round_storage(acc[e] + t[e]) : acc[e] + t[e];
                    }
                }
                const uint4 o = E::pack(acc);
                if (a.chunk > 0) {
                    const int64_t cv = a.chunk / P;
                    const int64_t k = v / cv;
                    reinterpret_cast<uint4*>(a.out[k])[v - k * cv] = o;
                } else {
                    for (int j = 0; j < a.nout; ++j) reinterpret_cast<uint4*>(a.out[j])[v - vshift] = o;
                }
            }
        }
    }
}

template <int DT, bool STORAGE>
__device__ __forceinline__ void reduce_scalars(const ReduceArgs& a) {
    using E = Elem<DT>;
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = a.slo + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.shi; i += step) {
        float acc = E::load1(a.in[0] + i * E::kBytes);
        for (int r = 1; r < a.n; ++r) {
            const float t = E::load1(a.in[r] + i * E::kBytes);
            acc = STORAGE ? E::round_storage(acc + t) : acc + t;
        }
        if (a.chunk > 0) {
            const int64_t k = i / a.chunk;
            E::store1(a.out[k] + (i - k * a.chunk) * E::kBytes, acc);
        } else {
            for (int j = 0; j < a.nout; ++j) E::store1(a.out[j] + (i - a.out_shift) * E::kBytes, acc);
        }
    }
}

template <int DT, int NRMAX, bool STORAGE, bool BARRIER>
__global__ void __launch_bounds__(kThreads) k_reduce(const __grid_constant__ ReduceArgs a) {
    uint32_t e = 0;
    if (BARRIER) {
        e = block_epoch(a.sig);
        if (!block_barrier(a.sig, 2 * e - 1)) return;
    }
    reduce_vectors<DT, NRMAX, STORAGE>(a);
    reduce_scalars<DT, STORAGE>(a);
    if (BARRIER) block_barrier(a.sig, 2 * e);
}

// ------------------------------------------------------------------------------------------------------------
// Segment-copy engine. A segment set moves rows of `run` contiguous bytes; rows are indexed by (i0, i1, i2)
// with independent source and destination byte strides. All-gather along any dim and the all-to-all pack
// and concat are all such sets: the strided read of the shard-dim slice and the placement at the concat
// offset happen inside the copy, so no separate contiguous() or concat pass touches HBM.
// Work item = one piece of up to seg_bytes of one row, copied by one warp with the segment's own access
// width (16-byte vectors when its pointers, strides and run allow, narrower otherwise -- one odd segment
// does not slow the others down). Items of different destinations are interleaved so every peer link is
// busy at once.
// ------------------------------------------------------------------------------------------------------------
struct Seg {
    const char* src;
    char* dst;
    int64_t run;       // bytes per row
    int64_t cnt[3];    // row index extents (i0, i1, i2)
    int64_t ss[3];     // source byte strides
    int64_t ds[3];     // destination byte strides
    int64_t spr;       // pieces per row
    int64_t items;     // rows * spr, or ceil(rows / rpi) for short rows
    int32_t vw;        // access width in bytes: 16, 8, 4, 2 or 1
    int32_t seg_bytes; // bytes per piece (CopyGeom<vw>::kSegBytes)
    int32_t rpi;       // > 1: short rows, rpi whole rows per item, one access per lane slot
    int32_t vpr;       // short rows: accesses per row
};

template <int MAXSEG>
struct CopyArgs {
    Seg seg[MAXSEG];
    SignalCtx sig;
    int64_t max_items;  // max over segs of items
    int nseg;
};

template <int VW>
struct VecOf;
template <>
struct VecOf<16> { using T = uint4; };
template <>
struct VecOf<8> { using T = uint2; };
template <>
struct VecOf<4> { using T = uint32_t; };
template <>
struct VecOf<2> { using T = uint16_t; };
template <>
struct VecOf<1> { using T = uint8_t; };

template <int VW>
struct CopyGeom {
    static constexpr int kU = VW >= 8 ? 4 : 8;        // vectors per lane per item
    static constexpr int kSegBytes = 32 * VW * kU;    // bytes per item
};

// One piece (`len` bytes at src -> dst) copied by one warp with VW-byte accesses: all loads first, then all
// stores, so each lane has kU independent accesses in flight.
template <int VW>
__device__ __forceinline__ void copy_piece(const char* src, char* dst, int64_t len, int lane) {
    using V = typename VecOf<VW>::T;
    constexpr int U = CopyGeom<VW>::kU;
    const V* s = reinterpret_cast<const V*>(src);
    V* d = reinterpret_cast<V*>(dst);
    V buf[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t off = static_cast<int64_t>(u * 32 + lane) * VW;
        if (off < len) buf[u] = s[u * 32 + lane];
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t off = static_cast<int64_t>(u * 32 + lane) * VW;
        if (off < len) d[u * 32 + lane] = buf[u];
    }
}

// Pieces of segments whose pointers, strides or run are not 16-byte multiples: the same work with 8-, 4-, 2- or
// 1-byte accesses, a plain strided loop per lane. Kept out of line and lean so that it does not weigh on the
// registers of the 16-byte path around it; such segments are the exception (odd shard extents).
template <typename V>
__device__ __forceinline__ void copy_strided(const char* src, char* dst, int64_t len, int lane) {
    constexpr int64_t W = sizeof(V);
    for (int64_t o = lane * W; o < len; o += 32 * W)
        *reinterpret_cast<V*>(dst + o) = *reinterpret_cast<const V*>(src + o);
}

__device__ __noinline__ void copy_piece_narrow(const char* src, char* dst, int64_t len, int lane, int vw) {
    switch (vw) {
        case 8: copy_strided<uint2>(src, dst, len, lane); break;
        case 4: copy_strided<uint32_t>(src, dst, len, lane); break;
        case 2: copy_strided<uint16_t>(src, dst, len, lane); break;
        default: copy_strided<uint8_t>(src, dst, len, lane); break;
    }
}

constexpr int kShortRowSlotsDev = 4 * 32;  // accesses per short-row item (kShortRowSlots on the host)

// Rows much shorter than an item (the all-to-all of a narrow dst-dim chunk, an all-gather of a thin shard): one
// item holds `rpi` whole rows and each lane slot moves one access of one row, so every lane works instead of
// one lane per row. Out of line, like the narrow path.
template <typename V>
__device__ __forceinline__ void copy_rows_v(const Seg& s, int64_t j, int lane) {
    constexpr int64_t W = sizeof(V);
    const int64_t rows = s.cnt[0] * s.cnt[1] * s.cnt[2];
#pragma unroll 1
    for (int f = lane; f < kShortRowSlotsDev; f += 32) {
        const int r = f / s.vpr;
        const int64_t row = j * s.rpi + r;
        if (r >= s.rpi || row >= rows) break;
        const int64_t off = static_cast<int64_t>(f - r * s.vpr) * W;
        if (off >= s.run) continue;
        const int64_t i2 = row % s.cnt[2];
        const int64_t r01 = row / s.cnt[2];
        const int64_t i1 = r01 % s.cnt[1];
        const int64_t i0 = r01 / s.cnt[1];
        *reinterpret_cast<V*>(s.dst + i0 * s.ds[0] + i1 * s.ds[1] + i2 * s.ds[2] + off) =
            *reinterpret_cast<const V*>(s.src + i0 * s.ss[0] + i1 * s.ss[1] + i2 * s.ss[2] + off);
    }
}

__device__ __noinline__ void copy_short_rows(const Seg& s, int64_t j, int lane) {
    switch (s.vw) {
        case 16: copy_rows_v<uint4>(s, j, lane); break;
        case 8: copy_rows_v<uint2>(s, j, lane); break;
        case 4: copy_rows_v<uint32_t>(s, j, lane); break;
        case 2: copy_rows_v<uint16_t>(s, j, lane); break;
        default: copy_rows_v<uint8_t>(s, j, lane); break;
    }
}

template <int MAXSEG, bool BARRIER>
__global__ void __launch_bounds__(kThreads) k_copy(const __grid_constant__ CopyArgs<MAXSEG> a) {
    uint32_t e = 0;
    if (BARRIER) {
        e = block_epoch(a.sig);
        if (!block_barrier(a.sig, 2 * e - 1)) return;
    }
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t total = a.max_items * a.nseg;
    for (int64_t t = warp; t < total; t += nwarps) {
        const int d = static_cast<int>(t % a.nseg);
        const int64_t j = t / a.nseg;
        const Seg& s = a.seg[d];
        if (j >= s.items) continue;
        if (s.rpi > 1) {
            copy_short_rows(s, j, lane);
            continue;
        }
        int64_t row = j, sg = 0;
        if (s.spr != 1) {
            row = j / s.spr;
            sg = j - row * s.spr;
        }
        int64_t so = sg * s.seg_bytes, dof = sg * s.seg_bytes;
        if (s.cnt[0] == 1 && s.cnt[1] == 1) {
            so += row * s.ss[2];
            dof += row * s.ds[2];
        } else {
            const int64_t i2 = row % s.cnt[2];
            const int64_t r01 = row / s.cnt[2];
            const int64_t i1 = r01 % s.cnt[1];
            const int64_t i0 = r01 / s.cnt[1];
            so += i0 * s.ss[0] + i1 * s.ss[1] + i2 * s.ss[2];
            dof += i0 * s.ds[0] + i1 * s.ds[1] + i2 * s.ds[2];
        }
        const int64_t len = min(static_cast<int64_t>(s.seg_bytes), s.run - sg * s.seg_bytes);
        if (s.vw == 16) {
            copy_piece<16>(s.src + so, s.dst + dof, len, lane);
        } else {
            copy_piece_narrow(s.src + so, s.dst + dof, len, lane, s.vw);
        }
    }
    if (BARRIER) block_barrier(a.sig, 2 * e);
}

// ------------------------------------------------------------------------------------------------------------
// NVLS all-reduce: the buffers live in memory bound to one NVLink multicast object, so one multimem load
// returns the sum of every rank's copy, reduced inside the NVSwitch (fp32 accumulation for bf16/fp16), and
// one multimem store writes the result into every rank's copy. Rank c handles chunk c. Per GPU this moves
// (1 + 1/n)·S each way instead of the two-shot's 2(n-1)/n·S; the summation order is the switch's, not rank
// order (within the reductions' tolerance, not bit-identical to the rank-order fold).
// ------------------------------------------------------------------------------------------------------------
struct NvlsArgs {
    SignalCtx sig;
    const char* mc_in;  // multicast address of the input
    char* mc_out;       // multicast address of the output
    int64_t vlo, vhi;   // 16-byte vectors handled by this rank
};

template <int DT>
__device__ __forceinline__ uint4 multimem_ld_reduce_v4(const void* p);

template <>
__device__ __forceinline__ uint4 multimem_ld_reduce_v4<0>(const void* p) {
    uint4 r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}

template <>
__device__ __forceinline__ uint4 multimem_ld_reduce_v4<1>(const void* p) {
    uint4 r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}

template <>
__device__ __forceinline__ uint4 multimem_ld_reduce_v4<2>(const void* p) {
    uint4 r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}

__device__ __forceinline__ void multimem_st_v4(void* p, const uint4& v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

template <int DT>
__global__ void __launch_bounds__(kThreads) k_allreduce_nvls(const __grid_constant__ NvlsArgs a) {
    const uint32_t e = block_epoch(a.sig);
    if (!block_barrier(a.sig, 2 * e - 1)) return;
    constexpr int U = 4;
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x * U;
    for (int64_t base = a.vlo + static_cast<int64_t>(blockIdx.x) * blockDim.x * U; base < a.vhi; base += step) {
        uint4 r[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t v = base + u * blockDim.x + threadIdx.x;
            if (v < a.vhi) r[u] = multimem_ld_reduce_v4<DT>(a.mc_in + v * 16);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t v = base + u * blockDim.x + threadIdx.x;
            if (v < a.vhi) multimem_st_v4(a.mc_out + v * 16, r[u]);
        }
    }
    // the stores went through the multicast alias; peers read the same memory through their unicast mapping
    asm volatile("fence.proxy.alias;" ::: "memory");
    block_barrier(a.sig, 2 * e);
}

// Barrier-only kernel (ThreadGroup::Barrier): one block, both phases of the epoch.
__global__ void k_barrier(const __grid_constant__ SignalCtx s) {
    const uint32_t e = block_epoch(s);
    if (block_barrier(s, 2 * e - 1)) block_barrier(s, 2 * e);
}

}  // namespace dtb
