/*
 * dt_oracle.c -- TEST INFRASTRUCTURE ONLY. A plain-C restatement, on the CPU, of what the reference's
 * same-device thread-group backend computes for the four redistribute collectives. It is the checker that
 * the parity tests, __graft_entry__.smoke() and bench.py's cpu_baseline leg compare the CUDA path against;
 * nothing in the product links or calls it.
 *
 * Reference being restated (tingkuanpei/dtorch):
 *   all-reduce      dtorch/core/communication/thread_group/thread_group_same_device_backend.cc:111-146
 *                   rank 0 folds result = in_0; result += in_r for r = 1..n-1 (torch CPU add_ in the tensor's
 *                   dtype: each partial sum is rounded to the storage type), every rank gets that tensor.
 *   all-gather      thread_group_same_device_backend.cc:203-236 (_allgather_base: concat along dim 0 in rank
 *                   order) and :177-201 + thread_group.cc:168-190 (allgather list + torch::concat(dim)).
 *   reduce-scatter  thread_group_same_device_backend.cc:238-274: the same fold over the full tensor, then
 *                   torch::chunk(n, 0)[rank].
 *   all-to-all      thread_group.cc:211-241: split(input, GetShardSizeForAllRank(size(dst), n), dst), chunk k
 *                   to rank k, concat(received, src) in rank order.
 *   shard sizes     dtorch/api/cpp/distributed_spec.cc:202-213: the first L % n ranks get floor(L/n) + 1.
 *
 * Floating point: fp32 sums are a strict left fold in single precision (built with -ffp-contract=off, SSE
 * arithmetic); bf16/fp16 sums convert both operands to fp32, add once in fp32 and round the sum to the
 * storage type with round-to-nearest-even (the behaviour of torch's CPU add for reduced-precision types).
 * `storage_round = 0` instead keeps the fp32 accumulator across the whole fold and rounds once at the end --
 * the semantics of the CUDA kernels' default mode, used to check them bit-for-bit too.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

/* ---- number formats --------------------------------------------------------------------------------------- */

static float bits_to_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint32_t f32_to_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

/* bf16 is the top half of an IEEE binary32. Round to nearest, ties to even, by adding 0x7fff plus the lowest
 * kept bit before truncating; NaN maps to the canonical quiet NaN 0x7fc0. */
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u = f32_to_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t h) { return bits_to_f32((uint32_t)h << 16); }

/* IEEE binary16 from binary32, round to nearest even, from the format definition: 1 sign bit, 5 exponent
 * bits (bias 15), 10 fraction bits; subnormals below 2^-14; overflow to infinity. */
uint16_t oracle_f32_to_f16(float f) {
    const uint32_t u = f32_to_bits(f);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t absu = u & 0x7fffffffu;
    if (absu > 0x7f800000u) return (uint16_t)(sign | 0x7e00u); /* NaN */
    if (absu == 0x7f800000u) return (uint16_t)(sign | 0x7c00u); /* inf */
    const int exp = (int)(absu >> 23) - 127;                      /* unbiased exponent */
    uint32_t mant = (absu & 0x7fffffu) | 0x800000u;               /* 24-bit significand with hidden bit */
    if (absu == 0) return sign;
    if (exp > 15) return (uint16_t)(sign | 0x7c00u);              /* overflow */
    int shift;                                                    /* bits dropped from the 24-bit significand */
    uint32_t hexp;
    if (exp >= -14) {
        shift = 13; /* normal half: keep 11 bits */
        hexp = (uint32_t)(exp + 15);
    } else {
        shift = 13 + (-14 - exp); /* subnormal half */
        hexp = 0;
        if (shift > 24) return sign; /* rounds to zero (below half of the smallest subnormal) */
    }
    uint32_t kept = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (kept & 1u))) kept += 1;
    if (hexp == 0) {
        /* subnormal: kept is the fraction; a carry into bit 10 becomes the smallest normal, which the
         * encoding below produces naturally */
        return (uint16_t)(sign | kept);
    }
    /* normal: kept has the hidden bit at bit 10; a carry to bit 11 bumps the exponent */
    if (kept & 0x800u) {
        kept >>= 1;
        hexp += 1;
        if (hexp >= 31) return (uint16_t)(sign | 0x7c00u);
    }
    return (uint16_t)(sign | (hexp << 10) | (kept & 0x3ffu));
}

float oracle_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    if (e == 0) {
        if (m == 0) return bits_to_f32(sign);
        /* subnormal: m * 2^-24 is exact in binary32 */
        const float v = (float)m * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    if (e == 31) return bits_to_f32(sign | 0x7f800000u | (m << 13));
    return bits_to_f32(sign | ((e + 112u) << 23) | (m << 13));
}

/* dtype codes match include/dtorch_b200.h: 0 fp32, 1 bf16, 2 fp16 */
static float load_elem(const void* p, size_t i, int dtype) {
    switch (dtype) {
        case 0: return ((const float*)p)[i];
        case 1: return oracle_bf16_to_f32(((const uint16_t*)p)[i]);
        default: return oracle_f16_to_f32(((const uint16_t*)p)[i]);
    }
}

static float round_storage(float x, int dtype) {
    switch (dtype) {
        case 0: return x;
        case 1: return oracle_bf16_to_f32(oracle_f32_to_bf16(x));
        default: return oracle_f16_to_f32(oracle_f32_to_f16(x));
    }
}

static void store_elem(void* p, size_t i, float x, int dtype) {
    switch (dtype) {
        case 0: ((float*)p)[i] = x; break;
        case 1: ((uint16_t*)p)[i] = oracle_f32_to_bf16(x); break;
        default: ((uint16_t*)p)[i] = oracle_f32_to_f16(x); break;
    }
}

/* ---- placement arithmetic --------------------------------------------------------------------------------- */

/* Placement::GetShardSizeForAllRank (distributed_spec.cc:202-213). */
void oracle_shard_sizes(int64_t L, int n, int64_t* out) {
    for (int i = 0; i < n; ++i) out[i] = L / n + ((int64_t)i < L % n ? 1 : 0);
}

/* ---- collectives ------------------------------------------------------------------------------------------ */

/* Rank-order fold of n buffers of `count` elements (thread_group_same_device_backend.cc:123-130). */
void oracle_fold_sum(int n, const void* const* ins, void* out, size_t count, int dtype, int storage_round) {
    for (size_t i = 0; i < count; ++i) {
        float acc = load_elem(ins[0], i, dtype);
        for (int r = 1; r < n; ++r) {
            const float x = load_elem(ins[r], i, dtype);
            acc = acc + x;
            if (storage_round) acc = round_storage(acc, dtype);
        }
        store_elem(out, i, acc, dtype);
    }
}

/* Reduce-scatter: fold of the full inputs, rank k keeps rows [k*out_count, (k+1)*out_count)
 * (thread_group_same_device_backend.cc:238-274; torch::chunk of an evenly divisible dim 0). */
void oracle_reduce_scatter(int n, const void* const* ins, void* const* outs, size_t out_count, int dtype,
                           int storage_round) {
    const size_t es = dtype == 0 ? 4 : 2;
    for (int k = 0; k < n; ++k) {
        const void* shifted[8];
        for (int r = 0; r < n; ++r) shifted[r] = (const char*)ins[r] + (size_t)k * out_count * es;
        oracle_fold_sum(n, shifted, outs[k], out_count, dtype, storage_round);
    }
}

/* All-gather: rank inputs [outer, lens[r], inner] concatenated along the middle dim in rank order
 * (_allgather_base for dim 0; allgather + torch::concat(dim) otherwise). */
void oracle_all_gather(int n, const void* const* ins, void* out, size_t outer, const int64_t* lens,
                       size_t inner_bytes) {
    int64_t total = 0;
    for (int r = 0; r < n; ++r) total += lens[r];
    for (size_t o = 0; o < outer; ++o) {
        int64_t off = 0;
        for (int r = 0; r < n; ++r) {
            const size_t run = (size_t)lens[r] * inner_bytes;
            memcpy((char*)out + (o * (size_t)total + (size_t)off) * inner_bytes,
                   (const char*)ins[r] + o * run, run);
            off += lens[r];
        }
    }
}

/* All-to-all (thread_group.cc:211-241): output k is the concatenation along src, in rank order, of chunk k
 * (along dst, split with the shard rule) of every rank's input. Walked over the output's index space: for each
 * output index, the source rank i is the one whose src-dim range holds the src coordinate, and the element is
 * rank i's input at the same coordinates except src (minus rank i's offset) and dst (plus chunk k's offset).
 * The dims after both src and dst are contiguous on both sides, so each index of the leading dims copies that
 * whole trailing run at once. A NULL outs[k] skips destination k (a checker that holds one rank's output
 * computes only that one). */
void oracle_all_to_all(int n, const void* const* ins, void* const* outs, int ndim, const int64_t* in_shape,
                       int src_dim, int dst_dim, const int64_t* src_lens, size_t elem_bytes) {
    int64_t split[8], doff[8], soff[8];
    const int64_t D = in_shape[dst_dim];
    oracle_shard_sizes(D, n, split);
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
    const int64_t A = acc;
    const int lead = (src_dim > dst_dim ? src_dim : dst_dim) + 1; /* dims [0, lead) are walked */
    int64_t run = 1;
    for (int d = lead; d < ndim; ++d) run *= in_shape[d];
    const size_t run_bytes = (size_t)run * elem_bytes;
    for (int k = 0; k < n; ++k) {
        if (outs[k] == NULL) continue;
        int64_t oshape[16];
        for (int d = 0; d < ndim; ++d) oshape[d] = in_shape[d];
        oshape[src_dim] = A;
        oshape[dst_dim] = split[k];
        int64_t total = 1;
        for (int d = 0; d < lead; ++d) total *= oshape[d];
        int64_t idx[16];
        for (int64_t e = 0; e < total; ++e) {
            int64_t rem = e;
            for (int d = lead - 1; d >= 0; --d) {
                idx[d] = rem % oshape[d];
                rem /= oshape[d];
            }
            int i = 0;
            while (i + 1 < n && idx[src_dim] >= soff[i + 1]) ++i;
            /* skip empty ranks */
            while (i < n && idx[src_dim] >= soff[i] + src_lens[i]) ++i;
            int64_t ishape[16];
            for (int d = 0; d < ndim; ++d) ishape[d] = in_shape[d];
            ishape[src_dim] = src_lens[i];
            int64_t lin = 0;
            for (int d = 0; d < lead; ++d) {
                int64_t c = idx[d];
                if (d == src_dim) c -= soff[i];
                if (d == dst_dim) c += doff[k];
                lin = lin * ishape[d] + c;
            }
            memcpy((char*)outs[k] + (size_t)e * run_bytes, (const char*)ins[i] + (size_t)lin * run_bytes, run_bytes);
        }
    }
}
