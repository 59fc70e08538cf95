// device_common.cuh -- device helpers shared by the sampling kernels:
// mbarrier / bulk-async copy PTX wrappers, the xorshift coin, 64-bit key
// sorting and the candidate key/bin encodings.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2s {
namespace {

constexpr int kBins = 2048;
constexpr int kBinShift = 17;  // 64 bins per binade of p
constexpr uint32_t kOneTop = 0x3F800000u >> kBinShift;
constexpr unsigned kSpinLimit = 1u << 22;  // polls of a bounded mbarrier wait (~0.5 s)
constexpr uint32_t kFullMask = 0xFFFFFFFFu;

// Row flags (mirrors of the public SAMPLER_ROW_* values)
constexpr int kFlagNan = 1, kFlagNoCand = 2, kFlagSlow = 4, kFlagSerial = 8, kFlagTimeout = 16;


// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned long long* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, unsigned bytes,
                                              unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after `limit` polls (kSpinLimit by default)
// instead of hanging the SM.
__device__ bool mbar_wait_bounded(unsigned long long* bar, unsigned parity, unsigned limit = kSpinLimit) {
    for (unsigned i = 0; i < limit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (i > 32) __nanosleep(64);
    }
    return false;
}


// Tiled 3-D tensor load (TMA) into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z,
                                            unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Named barrier over `count` threads (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// 2^x by the hardware approximation (approximate sums only: binade guesses
// and nucleus-size estimates, never a value the reference computes).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// xorshift* draw + 24-bit float, llama2.c:1071-1080.
__device__ __forceinline__ float draw_coin(unsigned long long& s) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    const unsigned u = (unsigned)((s * 0x2545F4914F6CDD1Dull) >> 32);
    return __fdiv_rn((float)(u >> 8), 16777216.0f);
}



// x / T for a row-constant divisor T with rT = RN(1/T): the product and one
// FMA correction step (P. Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990), which
// yields the correctly rounded quotient while no intermediate leaves the
// normal range.  Used where it was verified exhaustively against IEEE
// division (|T| in [2^-10, 2^10], |x| in [2^-60, 2^60]); IEEE division
// elsewhere.
__device__ __forceinline__ float xm_div_const(float x, float T, float rT) {
    const float ax = fabsf(x), aT = fabsf(T);
    if (ax >= 0x1p-60f && ax <= 0x1p60f && aT >= 0x1p-10f && aT <= 0x1p10f) {
        const float q = __fmul_rn(x, rT);
        const float r = __fmaf_rn(-q, T, x);
        return __fmaf_rn(r, rT, q);
    }
    return __fdiv_rn(x, T);
}

// ---------------------------------------------------------------------------
// Sorting of 64-bit keys, descending; candidate keys and bins
// ---------------------------------------------------------------------------
template <int R>
__device__ void warp_sort_desc(unsigned long long* seg, int n, int lane) {
    constexpr int P = 32 * R;
    unsigned long long k[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int i = r * 32 + lane;
        k[r] = (i < n) ? seg[i] : 0ull;
    }
#pragma unroll
    for (int size = 2; size <= P; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            unsigned long long nk[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int i = r * 32 + lane;
                unsigned long long other;
                if (stride >= 32) {
                    other = k[r ^ (stride >> 5)];
                } else {
                    other = __shfl_xor_sync(kFullMask, k[r], stride);
                }
                const bool desc = (i & size) == 0;
                const bool lower = (i & stride) == 0;
                const bool take_max = (lower == desc);
                nk[r] = take_max ? (k[r] > other ? k[r] : other) : (k[r] < other ? k[r] : other);
            }
#pragma unroll
            for (int r = 0; r < R; ++r) k[r] = nk[r];
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int i = r * 32 + lane;
        if (i < n) seg[i] = k[r];
    }
}

// Block-wide bitonic sort (descending) of a power-of-two array `a` of P keys.
// Works for shared or global memory (the block barrier orders both).
__device__ void block_bitonic_desc(unsigned long long* a, int P) {
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int q = threadIdx.x; q < (P >> 1); q += blockDim.x) {
                const int i = 2 * stride * (q / stride) + (q % stride);
                const int l = i + stride;
                const bool desc = (i & size) == 0;
                const unsigned long long x = a[i], y = a[l];
                if (desc ? (x < y) : (x > y)) {
                    a[i] = y;
                    a[l] = x;
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ unsigned long long cand_key(float p, int idx) {
    return ((unsigned long long)__float_as_uint(p) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ float key_prob(unsigned long long k) { return __uint_as_float((uint32_t)(k >> 32)); }
__device__ __forceinline__ int key_index(unsigned long long k) { return (int)(0xFFFFFFFFu - (uint32_t)k); }

__device__ __forceinline__ int bin_of(float p) {
    const int b = (int)kOneTop - (int)(__float_as_uint(p) >> kBinShift);
    return b < 0 ? 0 : (b >= kBins ? kBins - 1 : b);
}
__device__ __forceinline__ float bin_lo(int b) {
    return (b >= kBins - 1) ? 0.0f : __uint_as_float((kOneTop - (uint32_t)b) << kBinShift);
}

// Sorts the keys of one histogram bin (every key's value shares its top 15
// bits, so (low 17 value bits, 0x7FFF - index) orders them exactly as the
// 64-bit key does, for indices < 2^15 - 1, so that every real key is
// nonzero) with 32-bit keys in registers: half the shuffles of the 64-bit
// sort.  Not for the last bin, which collects everything below it.
template <int R>
__device__ void warp_sort_bin(unsigned long long* seg, int n, int lane) {
    constexpr int P = 32 * R;
    uint32_t k[R];
    uint32_t top = 0u;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int i = r * 32 + lane;
        const unsigned long long key = (i < n) ? seg[i] : 0ull;
        const uint32_t vb = (uint32_t)(key >> 32);
        if (i < n) top = vb >> 17;
        k[r] = (i < n) ? (((vb & 0x1FFFFu) << 15) | (uint32_t)(0x7FFF - key_index(key))) : 0u;
    }
    top = __shfl_sync(kFullMask, top, 0);  // lane 0 always holds a key (n >= 1)
#pragma unroll
    for (int size = 2; size <= P; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            uint32_t nk[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int i = r * 32 + lane;
                const uint32_t other = (stride >= 32) ? k[r ^ (stride >> 5)] : __shfl_xor_sync(kFullMask, k[r], stride);
                const bool desc = (i & size) == 0;
                const bool lower = (i & stride) == 0;
                nk[r] = (lower == desc) ? max(k[r], other) : min(k[r], other);
            }
#pragma unroll
            for (int r = 0; r < R; ++r) k[r] = nk[r];
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int i = r * 32 + lane;
        if (i < n) seg[i] = cand_key(__uint_as_float((top << 17) | (k[r] >> 15)), 0x7FFF - (int)(k[r] & 0x7FFFu));
    }
}

// Two bins of 1..32 keys each (not the last bin; indices < 2^15 - 1) sorted
// together: the two 32-key networks run in lockstep so their shuffle
// latencies overlap.
__device__ void warp_sort_bin_pair(unsigned long long* sa, int na, unsigned long long* sb, int nb, int lane) {
    auto k32 = [](unsigned long long key) {
        return ((((uint32_t)(key >> 32)) & 0x1FFFFu) << 15) | (uint32_t)(0x7FFF - key_index(key));
    };
    const unsigned long long a0 = (lane < na) ? sa[lane] : 0ull;
    const unsigned long long b0 = (lane < nb) ? sb[lane] : 0ull;
    const uint32_t ta = __shfl_sync(kFullMask, (uint32_t)(a0 >> 32) >> 17, 0);
    const uint32_t tb = __shfl_sync(kFullMask, (uint32_t)(b0 >> 32) >> 17, 0);
    uint32_t ka = (lane < na) ? k32(a0) : 0u;
    uint32_t kb = (lane < nb) ? k32(b0) : 0u;
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const uint32_t oa = __shfl_xor_sync(kFullMask, ka, stride);
            const uint32_t ob = __shfl_xor_sync(kFullMask, kb, stride);
            const bool take_max = ((lane & stride) == 0) == ((lane & size) == 0);
            ka = take_max ? max(ka, oa) : min(ka, oa);
            kb = take_max ? max(kb, ob) : min(kb, ob);
        }
    }
    if (lane < na) sa[lane] = cand_key(__uint_as_float((ta << 17) | (ka >> 15)), 0x7FFF - (int)(ka & 0x7FFFu));
    if (lane < nb) sb[lane] = cand_key(__uint_as_float((tb << 17) | (kb >> 15)), 0x7FFF - (int)(kb & 0x7FFFu));
}



}  // namespace
}  // namespace b2s
