// exact_math.cuh -- scalar building blocks shared by the device kernels and
// the host-side model used by the CPU tests.
//
// Two problems make the llama2.c sampler hard to reproduce on a GPU:
//
//  1. Its softmax calls glibc expf (llama2.c:588-606).  glibc's expf returns
//     the correctly rounded result for all but ~0.01% of inputs, so the device
//     exponential below is built to be correctly rounded except in rare
//     near-midpoint cases: Tang's table-driven method (P. T. P. Tang, "Table-
//     driven implementation of the exponential function in IEEE floating-point
//     arithmetic", ACM TOMS 15(2), 1989) in fp32 with a 128-entry 2^(j/N)
//     table held as hi/lo fp32 pairs (built from double-precision exp2).
//
//  2. It sums in a strict serial fp32 order (softmax denominator
//     llama2.c:598-601, sample_mult llama2.c:996-1002, sample_topp
//     llama2.c:1036-1054).  A tree or fp64 sum differs from that chain by up
//     to ~3e-4 relative on 32000-term rows.  The "binade chain" functions
//     below reproduce the serial chain exactly in parallel: while a running
//     sum s stays inside one binade [2^E, 2^(E+1)), every rounding of s + a
//     happens on the fixed grid u = 2^(E-23) and depends on s only through
//     the parity of s/u (round-half-to-even).  So a contiguous chunk of
//     addends acts on s as  s -> s + L[parity(s)]  with a parity map, and
//     those chunk functions compose associatively.  Chunks whose running sum
//     may leave the binade are replayed with real fp32 adds.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define XM_HD __host__ __device__ __forceinline__
#else
#define XM_HD inline
#endif

#if defined(__CUDA_ARCH__)
#define XM_FMA(a, b, c) __fmaf_rn((a), (b), (c))
#define XM_ADD(a, b) __fadd_rn((a), (b))
#define XM_SUB(a, b) __fsub_rn((a), (b))
#define XM_MUL(a, b) __fmul_rn((a), (b))
#define XM_F2U(x) __float_as_uint(x)
#define XM_U2F(x) __uint_as_float(x)
#else
#include <math.h>
#include <string.h>
static inline uint32_t xm_f2u_host(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float xm_u2f_host(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
#define XM_FMA(a, b, c) fmaf((a), (b), (c))
#define XM_ADD(a, b) ((a) + (b))
#define XM_SUB(a, b) ((a) - (b))
#define XM_MUL(a, b) ((a) * (b))
#define XM_F2U(x) xm_f2u_host(x)
#define XM_U2F(x) xm_u2f_host(x)
#endif

namespace xm {

// ---------------------------------------------------------------------------
// Table-driven exp
// ---------------------------------------------------------------------------
constexpr int kExpTableBits = 7;
constexpr int kExpTableSize = 1 << kExpTableBits;  // N = 128 entries of 2^(j/N)

// N/ln2 and the two-part split of ln2/N (C1 = RN(ln2/N), C2 = RN(ln2/N - C1)),
// written as exact hex-float literals computed from ln2 in double precision.
constexpr float kInvLn2N = 0x1.715476p+7f;       // 128/ln2
constexpr float kLn2N_hi = 0x1.62e430p-8f;       // RN(ln2/128)
constexpr float kLn2N_lo = -0x1.05c610p-36f;     // RN(ln2/128 - hi)
constexpr float kShifter = 0x1.8p+23f;           // 1.5*2^23: rounds to integer

struct ExpTableEntry {
    float hi, lo;  // 2^(j/N) = hi + lo, |lo| <= ulp(hi)/2
};

// exp(d) on [kExpFastMin, kExpFastMax] (exp_f32 below covers the rest).
// exp(d) = 2^k * 2^(j/N) * exp(r) with n = k*N + j = round(d*N/ln2) and
// r = d - n*ln2/N, |r| <= ln2/(2N).  r is formed with a two-constant
// Cody-Waite reduction whose first FMA is exact; exp(r) - 1 is the cubic
// Taylor polynomial (the r^4 term is below 2^-38); the table value enters as
// hi + lo.  Measured over every float in [-87, 0]: the result equals the
// correctly rounded exp except within ~1e-2 ulp of a rounding midpoint, and
// differs from glibc expf on 0.016% of inputs, never by more than 1 ulp.
XM_HD float exp_normal_range(float d, const ExpTableEntry* tab) {
    const float t = XM_FMA(d, kInvLn2N, kShifter);
    const float nf = XM_SUB(t, kShifter);
    const int n = (int)(XM_F2U(t) - XM_F2U(kShifter));  // exact integer n = round(d*N/ln2)
    const int j = n & (kExpTableSize - 1);
    const int k = n >> kExpTableBits;                     // arithmetic shift: floor(n/N)
    const float r1 = XM_FMA(-nf, kLn2N_hi, d);            // exact
    const float r = XM_FMA(-nf, kLn2N_lo, r1);
    const ExpTableEntry T = tab[j];
    const float a = XM_FMA(r, 0x1.555556p-3f, 0.5f);      // 1/2 + r/6
    const float p = XM_FMA(XM_MUL(r, r), a, r);           // exp(r) - 1
    const float y = XM_ADD(XM_FMA(T.hi, p, T.lo), T.hi);
    // scale by 2^k through the exponent field (the result is normal here)
    return XM_U2F(XM_F2U(y) + ((uint32_t)k << 23));
}

// exp_normal_range is used on [kExpFastMin, kExpFastMax]; there the result
// is a normal float and the exponent-field scaling is exact.  Outside it
// (subnormal/zero/overflow results, NaN) the value comes from double
// precision exp rounded once to fp32.
constexpr float kExpFastMin = -87.0f;  // ln(2^-126) = -87.3365...
constexpr float kExpFastMax = 88.0f;   // ln(FLT_MAX) = 88.7228...

// The rare out-of-range path, kept out of line so the unrolled callers do
// not carry its register footprint.
#if defined(__CUDACC__)
static __host__ __device__ __noinline__
#else
static inline
#endif
float exp_outside_fast_range(float d) {
    return (float)exp((double)d);
}

XM_HD float exp_f32(float d, const ExpTableEntry* tab) {
    if (d >= kExpFastMin && d <= kExpFastMax) return exp_normal_range(d, tab);
    return exp_outside_fast_range(d);
}

// The 2^(j/N) table entry j as an fp32 hi/lo pair, from double-precision exp2.
XM_HD ExpTableEntry exp_table_entry(int j) {
    const double t = exp2((double)j / (double)kExpTableSize);
    const float hi = (float)t;
    const float lo = (float)(t - (double)hi);
    return ExpTableEntry{hi, lo};
}

// ---------------------------------------------------------------------------
// Binade chain: exact emulation of a serial fp32 sum of non-negative addends
// ---------------------------------------------------------------------------

// Chunk function: s -> s + L[par(s)], par(s) -> pout[par(s)], valid while s
// stays in one binade.  pbits packs pout[0] in bit 0 and pout[1] in bit 1.
struct ChainFn {
    float L0, L1;
    uint32_t pbits;
};

XM_HD ChainFn chain_identity() { return ChainFn{0.0f, 0.0f, 2u}; }

// a then b (apply a first).  All L values are multiples of the binade grid u
// and the sums stay below 2^(E+1), so the fp32 additions are exact.
XM_HD ChainFn chain_compose(const ChainFn& a, const ChainFn& b) {
    const uint32_t q0 = a.pbits & 1u, q1 = (a.pbits >> 1) & 1u;
    ChainFn c;
    c.L0 = XM_ADD(a.L0, q0 ? b.L1 : b.L0);
    c.L1 = XM_ADD(a.L1, q1 ? b.L1 : b.L0);
    const uint32_t o0 = (b.pbits >> q0) & 1u;
    const uint32_t o1 = (b.pbits >> q1) & 1u;
    c.pbits = o0 | (o1 << 1);
    return c;
}

// Binade exponent field of a positive normal float (biased, 1..254).
XM_HD uint32_t binade_of(float s) { return (XM_F2U(s) >> 23) & 0xFFu; }

// Smallest biased exponent for which the chunk-function fast path is used.
// Below it (running sums < 2^-100) chunks are always replayed serially.
constexpr uint32_t kMinFastBinade = 27u;

// Applies chunk function f (built for binade `eb`) to an exact running sum s.
// Returns false (leaving s unchanged) if s is not in that binade or the
// result would leave it; the caller then replays the chunk serially.
XM_HD bool chain_apply(float& s, uint32_t eb, const ChainFn& f) {
    const uint32_t sb = XM_F2U(s);
    if (((sb >> 23) & 0xFFu) != eb || eb < kMinFastBinade || eb >= 254u) return false;
    const uint32_t par = sb & 1u;
    const float L = par ? f.L1 : f.L0;
    const float hi = XM_U2F((eb + 1u) << 23);
    if (!(L <= XM_SUB(hi, s))) return false;  // hi - s is exact (Sterbenz)
    s = XM_ADD(s, L);                         // exact: stays on the grid
    return true;
}

// Virtual chains of one chunk under the binade with biased exponent eb: run
// the real fp32 adds from the two grid points 2^E (even) and 2^E + u (odd).
// Returns false if either chain leaves the binade (the chunk is then treated
// as unclean).  a[] holds the chunk's addends in order.
template <int N>
XM_HD bool chain_build(const float (&a)[N], uint32_t eb, ChainFn& f) {
    const float v0s = XM_U2F(eb << 23);
    const float v1s = XM_U2F((eb << 23) | 1u);
    float v0 = v0s, v1 = v1s;
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
    for (int i = 0; i < N; ++i) {
        v0 = XM_ADD(v0, a[i]);
        v1 = XM_ADD(v1, a[i]);
    }
    const uint32_t b0 = XM_F2U(v0), b1 = XM_F2U(v1);
    if ((b0 >> 23) != eb || (b1 >> 23) != eb) return false;
    f.L0 = XM_SUB(v0, v0s);
    f.L1 = XM_SUB(v1, v1s);
    f.pbits = (b0 & 1u) | ((b1 & 1u) << 1);
    return true;
}

// Decides which binade a chunk's running sum will sit in from an approximate
// incoming value g and the chunk's approximate total sigma.  Returns the
// biased exponent, or 0 when the chunk may straddle a binade boundary (or
// the sums are too small), in which case it is replayed serially.
XM_HD uint32_t chain_guess_binade(float g, float sigma) {
    const uint32_t eb = binade_of(g);
    if (!(g > 0.0f) || eb < kMinFastBinade || eb >= 253u) return 0u;
    const float lo = XM_U2F(eb << 23);
    const float hi = XM_U2F((eb + 1u) << 23);
    // 2^-10 relative margins absorb the gap between the approximate prefix
    // and the exact serial sum (observed < 3e-4 on softmax rows).  A wrong
    // guess costs speed only: chain_apply rejects it and the chunk replays.
    if (!(g >= XM_MUL(lo, 1.0009765625f))) return 0u;
    if (!(XM_ADD(g, sigma) <= XM_MUL(hi, 0.9990234375f))) return 0u;
    return eb;
}


// Binade the running sum of a chunk is expected to sit in, from an
// approximate incoming value g: binade(g), or 0 when g is zero or below
// 2^-100 (such chunks are replayed).  `alt` receives the neighbouring binade
// the exact serial sum may fall into instead -- when g, or the chunk's end
// g + sigma, lies within 2^-10 of a binade boundary -- or 0.  The caller
// builds chunk functions for both, and the resolution picks whichever
// matches the exact running sum.
XM_HD uint32_t chain_guess_primary(float g, float sigma, uint32_t& alt) {
    alt = 0u;
    const uint32_t eb = binade_of(g);
    if (!(g > 0.0f) || eb < kMinFastBinade || eb >= 253u) return 0u;
    const float lo = XM_U2F(eb << 23);
    const float hi = XM_U2F((eb + 1u) << 23);
    if (!(g >= XM_MUL(lo, 1.0009765625f))) {
        if (eb - 1u >= kMinFastBinade) alt = eb - 1u;
    } else if (!(XM_ADD(g, sigma) <= XM_MUL(hi, 0.9990234375f))) {
        alt = eb + 1u;
    }
    return eb;
}

}  // namespace xm
