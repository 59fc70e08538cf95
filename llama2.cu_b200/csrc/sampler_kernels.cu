// sampler_kernels.cu -- sm_100a kernels of the logits -> token path.
//
// Per-row semantics follow llama2.c sample() (llama2.c:1082-1105) exactly:
//   temperature == 0  -> sample_argmax on the raw logits        (llama2.c:981-992)
//   else              -> logits /= T, softmax                   (llama2.c:588-606)
//                        coin = random_f32(state)               (llama2.c:1071-1080)
//                        topp <= 0 || topp >= 1 -> sample_mult  (llama2.c:994-1005)
//                        else                   -> sample_topp  (llama2.c:1015-1056)
//
// Row kernel (one persistent 1024-thread CTA per SM, one row at a time):
//   1. the row (<= 32768 fp32) is staged into shared memory by bulk-async
//      copies (cp.async.bulk, mbarrier completion) -- HBM is read once;
//   2. max/min pass (warp shuffles), then x = l/T, e = exp(x - max) with the
//      table-driven exponential, written back in a chunk-swizzled layout
//      (thread t owns 32 consecutive elements; 16-byte granules are XOR
//      swizzled so both passes are bank-conflict free);
//   3. the softmax denominator is the EXACT serial fp32 sum, computed in
//      parallel by the binade-chain engine (exact_math.cuh);
//   4. sample_mult: p = e/S in place, the same engine gives the exact serial
//      cdf and the first index with coin < cdf;
//      sample_topp: p >= cutoff candidates are binned by the top bits of p
//      (64 bins per binade); the smallest prefix of bins whose guaranteed mass
//      exceeds topp plus the worst-case fp32 drift is scattered in bin order,
//      each bin is sorted (p desc, index asc == glibc qsort's order for this
//      index-ordered input), and the engine replays the serial cumulative sum
//      and the r = coin*cum walk over that sorted nucleus only.
//   Nuclei beyond the on-chip capacity take a global-memory path (sort in the
//   per-CTA workspace, engine over 8192-element pieces).
#include "device_common.cuh"
#include "exact_math.cuh"
#include "sampler_kernels.cuh"

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace b2s {
namespace {

constexpr int kWarps = kRowThreads / 32;
constexpr int kSegSortMax = 256;
constexpr int kMaxBigSegs = 64;
constexpr int kTmaParts = 4;
constexpr int kMaxPieces = 8;

struct __align__(16) RowSmem {
    float row[kRowCap];                     // staged logits / e / p (swizzled chunks)
    unsigned long long cand[kCandCap];      // nucleus keys (p bits << 32 | ~index)
    union {
        float4 chunk_fn[kRowThreads];       // chain engine: per-chunk function + binade
        struct {
            int hist[kBins];
            int cursor[kBins];
        } bins;
    } u;
    float chunk_s[kRowThreads + 4];         // exact running sum entering each chunk
    float4 warp_fn[kWarps];
    float warp_state[kWarps];
    xm::ExpTableEntry exptab[xm::kExpTableSize];
    float red_f[kWarps];
    float red_f2[kWarps];
    int red_i[kWarps];
    unsigned long long mbar[2];
    float piece_state[kMaxPieces + 1];
    int big_start[kMaxBigSegs];
    int big_len[kMaxBigSegs];
    int n_big;
    int found_idx;
    float found_val;
    int n0;
    int ksel;
    int dbin;
    int result;
};

// ---------------------------------------------------------------------------
// small helpers
// ---------------------------------------------------------------------------
// Physical float4 granule of logical granule g of chunk t, for chunks of
// CPT floats (G = CPT/4 granules).  The XOR keeps the 8 threads of a
// quarter-warp on distinct 16-byte bank groups when each reads its own chunk.
template <int CPT>
__device__ __forceinline__ int gran_phys(int t, int g) {
    constexpr int G = CPT / 4;
    static_assert(G == 2 || G == 4 || G == 8, "chunk size");
    constexpr int S = (G == 8) ? 0 : (G == 4) ? 1 : 2;
    return t * G + (g ^ ((t >> S) & (G - 1)));
}

// Physical granule of natural granule gi (= element 4*gi .. 4*gi+3).
template <int CPT>
__device__ __forceinline__ int gran_phys_nat(int gi) {
    constexpr int G = CPT / 4;
    return gran_phys<CPT>(gi / G, gi % G);
}

template <int CPT>
__device__ __forceinline__ int elem_phys(int i) {
    return gran_phys_nat<CPT>(i >> 2) * 4 + (i & 3);
}

__device__ __forceinline__ float4 ld4(const float* base, int gran) {
    return reinterpret_cast<const float4*>(base)[gran];
}
__device__ __forceinline__ void st4(float* base, int gran, float4 v) {
    reinterpret_cast<float4*>(base)[gran] = v;
}

__device__ __forceinline__ float4 pack_fn(const xm::ChainFn& f, bool ok, uint32_t eb) {
    return make_float4(f.L0, f.L1, __uint_as_float(f.pbits | (ok ? 4u : 0u)), __uint_as_float(eb));
}

// Exclusive block scan of a float (approximate: only used as a guess).
__device__ float block_excl_scan(float v, RowSmem& sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(kFullMask, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sm.red_f[warp] = x;
    __syncthreads();
    if (warp == 0) {
        float w = sm.red_f[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(kFullMask, w, o);
            if (lane >= o) w += y;
        }
        float ex = __shfl_up_sync(kFullMask, w, 1);
        if (lane == 0) ex = 0.0f;
        sm.red_f2[lane] = ex;
    }
    __syncthreads();
    float within = __shfl_up_sync(kFullMask, x, 1);
    if (lane == 0) within = 0.0f;
    return sm.red_f2[warp] + within;
}

// ---------------------------------------------------------------------------
// Exact serial-sum engine over `nch` chunks of CPT floats stored swizzled in
// sm.row.  After return: sm.chunk_s[t] = exact serial running sum before the
// first element of chunk t (t <= nch; chunk_s[nch] is the total), starting
// from s_init.  All addends must be non-negative (NaN-free).
// ---------------------------------------------------------------------------
template <int CPT>
__device__ float chunk_replay(const RowSmem& sm, int t, float s) {
    constexpr int G = CPT / 4;
    float4 q[G];
#pragma unroll
    for (int g = 0; g < G; ++g) q[g] = ld4(sm.row, gran_phys<CPT>(t, g));
#pragma unroll
    for (int g = 0; g < G; ++g) {
        s = __fadd_rn(s, q[g].x);
        s = __fadd_rn(s, q[g].y);
        s = __fadd_rn(s, q[g].z);
        s = __fadd_rn(s, q[g].w);
    }
    return s;
}

template <int CPT>
__device__ void chain_run(RowSmem& sm, int nch, float s_init) {
    constexpr int G = CPT / 4;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const bool valid = t < nch;
    float v[CPT];
    if (valid) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float4 q = ld4(sm.row, gran_phys<CPT>(t, g));
            v[4 * g + 0] = q.x;
            v[4 * g + 1] = q.y;
            v[4 * g + 2] = q.z;
            v[4 * g + 3] = q.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < CPT; ++j) v[j] = 0.0f;
    }
    float sig = 0.0f;
#pragma unroll
    for (int j = 0; j < CPT; ++j) sig += v[j];
    const float guess = block_excl_scan(sig, sm) + s_init;

    uint32_t eb = xm::chain_guess_binade(guess, sig);
    xm::ChainFn f = xm::chain_identity();
    bool clean = false;
    if (valid && eb != 0u) clean = xm::chain_build(v, eb, f);
    if (valid) sm.u.chunk_fn[t] = pack_fn(f, clean, eb);

    // Warp-level composition when all chunks of the warp share one binade.
    const bool warp_live = warp * 32 < nch;
    const uint32_t eb0 = __shfl_sync(kFullMask, eb, 0);
    const bool uniform = __all_sync(kFullMask, !valid || (clean && eb == eb0)) && warp_live;
    xm::ChainFn inc = valid ? f : xm::chain_identity();
    xm::ChainFn excl = xm::chain_identity();
    if (uniform) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            xm::ChainFn y;
            y.L0 = __shfl_up_sync(kFullMask, inc.L0, o);
            y.L1 = __shfl_up_sync(kFullMask, inc.L1, o);
            y.pbits = __shfl_up_sync(kFullMask, inc.pbits, o);
            if (lane >= o) inc = xm::chain_compose(y, inc);
        }
        excl.L0 = __shfl_up_sync(kFullMask, inc.L0, 1);
        excl.L1 = __shfl_up_sync(kFullMask, inc.L1, 1);
        excl.pbits = __shfl_up_sync(kFullMask, inc.pbits, 1);
        if (lane == 0) excl = xm::chain_identity();
    }
    if (lane == 31 && warp_live) sm.warp_fn[warp] = pack_fn(inc, uniform, eb0);
    __syncthreads();

    // Sequential resolution across warps (warp 0; every lane computes the
    // same values, lane 0 stores).
    if (warp == 0) {
        float s = s_init;
        const int nw = (nch + 31) >> 5;
        for (int w = 0; w < nw; ++w) {
            const float4 wi = sm.warp_fn[w];
            const uint32_t wb = __float_as_uint(wi.z);
            if (wb & 4u) {
                float s2 = s;
                if (xm::chain_apply(s2, __float_as_uint(wi.w), xm::ChainFn{wi.x, wi.y, wb & 3u})) {
                    if (lane == 0) sm.warp_state[w] = s;
                    s = s2;
                    continue;
                }
            }
            if (lane == 0) sm.warp_state[w] = __uint_as_float(0x7FC00000u);  // resolved per chunk
            const int tend = min(nch, (w + 1) * 32);
            for (int tt = w * 32; tt < tend; ++tt) {
                if (lane == 0) sm.chunk_s[tt] = s;
                const float4 ci = sm.u.chunk_fn[tt];
                const uint32_t cb = __float_as_uint(ci.z);
                float s2 = s;
                if ((cb & 4u) &&
                    xm::chain_apply(s2, __float_as_uint(ci.w), xm::ChainFn{ci.x, ci.y, cb & 3u}))
                    s = s2;
                else
                    s = chunk_replay<CPT>(sm, tt, s);
            }
        }
        if (lane == 0) sm.chunk_s[nch] = s;
    }
    __syncthreads();
    if (valid) {
        const float ws = sm.warp_state[warp];
        if (!isnan(ws)) {
            const uint32_t par = __float_as_uint(ws) & 1u;
            sm.chunk_s[t] = __fadd_rn(ws, par ? excl.L1 : excl.L0);
        }
    }
    __syncthreads();
}

// First element (index < nch*CPT) whose exact running sum exceeds theta,
// using the chunk states of the last chain_run.  Result in sm.found_idx
// (-1 if none) and sm.found_val.
template <int CPT>
__device__ void chain_find(RowSmem& sm, int nch, float theta) {
    const int t = threadIdx.x;
    if (t == 0) sm.found_idx = -1;
    __syncthreads();
    if (t < nch) {
        const float s_in = sm.chunk_s[t];
        const float s_out = sm.chunk_s[t + 1];
        if (!(s_in > theta) && (s_out > theta)) {
            constexpr int G = CPT / 4;
            float s = s_in;
            int found = -1;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float4 q = ld4(sm.row, gran_phys<CPT>(t, g));
                const float a[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    s = __fadd_rn(s, a[w]);
                    if (found < 0 && s > theta) {
                        found = t * CPT + 4 * g + w;
                        sm.found_val = s;
                    }
                }
            }
            sm.found_idx = found;
        }
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// Sorting of 64-bit keys, descending
// ---------------------------------------------------------------------------
// Writes p values of sorted keys [first, first+count) from `src` into sm.row
// in the CPT=8 chunk layout (zero padded to whole chunks); returns #chunks.
__device__ int stage_sorted_probs(RowSmem& sm, const unsigned long long* src, int count) {
    const int nch = (count + 7) >> 3;
    for (int i = threadIdx.x; i < nch * 8; i += blockDim.x) {
        const float pv = (i < count) ? key_prob(src[i]) : 0.0f;
        sm.row[elem_phys<8>(i)] = pv;
    }
    __syncthreads();
    return nch;
}

// ---------------------------------------------------------------------------
// top-p pieces
// ---------------------------------------------------------------------------

// Global-memory path: every candidate (p >= cutoff) is sorted in the CTA's
// workspace and the nucleus walk runs over 8192-element pieces.  Returns the
// token id (-1 when there are no candidates).
__device__ int topp_global_path(RowSmem& sm, int V, float cutoff, float topp, float coin,
                                unsigned long long* ws) {
    const int tid = threadIdx.x;
    if (tid == 0) sm.n0 = 0;
    __syncthreads();
    const int ngran = (V + 3) >> 2;
    for (int gi = tid; gi < ngran; gi += blockDim.x) {
        const float4 q = ld4(sm.row, gran_phys_nat<kRowCPT>(gi));
        const float a[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const int i = 4 * gi + w;
            if (i < V && a[w] >= cutoff) {
                const int pos = atomicAdd(&sm.n0, 1);
                ws[pos] = cand_key(a[w], i);
            }
        }
    }
    __syncthreads();
    const int n0 = sm.n0;
    if (n0 == 0) return -1;
    int P = 1;
    while (P < n0) P <<= 1;
    for (int i = n0 + tid; i < P; i += blockDim.x) ws[i] = 0ull;
    __syncthreads();
    block_bitonic_desc(ws, P);

    const int npieces = (n0 + kCandCap - 1) / kCandCap;
    float carry = 0.0f;
    int last = -1, last_piece = npieces - 1;
    float cum = 0.0f;
    for (int q = 0; q < npieces; ++q) {
        const int first = q * kCandCap;
        const int cnt = min(kCandCap, n0 - first);
        if (tid == 0) sm.piece_state[q] = carry;
        const int nch = stage_sorted_probs(sm, ws + first, cnt);
        chain_run<8>(sm, nch, carry);
        chain_find<8>(sm, nch, topp);
        if (sm.found_idx >= 0 && sm.found_idx < cnt) {
            last = first + sm.found_idx;
            cum = sm.found_val;
            last_piece = q;
            break;
        }
        carry = sm.chunk_s[nch];
        __syncthreads();
    }
    if (last < 0) {  // llama2.c:1037: last_idx = n0 - 1 when the sum never exceeds topp
        last = n0 - 1;
        cum = carry;
        last_piece = npieces - 1;
    }
    const float r = __fmul_rn(coin, cum);
    __syncthreads();
    for (int q = 0; q <= last_piece; ++q) {
        const float end = (q < last_piece) ? sm.piece_state[q + 1] : cum;
        if (r < end) {
            const int first = q * kCandCap;
            const int cnt = (q == last_piece) ? (last - first + 1) : kCandCap;
            const int nch = stage_sorted_probs(sm, ws + first, cnt);
            chain_run<8>(sm, nch, sm.piece_state[q]);
            chain_find<8>(sm, nch, r);
            const int fi = sm.found_idx;
            if (fi >= 0 && fi < cnt) return key_index(ws[first + fi]);
            break;
        }
    }
    return key_index(ws[last]);  // llama2.c:1055 fallback
}

// ---------------------------------------------------------------------------
// The row kernel
// ---------------------------------------------------------------------------
struct RowCtx {
    int V;
    int nch;
    float T;
    float topp;
    float coin;
    bool probs_in;
    bool write_probs;
    float* probs_row;
};

// Greedy row: first index of the strict max over the raw logits with the
// reference's NaN behaviour (a NaN at index 0 wins; other NaNs never do).
__device__ int row_argmax(RowSmem& sm, int V) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    for (int i = tid; i < V; i += blockDim.x) {
        const float x = sm.row[i];
        if (x > bv || (x == bv && i < bi)) {
            bv = x;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(kFullMask, bv, o);
        const int oi = __shfl_xor_sync(kFullMask, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if (lane == 0) {
        sm.red_f[warp] = bv;
        sm.red_i[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        bv = sm.red_f[lane];
        bi = sm.red_i[lane];
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(kFullMask, bv, o);
            const int oi = __shfl_xor_sync(kFullMask, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) sm.result = (bi == 0x7FFFFFFF || isnan(sm.row[0])) ? 0 : bi;
    }
    __syncthreads();
    return sm.result;
}

// Block max and min (NaN ignored) of the staged logits.
__device__ void row_minmax(RowSmem& sm, int V, float& mx, float& mn) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float a = -INFINITY, b = INFINITY;
    for (int i = tid; i < V; i += blockDim.x) {
        const float x = sm.row[i];
        a = fmaxf(a, x);
        b = fminf(b, x);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        a = fmaxf(a, __shfl_xor_sync(kFullMask, a, o));
        b = fminf(b, __shfl_xor_sync(kFullMask, b, o));
    }
    if (lane == 0) {
        sm.red_f[warp] = a;
        sm.red_f2[warp] = b;
    }
    __syncthreads();
    a = sm.red_f[lane];
    b = sm.red_f2[lane];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        a = fmaxf(a, __shfl_xor_sync(kFullMask, a, o));
        b = fminf(b, __shfl_xor_sync(kFullMask, b, o));
    }
    mx = a;
    mn = b;
    __syncthreads();
}

// x = l/T, e = exp(x - max): natural layout in, swizzled layout out.
// Returns true if any e is NaN (the reference's softmax then yields NaN).
__device__ bool row_exp_pass(RowSmem& sm, const RowCtx& c, float max_x) {
    const int tid = threadIdx.x;
    const int ngran_used = c.nch * (kRowCPT / 4);
    const bool unit_t = (c.T == 1.0f);
    bool any_nan = false;
    // Trip counts are uniform across the block so the __syncwarp below (read
    // before any lane overwrites a granule of its chunk) sees full warps.
    for (int base = 0; base < ngran_used; base += blockDim.x) {
        const int gi = base + tid;
        const bool act = gi < ngran_used;
        float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (act) {
            const float4 q = ld4(sm.row, gi);
            a[0] = q.x;
            a[1] = q.y;
            a[2] = q.z;
            a[3] = q.w;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const int i = 4 * gi + w;
                if (i < c.V) {
                    const float x = unit_t ? a[w] : __fdiv_rn(a[w], c.T);
                    const float e = xm::exp_f32(__fsub_rn(x, max_x), sm.exptab);
                    any_nan |= isnan(e);
                    a[w] = e;
                } else {
                    a[w] = 0.0f;
                }
            }
        }
        __syncwarp();
        if (act) st4(sm.row, gran_phys_nat<kRowCPT>(gi), make_float4(a[0], a[1], a[2], a[3]));
    }
    return __syncthreads_or(any_nan) != 0;
}

// Probabilities given: natural -> swizzled in place; flags non-monotone input.
__device__ bool row_permute_pass(RowSmem& sm, const RowCtx& c) {
    const int tid = threadIdx.x;
    const int ngran_used = c.nch * (kRowCPT / 4);
    bool bad = false;
    for (int base = 0; base < ngran_used; base += blockDim.x) {
        const int gi = base + tid;
        const bool act = gi < ngran_used;
        float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (act) {
            const float4 q = ld4(sm.row, gi);
            a[0] = q.x;
            a[1] = q.y;
            a[2] = q.z;
            a[3] = q.w;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const int i = 4 * gi + w;
                if (i >= c.V) a[w] = 0.0f;
                bad |= (a[w] < 0.0f) || isnan(a[w]);
            }
        }
        __syncwarp();
        if (act) st4(sm.row, gran_phys_nat<kRowCPT>(gi), make_float4(a[0], a[1], a[2], a[3]));
    }
    return __syncthreads_or(bad) != 0;
}

// p = e / S in place (and to probs_row when requested), natural order walk.
__device__ void row_div_pass(RowSmem& sm, const RowCtx& c, float S) {
    for (int gi = threadIdx.x; gi * 4 < c.V; gi += blockDim.x) {
        const int pg = gran_phys_nat<kRowCPT>(gi);
        const float4 q = ld4(sm.row, pg);
        float a[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int w = 0; w < 4; ++w) a[w] = (4 * gi + w < c.V) ? __fdiv_rn(a[w], S) : 0.0f;
        st4(sm.row, pg, make_float4(a[0], a[1], a[2], a[3]));
        if (c.write_probs) {
#pragma unroll
            for (int w = 0; w < 4; ++w)
                if (4 * gi + w < c.V) c.probs_row[4 * gi + w] = a[w];
        }
    }
    __syncthreads();
}

// Reference serial walk for inputs the engine cannot take (negative or NaN
// probabilities): sample_mult exactly as llama2.c:994-1005.
__device__ int row_serial_mult(RowSmem& sm, const RowCtx& c) {
    if (threadIdx.x == 0) {
        float cdf = 0.0f;
        int id = c.V - 1;
        for (int i = 0; i < c.V; ++i) {
            cdf += sm.row[elem_phys<kRowCPT>(i)];
            if (c.coin < cdf) {
                id = i;
                break;
            }
        }
        sm.result = id;
    }
    __syncthreads();
    return sm.result;
}

// sample_topp over the staged row (e values when !probs_in, else p values).
__device__ int row_topp(RowSmem& sm, const RowCtx& c, float S, unsigned long long* ws, int& flags) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float cutoff = __fdiv_rn(__fsub_rn(1.0f, c.topp), (float)(c.V - 1));  // llama2.c:1024
    // e-space prefilter: fl(e/S) >= cutoff implies e >= cutoff*S*(1 - 2^-20).
    const float e_min = c.probs_in ? cutoff : __fmul_rn(__fmul_rn(cutoff, S), 0.99999905f);

    for (int b = tid; b < kBins; b += blockDim.x) sm.u.bins.hist[b] = 0;
    if (tid == 0) sm.n0 = 0;
    __syncthreads();

    // T1: p for candidates (for every element when probabilities are written
    // back), histogram of candidates by the top bits of p.
    int my_n0 = 0;
    for (int gi = tid; gi * 4 < c.V; gi += blockDim.x) {
        const int pg = gran_phys_nat<kRowCPT>(gi);
        const float4 q = ld4(sm.row, pg);
        float a[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const int i = 4 * gi + w;
            float pv = 0.0f;
            if (i < c.V) {
                if (c.probs_in) {
                    pv = a[w];
                } else if (c.write_probs || a[w] >= e_min) {
                    pv = __fdiv_rn(a[w], S);
                    if (c.write_probs) c.probs_row[i] = pv;
                }
                if (pv >= cutoff) {
                    atomicAdd(&sm.u.bins.hist[bin_of(pv)], 1);
                    ++my_n0;
                } else if (!c.probs_in) {
                    pv = 0.0f;
                }
            }
            a[w] = pv;
        }
        if (!c.probs_in) st4(sm.row, pg, make_float4(a[0], a[1], a[2], a[3]));
    }
    if (my_n0) atomicAdd(&sm.n0, my_n0);
    __syncthreads();
    const int n0 = sm.n0;
    if (n0 == 0) {
        flags |= kFlagNoCand;
        return 0;
    }

    // T2: smallest prefix of bins whose guaranteed mass exceeds topp plus the
    // worst-case drift of an fp32 serial sum over kCandCap terms.
    if (warp == 0) {
        constexpr int per = kBins / 32;
        int cnt = 0;
        float mass = 0.0f;
        for (int b = lane * per; b < lane * per + per; ++b) {
            const int h = sm.u.bins.hist[b];
            cnt += h;
            mass += (float)h * bin_lo(b);
        }
        int ci = cnt;
        float mi = mass;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int yc = __shfl_up_sync(kFullMask, ci, o);
            const float ym = __shfl_up_sync(kFullMask, mi, o);
            if (lane >= o) {
                ci += yc;
                mi += ym;
            }
        }
        int cex = __shfl_up_sync(kFullMask, ci, 1);
        float mex = __shfl_up_sync(kFullMask, mi, 1);
        if (lane == 0) {
            cex = 0;
            mex = 0.0f;
        }
        const float target = __fadd_rn(c.topp, (float)kCandCap * 0x1p-24f + 1e-5f);
        const unsigned hit = __ballot_sync(kFullMask, mi >= target);
        int D = kBins - 1;
        if (hit) {
            const int L = __ffs(hit) - 1;
            if (lane == L) {
                int cc = cex;
                float mm = mex;
                int d = lane * per + per - 1;
                for (int b = lane * per; b < lane * per + per; ++b) {
                    const int h = sm.u.bins.hist[b];
                    cc += h;
                    mm += (float)h * bin_lo(b);
                    if (mm >= target) {
                        d = b;
                        break;
                    }
                }
                sm.dbin = d;
            }
            __syncwarp();
            D = sm.dbin;
        }
        // exclusive offsets of bins 0..D
        int run = cex;
        for (int b = lane * per; b < lane * per + per; ++b) {
            if (b > D) break;
            sm.u.bins.cursor[b] = run;
            run += sm.u.bins.hist[b];
        }
        // ksel = count in bins 0..D
        const int lane_of_D = D / per;
        const int upto = (lane == lane_of_D) ? run : 0;
        const int ksel = __reduce_add_sync(kFullMask, upto);
        if (lane == 0) {
            sm.dbin = D;
            sm.ksel = ksel;
        }
    }
    __syncthreads();
    const int D = sm.dbin;
    const int ksel = sm.ksel;

    if (ksel > kCandCap) {
        flags |= kFlagSlow;
        const int id = topp_global_path(sm, c.V, cutoff, c.topp, c.coin, ws);
        if (id < 0) {
            flags |= kFlagNoCand;
            return 0;
        }
        return id;
    }

    // T3: scatter candidates of bins 0..D in bin order.
    for (int gi = tid; gi * 4 < c.V; gi += blockDim.x) {
        const float4 q = ld4(sm.row, gran_phys_nat<kRowCPT>(gi));
        const float a[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const int i = 4 * gi + w;
            if (i < c.V && a[w] >= cutoff) {
                const int b = bin_of(a[w]);
                if (b <= D) {
                    const int pos = atomicAdd(&sm.u.bins.cursor[b], 1);
                    sm.cand[pos] = cand_key(a[w], i);
                }
            }
        }
    }
    if (tid == 0) sm.n_big = 0;
    __syncthreads();

    // T4: sort each bin's segment (cursor[b] now holds the segment end).
    for (int b = warp; b <= D; b += kWarps) {
        const int n = sm.u.bins.hist[b];
        if (n <= 1) continue;
        unsigned long long* seg = sm.cand + (sm.u.bins.cursor[b] - n);
        if (n <= 32) {
            warp_sort_desc<1>(seg, n, lane);
        } else if (n <= 64) {
            warp_sort_desc<2>(seg, n, lane);
        } else if (n <= 128) {
            warp_sort_desc<4>(seg, n, lane);
        } else if (n <= kSegSortMax) {
            warp_sort_desc<8>(seg, n, lane);
        } else if (lane == 0) {
            const int k = atomicAdd(&sm.n_big, 1);
            if (k < kMaxBigSegs) {
                sm.big_start[k] = sm.u.bins.cursor[b] - n;
                sm.big_len[k] = n;
            }
        }
    }
    __syncthreads();
    const int nbig = sm.n_big;
    if (nbig > kMaxBigSegs) {  // too fragmented: one block sort of everything
        unsigned long long* scratch = reinterpret_cast<unsigned long long*>(sm.row);
        int P = 1;
        while (P < ksel) P <<= 1;
        for (int i = tid; i < P; i += blockDim.x) scratch[i] = (i < ksel) ? sm.cand[i] : 0ull;
        __syncthreads();
        block_bitonic_desc(scratch, P);
        for (int i = tid; i < ksel; i += blockDim.x) sm.cand[i] = scratch[i];
        __syncthreads();
    } else {
        for (int k = 0; k < nbig; ++k) {
            unsigned long long* scratch = reinterpret_cast<unsigned long long*>(sm.row);
            const int s0 = sm.big_start[k], n = sm.big_len[k];
            int P = 1;
            while (P < n) P <<= 1;
            for (int i = tid; i < P; i += blockDim.x) scratch[i] = (i < n) ? sm.cand[s0 + i] : 0ull;
            __syncthreads();
            block_bitonic_desc(scratch, P);
            for (int i = tid; i < n; i += blockDim.x) sm.cand[s0 + i] = scratch[i];
            __syncthreads();
        }
    }

    // T5: serial cumulative sum over the sorted nucleus until it exceeds topp
    // (llama2.c:1036-1043).
    const int nch = stage_sorted_probs(sm, sm.cand, ksel);
    chain_run<8>(sm, nch, 0.0f);
    chain_find<8>(sm, nch, c.topp);
    int last;
    float cum;
    if (sm.found_idx >= 0 && sm.found_idx < ksel) {
        last = sm.found_idx;
        cum = sm.found_val;
    } else if (ksel == n0) {
        last = n0 - 1;
        cum = sm.chunk_s[nch];
    } else {
        // The guaranteed-mass bound did not hold (not expected): the caller
        // re-stages the probabilities and takes the exact global path.
        flags |= kFlagSlow;
        return -2;
    }
    // T6: r = coin * cum, first sorted index with r < cdf (llama2.c:1046-1054).
    const float r = __fmul_rn(c.coin, cum);
    chain_find<8>(sm, nch, r);
    const int fi = (sm.found_idx >= 0 && sm.found_idx <= last) ? sm.found_idx : last;
    return key_index(sm.cand[fi]);
}

__global__ void __launch_bounds__(kRowThreads, 1) row_sampler_kernel(RowLaunch p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    RowSmem& sm = *reinterpret_cast<RowSmem*>(smem_raw);
    const int tid = threadIdx.x;

    if (tid < xm::kExpTableSize) sm.exptab[tid] = xm::exp_table_entry(tid);
    if (tid == 0) {
        mbar_init(&sm.mbar[0], 1);
        fence_mbar_init();
    }
    __syncthreads();

    const int V = p.vocab;
    const int nch = (V + kRowCPT - 1) / kRowCPT;
    const bool tma_ok = ((reinterpret_cast<uintptr_t>(p.logits) & 15u) == 0) && ((p.ld & 3) == 0);
    const int vbody = tma_ok ? (V & ~3) : 0;
    unsigned long long* ws = p.workspace ? p.workspace + (long long)blockIdx.x * p.ws_stride : nullptr;

    unsigned phase = 0;
    const int nrows = p.row_list ? *p.row_count : p.batch;
    for (int it = blockIdx.x; it < nrows; it += gridDim.x) {
        const int row = p.row_list ? p.row_list[it] : it;
        const float* src = p.logits + (long long)row * p.ld;
        int flags = 0;

        // 1. stage the row
        if (vbody > 0) {
            // the self-test issues no copy for its first row: nothing arrives
            const bool stall = p.wait_test != 0 && it == (int)blockIdx.x;
            if (tid == 0 && !stall) {
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&sm.mbar[0], (unsigned)vbody * 4u);
                const int part = ((vbody / kTmaParts) + 3) & ~3;
                for (int off = 0; off < vbody; off += part) {
                    const int len = min(part, vbody - off);
                    bulk_copy_g2s(sm.row + off, src + off, (unsigned)len * 4u, &sm.mbar[0]);
                }
            }
            const bool ok = mbar_wait_bounded(&sm.mbar[0], phase, p.wait_test ? p.wait_test : kSpinLimit);
            phase ^= 1u;
            if (!__syncthreads_and(ok)) {
                // The copy did not land in time: report, wait (bounded) for the
                // copies in flight, mark this CTA's unfinished rows, stop.
                if (tid == 0) atomicExch(p.error_word, 1);
                if (!stall) mbar_wait_bounded(&sm.mbar[0], phase ^ 1u);
                for (int j = it + tid * (int)gridDim.x; j < nrows; j += (int)(blockDim.x * gridDim.x)) {
                    const int r = p.row_list ? p.row_list[j] : j;
                    if (p.row_flags) p.row_flags[r] = kFlagTimeout;
                    p.out_ids[r] = 0;
                }
                return;
            }
        }
        for (int i = vbody + tid; i < V; i += blockDim.x) sm.row[i] = src[i];
        __syncthreads();

        RowCtx c;
        c.V = V;
        c.nch = nch;
        c.T = p.temperature_rows ? p.temperature_rows[row] : p.temperature;
        c.topp = p.topp_rows ? p.topp_rows[row] : p.topp;
        c.probs_in = p.probs_in != 0;
        c.write_probs = p.probs_out != nullptr;
        c.probs_row = p.probs_out ? p.probs_out + (long long)row * V : nullptr;
        // sample(): T == 0 (llama2.c:1085); do_sample / sample_debug: T < 1e-6f
        // (llama2_cublas_fp16.cu:1179, llama2_cublas.cu:5089)
        const bool greedy = !c.probs_in && (c.T == 0.0f || (p.greedy_eps && c.T < 1e-6f));
        // sample_debug's NaN test on the raw logits (llama2_cublas.cu:5071-5085)
        bool nan1 = false;
        if (p.nan_token1) {
            bool h = false;
            for (int i = tid; i < V; i += blockDim.x) h |= isnan(sm.row[i]);
            nan1 = __syncthreads_or(h) != 0;
        }

        int id = 0;
        if (nan1) {
            // token 1, no coin drawn, the buffer keeps the logits
            id = 1;
            flags |= kFlagNan;
            if (c.write_probs)
                for (int i = tid; i < V; i += blockDim.x) c.probs_row[i] = sm.row[i];
        } else if (greedy) {
            id = row_argmax(sm, V);
            if (c.write_probs)
                for (int i = tid; i < V; i += blockDim.x) c.probs_row[i] = sm.row[i];
        } else {
            unsigned long long st = 0;
            if (p.coins) {
                c.coin = p.coins[row];
            } else {
                st = p.rng_state[row];
                c.coin = draw_coin(st);
            }
            const bool mult = (p.force_mode == 1) ||
                              (p.force_mode == 0 && (c.topp <= 0.0f || c.topp >= 1.0f));
            bool nan_row = false, serial = false;
            float S = 1.0f, max_x = 0.0f;
            if (!c.probs_in) {
                float mx, mn;
                row_minmax(sm, V, mx, mn);
                max_x = (c.T == 1.0f) ? mx : (c.T > 0.0f ? __fdiv_rn(mx, c.T) : __fdiv_rn(mn, c.T));
                nan_row = row_exp_pass(sm, c, max_x);
                if (!nan_row) {
                    chain_run<kRowCPT>(sm, nch, 0.0f);
                    S = sm.chunk_s[nch];
                }
            } else {
                serial = row_permute_pass(sm, c);
            }
            if (nan_row) {
                flags |= kFlagNan;
                if (c.write_probs)
                    for (int i = tid; i < V; i += blockDim.x) c.probs_row[i] = __uint_as_float(0x7FC00000u);
                if (mult) {
                    id = V - 1;
                } else {
                    id = 0;
                    flags |= kFlagNoCand;
                }
            } else if (mult) {
                if (!c.probs_in) row_div_pass(sm, c, S);
                if (serial) {
                    flags |= kFlagSerial;
                    id = row_serial_mult(sm, c);
                } else {
                    chain_run<kRowCPT>(sm, nch, 0.0f);
                    chain_find<kRowCPT>(sm, nch, c.coin);
                    id = (sm.found_idx >= 0 && sm.found_idx < V) ? sm.found_idx : V - 1;
                }
            } else {
                id = row_topp(sm, c, S, ws, flags);
                if (id == -2) {
                    // Rebuild p in the swizzled layout from the source row (same
                    // arithmetic as above) and run the global-memory path.
                    __syncthreads();
                    for (int i = tid; i < V; i += blockDim.x) sm.row[i] = src[i];
                    __syncthreads();
                    if (!c.probs_in) {
                        row_exp_pass(sm, c, max_x);
                        RowCtx c2 = c;
                        c2.write_probs = false;
                        row_div_pass(sm, c2, S);
                    } else {
                        row_permute_pass(sm, c);
                    }
                    const float cutoff = __fdiv_rn(__fsub_rn(1.0f, c.topp), (float)(V - 1));
                    const int g = topp_global_path(sm, V, cutoff, c.topp, c.coin, ws);
                    if (g < 0) flags |= kFlagNoCand;
                    id = g < 0 ? 0 : g;
                }
            }
            if (tid == 0 && !p.coins) p.rng_state[row] = st;
        }
        if (tid == 0) {
            p.out_ids[row] = id;
            if (p.row_flags) p.row_flags[row] = flags;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// Greedy kernel: one 256-thread CTA per row, streaming float4 loads.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) argmax_kernel(ArgmaxLaunch p) {
    const int row = blockIdx.x;
    const float* src = p.logits + (long long)row * p.ld;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
    const int V = p.vocab;
    const bool vec = ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) &&
                     (!p.probs_out || ((reinterpret_cast<uintptr_t>(p.probs_out + (long long)row * V) & 15u) == 0));
    if (vec) {
        const int ng = V >> 2;
        const float4* s4 = reinterpret_cast<const float4*>(src);
        for (int g = tid; g < ng; g += blockDim.x) {
            const float4 q = __ldcs(s4 + g);
            const float a[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const int i = 4 * g + w;
                if (a[w] > bv || (a[w] == bv && i < bi)) {
                    bv = a[w];
                    bi = i;
                }
            }
            if (p.probs_out) reinterpret_cast<float4*>(p.probs_out + (long long)row * V)[g] = q;
        }
        for (int i = (ng << 2) + tid; i < V; i += blockDim.x) {
            const float x = src[i];
            if (x > bv || (x == bv && i < bi)) {
                bv = x;
                bi = i;
            }
            if (p.probs_out) p.probs_out[(long long)row * V + i] = x;
        }
    } else {
        for (int i = tid; i < V; i += blockDim.x) {
            const float x = src[i];
            if (x > bv || (x == bv && i < bi)) {
                bv = x;
                bi = i;
            }
            if (p.probs_out) p.probs_out[(long long)row * V + i] = x;
        }
    }
    __shared__ float sv[8];
    __shared__ int si[8];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(kFullMask, bv, o);
        const int oi = __shfl_xor_sync(kFullMask, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < 8; ++w) {
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
                bv = sv[w];
                bi = si[w];
            }
        }
        const bool nan0 = isnan(src[0]);
        p.out_ids[row] = (nan0 || bi == 0x7FFFFFFF) ? 0 : bi;
    }
}

__global__ void seed_kernel(unsigned long long* st, int batch, unsigned long long seed, long long off) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < batch) st[i] = seed + (unsigned long long)(off + i);
}

}  // namespace

size_t row_kernel_smem_bytes() { return sizeof(RowSmem); }

int launch_row_sampler(const RowLaunch& p, int num_ctas, cudaStream_t stream) {
    // The opt-in shared-memory size is a per-device attribute of the kernel.
    static std::atomic<unsigned long long> attr_done{0};
    int dev = 0;
    cudaError_t e0 = cudaGetDevice(&dev);
    if (e0 != cudaSuccess) return -(int)e0;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_done.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(row_sampler_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sizeof(RowSmem));
        if (e != cudaSuccess) return -(int)e;
        attr_done.fetch_or(bit);
    }
    row_sampler_kernel<<<num_ctas, kRowThreads, sizeof(RowSmem), stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -(int)e;
}

int launch_argmax(const ArgmaxLaunch& p, cudaStream_t stream) {
    argmax_kernel<<<p.batch, 256, 0, stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -(int)e;
}

int launch_seed_states(unsigned long long* st, int batch, unsigned long long seed, long long offset,
                       cudaStream_t stream) {
    seed_kernel<<<(batch + 255) / 256, 256, 0, stream>>>(st, batch, seed, offset);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -(int)e;
}

}  // namespace b2s
