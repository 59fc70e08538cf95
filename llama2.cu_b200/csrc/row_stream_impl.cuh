// row_stream_impl.cuh -- body of the streaming top-p kernel, included by
// row_stream.cu once per CTA shape (RS_THREADS threads, RS_CTAS_PER_SM CTAs
// per SM, RS_SORT_GROUP bins per sort group, RS_KEY_CAP nucleus keys on chip,
// in namespace b2s::RS_NS).  The
// algorithm is described in row_stream.cu.
namespace RS_NS {
namespace {

constexpr int kST = RS_THREADS;  // threads per CTA
constexpr int kSW = kST / 32;  // warps per CTA
constexpr int kSC = 32;        // elements per chunk
constexpr int kChunks = 1024;  // chunks of 32 (V <= 32768)
constexpr int kStrips = kChunks / kST;  // chunks per thread (strip s: chunk kST*s + t)
constexpr int kSegs = kChunks / 32;         // 32 segments of 32 chunks
constexpr int kKCap = RS_KEY_CAP;  // nucleus keys kept on chip (more spill to L2)
// Shapes with a large on-chip nucleus also keep its p values with each chunk
// of 32 padded to 33 floats, so that thread t reading value j of chunk t hits
// bank (t + j) mod 32 (the keys themselves, 256 bytes per chunk, put every
// thread of a warp on one bank).
constexpr bool kPadP = kKCap > 4096;
constexpr int kPadPLen = kPadP ? ((kKCap / kSC) * (kSC + 1) + 3) / 4 * 4 : 4;  // whole 16-byte units
constexpr int kSideCap = 48;   // chunks whose values are kept for replays
constexpr int kAltCap = 96;    // chunks with an alternative-binade function
constexpr int kBinsPerThread = kBins / kST;
constexpr int kWalkDirect = 1024;  // nuclei walked by the serial loop (their sums fit the chunk table)
constexpr int kPairCap = 128;   // equal-p neighbour positions recorded for the tie fix

// chunk entry: x=L0 y=L1 z=bits(pbits | flags | alt<<8 | side<<16 | run end<<24) w=bits(eb)
// A run chunk (kFRun) is clean in its guessed binade with no alternative; its
// entry holds the composition of the chunks from it to the end of its run
// (the consecutive run chunks of one binade among the warp's 32), and bits
// 24-28 the lane of that last chunk.  Other chunks hold their own function.
constexpr uint32_t kFClean = 4u, kFValid = 8u, kFAlt = 16u, kFRun = 32u;

struct StreamSmem {
    unsigned long long kbuf[kKCap];
    float padp[kPadPLen];  // p of key i at (i / 32) * 33 + i % 32 (kPadP shapes)
    int hist[kBins];
    unsigned short bstart[kBins];  // bin offsets in the nucleus (< 2^16)
    alignas(16) float side[kSideCap][kSC];  // read and written as float4
    float4 fn[kChunks];
    float4 alt[kAltCap];
    float4 wfn[kSegs];
    xm::ExpTableEntry exptab[xm::kExpTableSize];
    float red_a[kSW];
    float red_b[kSW];
    float red_c[kSW];
    int red_i[kSW];
    int n_alt;
    int n_side;
    int flag;
    int dbin;
    int sort_next;  // next group of 32 bins to sort
    int next_row[2];  // the row this CTA takes next (two slots: claimed one row ahead)
    int n_pairs;    // equal-p neighbours found by the p pass
    int pairs[kPairCap];
    int ksel;
    int result;
    int n0;
    float fval;
    // running sums of the first walk over a large nucleus (cum > topp) at
    // segment starts, where the second (r < cdf, the same serial sums) may
    // resume
    float ck_s[32];
};

// RS_CTAS_PER_SM CTAs per SM: 228 KB of shared memory per SM, 1 KB reserved per CTA.
static_assert(RS_CTAS_PER_SM * (sizeof(StreamSmem) + 1024) <= 228 * 1024, "StreamSmem too large");
static_assert(kWalkDirect <= 4 * kChunks, "the serial walk records its sums in the chunk table");
static_assert(offsetof(StreamSmem, side) % 16 == 0 && offsetof(StreamSmem, fn) % 16 == 0 &&
                  offsetof(StreamSmem, alt) % 16 == 0 && offsetof(StreamSmem, wfn) % 16 == 0 &&
                  offsetof(StreamSmem, kbuf) % 16 == 0,
              "members accessed as float4 / 16-byte units must be 16-byte aligned");

struct Ctx {
    const float* src;  // row
    int V;
    int nch;
    float T, rT;
    float max_x;
    bool unit;
    bool v32;  // rows 32-byte aligned: chunks load as 32-byte vectors
};

// ---------------------------------------------------------------------------
// block helpers (256 threads)
// ---------------------------------------------------------------------------
struct ScanF {
    float incl, excl, total;
};

// Float scan whose exclusive value of thread t+1 is bitwise the inclusive
// value of thread t, so "excl < x <= incl" selects exactly one thread.
__device__ ScanF block_scan_f(float v, StreamSmem& sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(kFullMask, v, o);
        if (lane >= o) v += y;
    }
    const float e = __shfl_up_sync(kFullMask, v, 1);
    if (lane == 31) sm.red_a[warp] = v;
    __syncthreads();
    float p = 0.0f, t = 0.0f;
#pragma unroll
    for (int w = 0; w < kSW; ++w) {
        const float x = sm.red_a[w];
        if (w < warp) p += x;
        t += x;
    }
    __syncthreads();
    ScanF r;
    r.incl = p + v;
    r.excl = lane == 0 ? p : p + e;
    r.total = t;
    return r;
}

__device__ int block_scan_i(int v, StreamSmem& sm, int& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFullMask, v, o);
        if (lane >= o) v += y;
    }
    if (lane == 31) sm.red_i[warp] = v;
    __syncthreads();
    int p = 0, t = 0;
#pragma unroll
    for (int w = 0; w < kSW; ++w) {
        const int x = sm.red_i[w];
        if (w < warp) p += x;
        t += x;
    }
    __syncthreads();
    total = t;
    return p + v;
}

__device__ __forceinline__ xm::ChainFn fn_shfl_up(const xm::ChainFn& f, int o) {
    return xm::ChainFn{__shfl_up_sync(kFullMask, f.L0, o), __shfl_up_sync(kFullMask, f.L1, o),
                       __shfl_up_sync(kFullMask, f.pbits, o)};
}
__device__ __forceinline__ xm::ChainFn fn_shfl_down(const xm::ChainFn& f, int o) {
    return xm::ChainFn{__shfl_down_sync(kFullMask, f.L0, o), __shfl_down_sync(kFullMask, f.L1, o),
                       __shfl_down_sync(kFullMask, f.pbits, o)};
}

// Segmented suffix composition across the warp's lanes: lane i returns
// f_i then f_(i+1) ... up to the last lane of its run (`end`), where `link`
// says that lane i's run continues into lane i + 1.  Lanes outside a run pass
// the identity with link = false.
__device__ __forceinline__ xm::ChainFn warp_run_suffix(xm::ChainFn f, bool link, int& end) {
    const int lane = threadIdx.x & 31;
    end = lane;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const xm::ChainFn g = fn_shfl_down(f, o);
        const int link_g = __shfl_down_sync(kFullMask, (int)link, o);
        const int end_g = __shfl_down_sync(kFullMask, end, o);
        if (link && lane + o < 32) {  // f covers [lane, lane + o) and the run goes on
            f = xm::chain_compose(f, g);
            link = link_g != 0;
            end = end_g;
        }
    }
    return f;
}

__device__ __forceinline__ xm::ChainFn warp_incl_compose(xm::ChainFn f) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const xm::ChainFn y = fn_shfl_up(f, o);
        if (lane >= o) f = xm::chain_compose(y, f);
    }
    return f;
}

__device__ __forceinline__ bool regular_sum(float s) {
    const uint32_t eb = xm::binade_of(s);
    return s > 0.0f && eb >= xm::kMinFastBinade && eb < 254u;
}

// Exact e value of one logit.
__device__ __forceinline__ float exact_e(const Ctx& c, const StreamSmem& sm, float l) {
    const float x = c.unit ? l : xm_div_const(l, c.T, c.rT);
    return xm::exp_f32(__fsub_rn(x, c.max_x), sm.exptab);
}

// Replays chunk t exactly starting from s (warp 0): kept values, or values
// recomputed from the row.  A replayed chunk is one whose running sum crosses
// a binade (often several, early in the row), so the 32 adds are done
// serially -- redundantly in every lane, on values gathered into registers
// first -- rather than by the warp-parallel chain, whose steps end at every
// crossing.  Padding lanes add +0, which leaves s >= 0 unchanged.
__device__ float replay_chunk(StreamSmem& sm, const Ctx& c, int t, uint32_t side_plus1, float s) {
    const int lane = threadIdx.x & 31;
    const int base = t * kSC;
    const int cnt = min(kSC, c.V - base);
    if (side_plus1) {
        // kept values (zero past cnt): every lane reads the same 16 bytes
        const float4* kv = reinterpret_cast<const float4*>(sm.side[side_plus1 - 1]);
#pragma unroll
        for (int q = 0; q < kSC / 4; ++q) {
            const float4 x = kv[q];
            s = __fadd_rn(s, x.x);
            s = __fadd_rn(s, x.y);
            s = __fadd_rn(s, x.z);
            s = __fadd_rn(s, x.w);
        }
        return s;
    }
    float e = 0.0f;
    if (lane < cnt) e = exact_e(c, sm, __ldg(c.src + base + lane));
    float v[kSC];
#pragma unroll
    for (int i = 0; i < kSC; ++i) v[i] = __shfl_sync(kFullMask, e, i);
#pragma unroll
    for (int i = 0; i < kSC; ++i) s = __fadd_rn(s, v[i]);
    return s;
}

// Exact serial walk over the chunks of segment seg from s (warp 0, every
// lane the same values): a run chunk applies its whole run at once, other
// chunks their own or their alternative-binade function; a chunk whose
// function does not hold for s (its running sum leaves the binade, or the
// binade guess was wrong) is replayed.
__device__ float walk_segment(StreamSmem& sm, const Ctx& c, int seg, float s) {
    const int cnt = min(32, c.nch - seg * 32);
    int cpos = 0;
    while (cpos < cnt) {
        const int t = seg * 32 + cpos;
        const float4 ent = sm.fn[t];
        const uint32_t ez = __float_as_uint(ent.z);
        if (ez & kFClean) {
            float s2 = s;
            if (xm::chain_apply(s2, __float_as_uint(ent.w), xm::ChainFn{ent.x, ent.y, ez & 3u})) {
                s = s2;
                cpos = (ez & kFRun) ? (int)((ez >> 24) & 31u) + 1 : cpos + 1;
                continue;
            }
        }
        if (ez & kFAlt) {
            const float4 a = sm.alt[(ez >> 8) & 0xFFu];
            float s2 = s;
            if (xm::chain_apply(s2, __float_as_uint(a.w), xm::ChainFn{a.x, a.y, __float_as_uint(a.z) & 3u})) {
                s = s2;
                ++cpos;
                continue;
            }
        }
        s = replay_chunk(sm, c, t, (ez >> 16) & 0xFFu, s);
        ++cpos;
    }
    return s;
}

// Exact serial softmax denominator from the chunk tables (warp 0).  Lane k
// holds segment k's function (clean when its 32 chunks are one run); runs of
// clean segments of one binade are composed (segmented suffix scan), so the
// walk jumps over each run of segments at once and walks chunk by chunk only
// where a binade boundary lies.
__device__ float resolve_S(StreamSmem& sm, const Ctx& c) {
    const int lane = threadIdx.x & 31;
    const int nseg = (c.nch + 31) / 32;
    const float4 wf = (lane < nseg) ? sm.wfn[lane] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const uint32_t wz = __float_as_uint(wf.z), web = __float_as_uint(wf.w);
    const bool su = (lane < nseg) && (wz & kFClean);
    const xm::ChainFn own = su ? xm::ChainFn{wf.x, wf.y, wz & 3u} : xm::chain_identity();
    const bool su_n = __shfl_down_sync(kFullMask, (int)su, 1) != 0;
    const uint32_t web_n = __shfl_down_sync(kFullMask, web, 1);
    int run_end = lane;
    const xm::ChainFn run = warp_run_suffix(own, su && lane < 31 && su_n && web_n == web, run_end);
    float s = 0.0f;
    int seg = 0;
    while (seg < nseg) {
        if (__shfl_sync(kFullMask, (int)su, seg)) {
            const uint32_t eb = __shfl_sync(kFullMask, web, seg);
            float s2 = s;
            const xm::ChainFn R{__shfl_sync(kFullMask, run.L0, seg), __shfl_sync(kFullMask, run.L1, seg),
                                __shfl_sync(kFullMask, run.pbits, seg)};
            if (xm::chain_apply(s2, eb, R)) {
                s = s2;
                seg = __shfl_sync(kFullMask, run_end, seg) + 1;
                continue;
            }
            s2 = s;
            const xm::ChainFn O{__shfl_sync(kFullMask, own.L0, seg), __shfl_sync(kFullMask, own.L1, seg),
                                __shfl_sync(kFullMask, own.pbits, seg)};
            if (xm::chain_apply(s2, eb, O)) {
                s = s2;
                ++seg;
                continue;
            }
        }
        s = walk_segment(sm, c, seg, s);
        ++seg;
    }
    return s;
}

// ---------------------------------------------------------------------------
// Large nuclei: the serial cumulative sum of the sorted p (llama2.c:1036-1054)
// walked by chunk functions, as the softmax denominator is resolved.
// ---------------------------------------------------------------------------

// All threads: chunk t = sorted keys [32t, 32t + 32) of the first n0; its
// incoming cumulative sum is guessed from a block scan of approximate chunk
// sums.  Fills fn / alt / wfn (free again once S is resolved).  padp: the
// nucleus's p values in the padded layout, or null (read the keys).  Out of
// line: inlined, it raised the kernel's register demand into spills.
__device__ __noinline__ void build_walk_fns(StreamSmem& sm, const unsigned long long* kb, const float* padp, int n0) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nchk = (n0 + kSC - 1) / kSC;
    if (tid == 0) sm.n_alt = 0;
    float sig[kStrips], gss[kStrips];
#pragma unroll
    for (int sidx = 0; sidx < kStrips; ++sidx) {
        const int t = sidx * kST + tid;
        float a = 0.0f;
        if (t < nchk) {
            const int cnt = min(kSC, n0 - kSC * t);
#pragma unroll 8  // loads in flight from the L2 scratch
            for (int j = 0; j < cnt; ++j) a += padp ? padp[(kSC + 1) * t + j] : key_prob(kb[kSC * t + j]);
        }
        sig[sidx] = a;
    }
    float off = 0.0f;
#pragma unroll
    for (int sidx = 0; sidx < kStrips; ++sidx) {
        const ScanF sc = block_scan_f(sig[sidx], sm);
        gss[sidx] = off + sc.excl;
        off += sc.total;
    }
#pragma unroll 1
    for (int sidx = 0; sidx < kStrips; ++sidx) {
        const int t = sidx * kST + tid;
        const bool valid = t < nchk;
        const int cnt = valid ? min(kSC, n0 - kSC * t) : 0;
        uint32_t alt = 0u;
        const uint32_t eb = valid ? xm::chain_guess_primary(gss[sidx], sig[sidx], alt) : 0u;
        const float lo = __uint_as_float(eb << 23), lo1 = __uint_as_float((eb << 23) | 1u);
        const float alo = __uint_as_float(alt << 23), alo1 = __uint_as_float((alt << 23) | 1u);
        float v0 = lo, v1 = lo1, w0 = alo, w1 = alo1;
#pragma unroll 8
        for (int j = 0; j < cnt; ++j) {
            const float x = padp ? padp[(kSC + 1) * t + j] : key_prob(kb[kSC * t + j]);
            v0 = __fadd_rn(v0, x);
            v1 = __fadd_rn(v1, x);
            w0 = __fadd_rn(w0, x);
            w1 = __fadd_rn(w1, x);
        }
        const bool clean = valid && eb != 0u && (__float_as_uint(v0) >> 23) == eb && (__float_as_uint(v1) >> 23) == eb;
        const bool aclean = valid && alt != 0u && (__float_as_uint(w0) >> 23) == alt && (__float_as_uint(w1) >> 23) == alt;
        const xm::ChainFn f{__fsub_rn(v0, lo), __fsub_rn(v1, lo1),
                            (__float_as_uint(v0) & 1u) | ((__float_as_uint(v1) & 1u) << 1)};
        uint32_t z = (clean ? (f.pbits | kFClean) : 0u) | (valid ? kFValid : 0u);
        if (aclean) {
            const int ai = atomicAdd(&sm.n_alt, 1);
            if (ai < kAltCap) {
                sm.alt[ai] = make_float4(__fsub_rn(w0, alo), __fsub_rn(w1, alo1),
                                         __uint_as_float((__float_as_uint(w0) & 1u) |
                                                         ((__float_as_uint(w1) & 1u) << 1) | kFClean),
                                         __uint_as_float(alt));
                z |= kFAlt | ((uint32_t)ai << 8);
            }
        }
        if (valid) sm.fn[t] = make_float4(f.L0, f.L1, __uint_as_float(z), __uint_as_float(eb));
        const uint32_t eb0 = __shfl_sync(kFullMask, eb, 0);
        const bool uni = __all_sync(kFullMask, !valid || (clean && eb == eb0 && !(z & kFAlt)));
        const xm::ChainFn F = warp_incl_compose((valid && clean) ? f : xm::chain_identity());
        if (lane == 31)
            sm.wfn[sidx * kSW + warp] =
                make_float4(F.L0, F.L1, __uint_as_float(F.pbits | (uni ? kFClean : 0u)), __uint_as_float(eb0));
    }
    __syncthreads();
}

// Warp 0: the first i < n with cum_i = fl(cum_{i-1} + p_i) > theta (cum is
// then cum_i), or n (cum = cum_{n-1}), over the chunk functions of
// build_walk_fns (built for n0 >= n keys).  Whole segments and chunks are
// applied while they stay in one binade and end at or below theta; the chunk
// that crosses theta or a binade is walked element by element.  ck_s records
// the sum before each segment walked; (seg0, s0) resumes at a recorded one.
template <class Get>
__device__ int walk_fns(const StreamSmem& sm, int n, float theta, float& cum, const Get& get, float* ck_s = nullptr,
                        int seg0 = 0, float s0 = 0.0f) {
    const int lane = threadIdx.x & 31;
    float s = s0;
    const int nchk = (n + kSC - 1) / kSC;
    const int nseg = (nchk + 31) / 32;
    for (int seg = seg0; seg < nseg; ++seg) {
        if (ck_s && lane == 0) ck_s[seg] = s;  // the sum of the elements before segment seg
        const int cnt = min(32, nchk - seg * 32);
        const float4 wf = sm.wfn[seg];
        const uint32_t wz = __float_as_uint(wf.z);
        // a whole segment only when all of its chunks are inside [0, n)
        if ((wz & kFClean) && seg * 32 * kSC + 32 * kSC <= n) {
            float s2 = s;
            if (xm::chain_apply(s2, __float_as_uint(wf.w), xm::ChainFn{wf.x, wf.y, wz & 3u}) && !(s2 > theta)) {
                s = s2;
                continue;
            }
        }
        // chunks wholly inside [0, n) may use their functions
        const int t_lane = seg * 32 + lane;
        const bool whole = (t_lane + 1) * kSC <= n;
        const float4 ent = (lane < cnt) ? sm.fn[t_lane] : make_float4(0, 0, 0, 0);
        const uint32_t ez = __float_as_uint(ent.z);
        float4 aent = make_float4(0, 0, 0, 0);
        if (lane < cnt && (ez & kFAlt)) aent = sm.alt[(ez >> 8) & 0xFFu];
        const uint32_t az = __float_as_uint(aent.z);
        int cpos = 0;
        while (cpos < cnt) {
            if (regular_sum(s)) {
                const uint32_t eb = xm::binade_of(s);
                const bool use_p = whole && (ez & kFClean) && __float_as_uint(ent.w) == eb;
                const bool use_a = whole && !use_p && (ez & kFAlt) && (az & kFClean) && __float_as_uint(aent.w) == eb;
                const bool has = (lane >= cpos) && (lane < cnt) && (use_p || use_a);
                xm::ChainFn f = xm::chain_identity();
                if (has) f = use_p ? xm::ChainFn{ent.x, ent.y, ez & 3u} : xm::ChainFn{aent.x, aent.y, az & 3u};
                const unsigned hm = __ballot_sync(kFullMask, has || lane < cpos);
                const int fi = (~hm) ? (__ffs(~hm) - 1) : 32;
                f = warp_incl_compose(f);
                const float hi = __uint_as_float((eb + 1u) << 23);
                const float L = (__float_as_uint(s) & 1u) ? f.L1 : f.L0;
                const bool fits_b = (lane < fi) && (L <= __fsub_rn(hi, s));
                const float sl = __fadd_rn(s, L);
                // chunks [cpos, m) end inside the binade and at or below theta
                const bool inb = (lane < cpos) || (fits_b && !(sl > theta));
                const unsigned inm = __ballot_sync(kFullMask, inb);
                const int m = (~inm) ? (__ffs(~inm) - 1) : 32;
                if (m > cpos) {
                    s = __shfl_sync(kFullMask, sl, m - 1);
                    cpos = m;
                }
            }
            if (cpos < cnt) {
                const int base = (seg * 32 + cpos) * kSC;
                const int ne = min(kSC, n - base);
                // the crossing chunk: 32 serial adds (one coalesced load),
                // 16 values gathered at a time and added as one dependent
                // chain; the sums only grow, so a group holds the crossing
                // of theta iff its last sum does (padding lanes add +0, so
                // the first crossing is a real element)
                const float x = (lane < ne) ? get(base + lane) : 0.0f;
#pragma unroll
                for (int h = 0; h < kSC / 16; ++h) {
                    float c16[16];
#pragma unroll
                    for (int q = 0; q < 16; ++q) c16[q] = __shfl_sync(kFullMask, x, 16 * h + q);
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        s = __fadd_rn(s, c16[q]);
                        c16[q] = s;
                    }
                    if (c16[15] > theta) {
                        int u = 15;
                        float cu = c16[15];
#pragma unroll
                        for (int v = 14; v >= 0; --v)
                            if (c16[v] > theta) {
                                u = v;
                                cu = c16[v];
                            }
                        cum = cu;
                        return base + 16 * h + u;
                    }
                }
                ++cpos;
            }
        }
    }
    cum = s;
    return n;
}

__device__ int walk_chunks(const StreamSmem& sm, const unsigned long long* kb, int n, float theta, float& cum,
                           float* ck_s = nullptr, int seg0 = 0, float s0 = 0.0f) {
    return walk_fns(sm, n, theta, cum, [&](int i) { return key_prob(kb[i]); }, ck_s, seg0, s0);
}

// ---------------------------------------------------------------------------
// sample_mult rows (llama2.c:994-1005): the first i with coin < cdf_i, cdf_i
// the serial fp32 sum of p_j = fl(e_j / S) over j <= i in index order, or
// n - 1.  The chunk functions of the p's (recomputed exactly from the row)
// give the cdf; the incoming cdf of each chunk is guessed from pass 1's
// approximate prefix of e divided by S.
// ---------------------------------------------------------------------------
// p = fl(e/S): Markstein division where it is correctly rounded (S in
// [1, 2^15], e >= 2^-60), IEEE division below (tiny and subnormal quotients).
__device__ __forceinline__ float p_of(const Ctx& c, const StreamSmem& sm, float l, float S, float rS) {
    const float e = exact_e(c, sm, l);
    if (!(e >= 0x1p-60f)) return __fdiv_rn(e, S);
    const float q = __fmul_rn(e, rS);
    return __fmaf_rn(__fmaf_rn(-q, S, e), rS, q);
}

// All threads: cdf chunk functions for chunks 0..nch-1 (chunk t = elements
// [32t, 32t + 32) of the row).  gss/sig: pass 1's approximate e prefix and
// chunk sums of this thread's strips.
__device__ void build_cdf_fns(StreamSmem& sm, const Ctx& c, float S, const float (&gss)[kStrips],
                              const float (&sig)[kStrips], float* probs_row) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float rS = __frcp_rn(S);
    if (tid == 0) sm.n_alt = 0;
    __syncthreads();
#pragma unroll 1
    for (int sidx = 0; sidx < kStrips; ++sidx) {
        const int t = sidx * kST + tid;
        const bool valid = t < c.nch;
        const int cnt = valid ? min(kSC, c.V - t * kSC) : 0;
        uint32_t alt = 0u;
        const uint32_t eb = valid ? xm::chain_guess_primary(gss[sidx] * rS, sig[sidx] * rS, alt) : 0u;
        const float lo = __uint_as_float(eb << 23), lo1 = __uint_as_float((eb << 23) | 1u);
        const float alo = __uint_as_float(alt << 23), alo1 = __uint_as_float((alt << 23) | 1u);
        float v0 = lo, v1 = lo1, w0 = alo, w1 = alo1;
        const float* cp = c.src + t * kSC;
#pragma unroll 1
        for (int g = 0; g < kSC / 4; ++g) {
            if (4 * g >= cnt) break;
            const float4 q = __ldg(reinterpret_cast<const float4*>(cp + 4 * g));
            const float a[4] = {q.x, q.y, q.z, q.w};
            float pv[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const float x = (4 * g + w < cnt) ? p_of(c, sm, a[w], S, rS) : 0.0f;
                pv[w] = x;
                v0 = __fadd_rn(v0, x);
                v1 = __fadd_rn(v1, x);
                w0 = __fadd_rn(w0, x);
                w1 = __fadd_rn(w1, x);
            }
            if (probs_row)  // the softmax sample() leaves in the buffer (cnt is a multiple of 4)
                reinterpret_cast<float4*>(probs_row + t * kSC)[g] = make_float4(pv[0], pv[1], pv[2], pv[3]);
        }
        const bool clean = valid && eb != 0u && (__float_as_uint(v0) >> 23) == eb && (__float_as_uint(v1) >> 23) == eb;
        const bool aclean = valid && alt != 0u && (__float_as_uint(w0) >> 23) == alt && (__float_as_uint(w1) >> 23) == alt;
        const xm::ChainFn f{__fsub_rn(v0, lo), __fsub_rn(v1, lo1),
                            (__float_as_uint(v0) & 1u) | ((__float_as_uint(v1) & 1u) << 1)};
        uint32_t z = (clean ? (f.pbits | kFClean) : 0u) | (valid ? kFValid : 0u);
        if (aclean) {
            const int ai = atomicAdd(&sm.n_alt, 1);
            if (ai < kAltCap) {
                sm.alt[ai] = make_float4(__fsub_rn(w0, alo), __fsub_rn(w1, alo1),
                                         __uint_as_float((__float_as_uint(w0) & 1u) |
                                                         ((__float_as_uint(w1) & 1u) << 1) | kFClean),
                                         __uint_as_float(alt));
                z |= kFAlt | ((uint32_t)ai << 8);
            }
        }
        if (valid) sm.fn[t] = make_float4(f.L0, f.L1, __uint_as_float(z), __uint_as_float(eb));
        const uint32_t eb0 = __shfl_sync(kFullMask, eb, 0);
        const bool uni = __all_sync(kFullMask, !valid || (clean && eb == eb0 && !(z & kFAlt)));
        const xm::ChainFn F = warp_incl_compose((valid && clean) ? f : xm::chain_identity());
        if (lane == 31)
            sm.wfn[sidx * kSW + warp] =
                make_float4(F.L0, F.L1, __uint_as_float(F.pbits | (uni ? kFClean : 0u)), __uint_as_float(eb0));
    }
    __syncthreads();
}

// Sorts every bin 0..D of the scattered nucleus by (e desc, index asc).  Warps
// 1.. take groups of RS_SORT_GROUP bins from a shared counter (warp 0
// resolving S in the meantime; having it join afterwards measured slower):
// 32 bins with 4 CTAs per SM, where many rows share the SM; 8 bins with one
// CTA per SM, where a single row's large nucleus would otherwise leave most
// of its 31 warps without a group (15% faster there; 2% slower on the
// 4-CTA shape's mostly small nuclei).  Bins of up to 16 keys: each key's rank
// is the number of larger keys in its bin (keys are distinct); larger bins:
// bitonic networks.  Inside one bin (not the last) the value's top 15 bits
// are fixed, so 32-bit keys (low 17 value bits, 0x7FFF - index) order them
// for V < 0x7FFF.
constexpr int kSortGroup = RS_SORT_GROUP;  // bins per group taken by one warp (<= 32)
static_assert(kSortGroup >= 1 && kSortGroup <= 32, "a warp sorts up to 32 bins at a time");

__device__ void sort_bins(StreamSmem& sm, unsigned long long* kb, int D, int K, int V) {
    const int lane = threadIdx.x & 31;
    for (;;) {
        int g = 0;
        if (lane == 0) g = atomicAdd(&sm.sort_next, 1);
        const int b0 = __shfl_sync(kFullMask, g, 0) * kSortGroup;
        if (b0 > D) break;
        const int b = b0 + lane;
        int s0 = 0, n = 0;
        if (lane < kSortGroup && b <= D) {
            s0 = sm.bstart[b];
            n = sm.hist[b] - s0;
            if (s0 < 0 || s0 + n > K || n > 256) sm.flag = 1;
        }
        unsigned todo = __ballot_sync(kFullMask, n >= 2 && n <= 256 && s0 >= 0 && s0 + n <= K);
        const unsigned small = __ballot_sync(kFullMask, n <= 16);
        const unsigned mid = __ballot_sync(kFullMask, n > 16 && n <= 32);
        while (todo) {
            const int src = __ffs(todo) - 1;
            todo &= todo - 1;
            const int ss = __shfl_sync(kFullMask, s0, src);
            const int nn = __shfl_sync(kFullMask, n, src);
            unsigned long long* seg = kb + ss;
            const bool narrow = (b0 + src < kBins - 1) && V < 0x7FFF;
            if (nn <= 16) {
                // two small bins at a time, one per half-warp
                const unsigned rest = todo & small;
                const int src2 = rest ? (__ffs(rest) - 1) : -1;
                if (src2 >= 0) todo &= ~(1u << src2);
                const int ss2 = __shfl_sync(kFullMask, s0, src2 < 0 ? 0 : src2);
                const int nn2 = (src2 < 0) ? 0 : __shfl_sync(kFullMask, n, src2 < 0 ? 0 : src2);
                const bool narrow2 = narrow && (src2 < 0 || b0 + src2 < kBins - 1);
                const int hl = lane & 15;
                const int my_ss = (lane < 16) ? ss : ss2;
                const int my_nn = (lane < 16) ? nn : nn2;
                const unsigned long long key = (hl < my_nn) ? kb[my_ss + hl] : 0ull;
                const int top = max(nn, nn2);
                int rank = 0;
                if (narrow2) {
                    const uint32_t vb = (uint32_t)(key >> 32);
                    const uint32_t k32 = ((vb & 0x1FFFFu) << 15) | (uint32_t)(0x7FFF - key_index(key));
                    for (int t = 0; t < top; ++t) {
                        const uint32_t o = __shfl_sync(kFullMask, k32, (lane & 16) | t);
                        rank += (t < my_nn && o > k32) ? 1 : 0;
                    }
                } else {
                    for (int t = 0; t < top; ++t) {
                        const unsigned long long o = __shfl_sync(kFullMask, key, (lane & 16) | t);
                        rank += (t < my_nn && o > key) ? 1 : 0;
                    }
                }
                __syncwarp();
                if (hl < my_nn) kb[my_ss + rank] = key;
                __syncwarp();
            } else if (narrow && nn <= 32) {
                // pair it with the next bin of 17..32 keys, if any
                const unsigned rest = todo & mid;
                const int src2 = rest ? (__ffs(rest) - 1) : -1;
                if (src2 >= 0 && b0 + src2 < kBins - 1) {
                    todo &= ~(1u << src2);
                    warp_sort_bin_pair(seg, nn, kb + __shfl_sync(kFullMask, s0, src2), __shfl_sync(kFullMask, n, src2),
                                       lane);
                } else {
                    warp_sort_bin<1>(seg, nn, lane);
                }
            } else if (narrow) {
                if (nn <= 64) warp_sort_bin<2>(seg, nn, lane);
                else if (nn <= 128) warp_sort_bin<4>(seg, nn, lane);
                else warp_sort_bin<8>(seg, nn, lane);
            } else {
                if (nn <= 32) warp_sort_desc<1>(seg, nn, lane);
                else if (nn <= 64) warp_sort_desc<2>(seg, nn, lane);
                else if (nn <= 128) warp_sort_desc<4>(seg, nn, lane);
                else warp_sort_desc<8>(seg, nn, lane);
            }
        }
    }
}

// Rows past the first gridDim.x are handed out in order of demand when a
// counter is given: rows differ in cost (nucleus size, the serial sums'
// binade crossings), and a fixed stride leaves the CTAs that drew heavy rows
// finishing last.  A CTA claims its next row one row ahead (claim_next_row at
// the start of iteration `it`, into slot (it + 1) & 1) so that the row's
// logits can be prefetched into L2 while the current row is finished; the
// slot written during an iteration is never the one read at its start.
__device__ __forceinline__ void claim_next_row(const RowLaunch& p, StreamSmem& sm, int row, int it) {
    if (threadIdx.x == 0)
        sm.next_row[(it + 1) & 1] = p.row_counter ? (int)gridDim.x + atomicAdd(p.row_counter, 1) : row + gridDim.x;
}
__device__ __forceinline__ int next_row(StreamSmem& sm, int& it) {
    __syncthreads();  // slot (it + 1) & 1 written
    ++it;
    return sm.next_row[it & 1];
}

// Bulk prefetch of a row's logits into L2 (one instruction; 16-byte aligned
// address, a multiple of 16 bytes).
__device__ __forceinline__ void prefetch_row_l2(const float* src, int V) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"((unsigned)V * 4u) : "memory");
}

__device__ void defer_row_s(const RowLaunch& p, int row) {
    const int k = atomicAdd(p.defer_count, 1);
    p.defer_rows[k] = row;
}

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Eight consecutive floats.  A thread reads its own 128-byte chunk, so a
// warp's load touches 32 lines; as one 32-byte vector (a whole sector) per
// lane the sector is requested once, where two 16-byte loads of the same
// sector issued apart each fetch it from L2 when L1 (small beside four CTAs'
// shared memory) has dropped it in between.
struct F8 {
    float v[8];
};
__device__ __forceinline__ F8 ldg8(const float* p, bool v32) {
    F8 r;
    if (v32) {  // 32-byte aligned
        asm("ld.global.nc.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
            : "=f"(r.v[0]), "=f"(r.v[1]), "=f"(r.v[2]), "=f"(r.v[3]), "=f"(r.v[4]), "=f"(r.v[5]), "=f"(r.v[6]),
              "=f"(r.v[7])
            : "l"(p));
    } else {
        const float4 a = ldg4(p), b = ldg4(p + 4);
        r.v[0] = a.x, r.v[1] = a.y, r.v[2] = a.z, r.v[3] = a.w;
        r.v[4] = b.x, r.v[5] = b.y, r.v[6] = b.z, r.v[7] = b.w;
    }
    return r;
}

// Loads chunk t (32 floats): four 32-byte loads in flight (eight 16-byte
// ones when the rows are only 16-byte aligned or the chunk is partial).
__device__ __forceinline__ void load_chunk(const Ctx& c, int t, float (&a)[kSC]) {
    const int base = t * kSC;
    const int cnt = min(kSC, c.V - base);  // multiple of 4 when > 0
    if (c.v32 && cnt == kSC) {
#pragma unroll
        for (int g = 0; g < kSC / 8; ++g) {
            const F8 x = ldg8(c.src + base + 8 * g, true);
#pragma unroll
            for (int i = 0; i < 8; ++i) a[8 * g + i] = x.v[i];
        }
        return;
    }
#pragma unroll
    for (int g = 0; g < kSC / 4; ++g) {
        float4 q = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (4 * g < cnt) q = ldg4(c.src + base + 4 * g);
        a[4 * g] = q.x;
        a[4 * g + 1] = q.y;
        a[4 * g + 2] = q.z;
        a[4 * g + 3] = q.w;
    }
}


// Counts e in its histogram bin (bin_of) when e >= e_min, without a branch:
// one predicated shared-memory reduction.  A conditional atomicAdd splits the
// unrolled element loop into one basic block per element, so the elements'
// independent exp work cannot be interleaved.  e <= 1 here (d <= 0); NaN
// fails the compare.
__device__ __forceinline__ void hist_count(uint32_t hist_base, float e, float e_min) {
    const uint32_t b = min((uint32_t)((int)kOneTop - (int)(__float_as_uint(e) >> kBinShift)), (uint32_t)(kBins - 1));
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ge.f32 p, %1, %2;\n\t@p red.shared.add.u32 [%0], 1;\n\t}" ::"r"(hist_base + (b << 2)),
        "f"(e), "f"(e_min));
}

// x = l/T for the rows the kernel takes (see the lean-row rule in the kernel).
__device__ __forceinline__ float div_lean(float l, const Ctx& c) {
    const float q = __fmul_rn(l, c.rT);
    const float r = __fmaf_rn(-q, c.T, l);
    return __fmaf_rn(r, c.rT, q);
}

// Pass 2 over one chunk: exact e = exp(l/T - max) of every element (a
// per-element skip of the values the serial sum absorbs costs more in
// divergence than the exp it saves), the chain sums in the primary (v0, v1)
// and alternative (w0, w1) binade, candidate counts in the histogram, and the
// values of kept chunks.  kGeneral: a partial chunk, or a row whose d range
// reaches below the fast exp range.  kAlt: some chunk of the warp has an
// alternative binade (else w0, w1 are left as they are).
template <bool kGeneral, bool kAlt>
__device__ __forceinline__ void pass2_chunk(const float* cp, int cnt, const Ctx& c, StreamSmem& sm, float e_min,
                                            float* keep, float& v0, float& v1, float& w0, float& w1) {
    const uint32_t hbase = smem_addr(sm.hist);
    if (!kGeneral) {
        // whole chunk: 8-float granules, two in flight ahead
        F8 xa = ldg8(cp, c.v32), xb = ldg8(cp + 8, c.v32);
#pragma unroll 1
        for (int g = 0; g < kSC / 8; ++g) {
            F8 xn;
            if (g + 2 < kSC / 8) xn = ldg8(cp + 8 * (g + 2), c.v32);
            F8 a = xa;
            xa = xb;
            xb = xn;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                const float d = __fsub_rn(div_lean(a.v[w], c), c.max_x);
                const float e = xm::exp_normal_range(d, sm.exptab);
                hist_count(hbase, e, e_min);
                a.v[w] = e;
                v0 = __fadd_rn(v0, e);
                v1 = __fadd_rn(v1, e);
                if (kAlt) {
                    w0 = __fadd_rn(w0, e);
                    w1 = __fadd_rn(w1, e);
                }
            }
            if (keep) {
                reinterpret_cast<float4*>(keep)[2 * g] = make_float4(a.v[0], a.v[1], a.v[2], a.v[3]);
                reinterpret_cast<float4*>(keep)[2 * g + 1] = make_float4(a.v[4], a.v[5], a.v[6], a.v[7]);
            }
        }
        return;
    }
    // three granules in flight: rotate qa <- qb <- qc <- load(g + 3)
    float4 qa = make_float4(0.0f, 0.0f, 0.0f, 0.0f), qb = qa, qc = qa;
    if (!kGeneral || 0 < cnt) qa = ldg4(cp);
    if (!kGeneral || 4 < cnt) qb = ldg4(cp + 4);
    if (!kGeneral || 8 < cnt) qc = ldg4(cp + 8);
#pragma unroll 1
    for (int g = 0; g < kSC / 4; ++g) {
        float4 qn = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (4 * (g + 3) < (kGeneral ? cnt : kSC)) qn = ldg4(cp + 4 * (g + 3));
        float a[4] = {qa.x, qa.y, qa.z, qa.w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            float e = 0.0f;
            if (!kGeneral || 4 * g + w < cnt) {
                const float d = __fsub_rn(div_lean(a[w], c), c.max_x);
                e = kGeneral ? xm::exp_f32(d, sm.exptab) : xm::exp_normal_range(d, sm.exptab);
                hist_count(hbase, e, e_min);
            }
            a[w] = e;
            v0 = __fadd_rn(v0, e);
            v1 = __fadd_rn(v1, e);
            if (kAlt) {
                w0 = __fadd_rn(w0, e);
                w1 = __fadd_rn(w1, e);
            }
        }
        if (keep) reinterpret_cast<float4*>(keep)[g] = make_float4(a[0], a[1], a[2], a[3]);
        qa = qb;
        qb = qc;
        qc = qn;
    }
}

__global__ void __launch_bounds__(kST, RS_CTAS_PER_SM) row_stream_kernel(RowLaunch p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    StreamSmem& sm = *reinterpret_cast<StreamSmem*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < xm::kExpTableSize) sm.exptab[tid] = xm::exp_table_entry(tid);
    __syncthreads();
    const int V = p.vocab;
    const int nch = (V + kSC - 1) / kSC;
    // per-CTA L2-resident scratch for nuclei above the on-chip capacity
    unsigned long long* super = p.workspace + (long long)blockIdx.x * p.ws_stride;

    int it = 0;
    for (int row = blockIdx.x; row < p.batch; row = next_row(sm, it)) {
        claim_next_row(p, sm, row, it);
        Ctx c;
        c.src = p.logits + (long long)row * p.ld;
        c.v32 = p.vec32 != 0;
        c.V = V;
        c.nch = nch;
        c.T = p.temperature_rows ? p.temperature_rows[row] : p.temperature;
        const float topp = p.topp_rows ? p.topp_rows[row] : p.topp;
        // sample(): T == 0 (llama2.c:1085); do_sample / sample_debug: T < 1e-6f
        // (llama2_cublas_fp16.cu:1179, llama2_cublas.cu:5089)
        const bool greedy = (c.T == 0.0f) || (p.greedy_eps && c.T < 1e-6f);
        // sample_mult rows (topp outside (0, 1), llama2.c:1098-1100) share the
        // passes and take the cdf walk at the end
        const bool mult = !greedy && (topp <= 0.0f || topp >= 1.0f);

        if (greedy) {
            // first index of the strict max, NaN at index 0 wins (llama2.c:981-992)
            float bv = -INFINITY;
            int bi = 0x7FFFFFFF;
            bool has_nan = false;
            for (int sidx = 0; sidx < kStrips; ++sidx) {
                const int t = sidx * kST + tid;
                if (t >= nch) break;
                float a[kSC];
                load_chunk(c, t, a);
                const int cnt = min(kSC, V - t * kSC);
                if (p.nan_token1) {  // sample_debug's NaN test (padding lanes are 0)
#pragma unroll
                    for (int j = 0; j < kSC; ++j) has_nan |= isnan(a[j]);
                }
                if (p.probs_out) {  // sample() leaves the logits in place when greedy
                    float4* dst = reinterpret_cast<float4*>(p.probs_out + (long long)row * V + t * kSC);
#pragma unroll
                    for (int g = 0; g < kSC / 4; ++g)
                        if (4 * g < cnt) dst[g] = make_float4(a[4 * g], a[4 * g + 1], a[4 * g + 2], a[4 * g + 3]);
                }
#pragma unroll
                for (int j = 0; j < kSC; ++j)
                    if (j < cnt && (a[j] > bv || (a[j] == bv && t * kSC + j < bi))) {
                        bv = a[j];
                        bi = t * kSC + j;
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
                sm.red_a[warp] = bv;
                sm.red_i[warp] = bi;
            }
            const bool nan1 = __syncthreads_or(has_nan) != 0;
            if (tid == 0) {
                for (int w = 1; w < kSW; ++w)
                    if (sm.red_a[w] > bv || (sm.red_a[w] == bv && sm.red_i[w] < bi)) {
                        bv = sm.red_a[w];
                        bi = sm.red_i[w];
                    }
                // a NaN row under sample_debug's rule is token 1 (llama2_cublas.cu:5081-5084)
                p.out_ids[row] = nan1 ? 1 : ((isnan(__ldg(c.src)) || bi == 0x7FFFFFFF) ? 0 : bi);
                if (p.row_flags) p.row_flags[row] = nan1 ? kFlagNan : 0;
            }
            __syncthreads();
            continue;
        }

        // ---- pass 1: max/min of l; per-chunk approximate sum of exp(x - max)
        c.rT = __frcp_rn(c.T);
        c.unit = (c.T == 1.0f);
        const float k2 = c.rT * 1.4426950408889634f;  // log2(e)/T, approximate scale
        float mxl = -INFINITY, mnl = INFINITY, M2loc = -3.4e38f;
        float cm2[kStrips], cs2[kStrips];
        bool has_nan = false;  // any NaN logit, tested only under sample_debug's rule
        const float4* stats = p.stats ? p.stats + (long long)row * p.stats_ld : nullptr;
#pragma unroll
        for (int sidx = 0; sidx < kStrips; ++sidx) {
            const int t = sidx * kST + tid;
            float m2 = -3.4e38f, s2 = 0.0f;
            if (stats) {
                // the same quantities from the classifier GEMM epilogue
                if (p.nan_token1 && t < nch) {
                    float a[kSC];
                    load_chunk(c, t, a);
#pragma unroll
                    for (int j = 0; j < kSC; ++j) has_nan |= isnan(a[j]);
                }
                if (t < nch) {
                    const float4 q = stats[t];
                    mxl = fmaxf(mxl, q.x);
                    mnl = fminf(mnl, q.y);
                    m2 = fmaxf(m2, (k2 > 0.0f ? q.x : q.y) * k2);
                    s2 = q.z;
                }
            } else if (t < nch) {
                float a[kSC];
                load_chunk(c, t, a);  // eight loads in flight
                const int cnt = min(kSC, V - t * kSC);
                if (p.nan_token1) {
#pragma unroll
                    for (int j = 0; j < kSC; ++j) has_nan |= isnan(a[j]);
                }
                if (cnt == kSC) {
                    // max of fl(a*k2) is fl(max(a)*k2) for k2 > 0 (rounding is
                    // monotone), fl(min(a)*k2) for k2 < 0
                    float cmx = -INFINITY, cmn = INFINITY;
#pragma unroll
                    for (int j = 0; j < kSC; ++j) {
                        cmx = fmaxf(cmx, a[j]);
                        cmn = fminf(cmn, a[j]);
                    }
                    mxl = fmaxf(mxl, cmx);
                    mnl = fminf(mnl, cmn);
                    m2 = fmaxf(m2, (k2 > 0.0f ? cmx : cmn) * k2);
#pragma unroll
                    for (int j = 0; j < kSC; ++j) s2 += ex2_approx(__fmaf_rn(a[j], k2, -m2));
                } else {
#pragma unroll
                    for (int j = 0; j < kSC; ++j)
                        if (j < cnt) {
                            mxl = fmaxf(mxl, a[j]);
                            mnl = fminf(mnl, a[j]);
                            m2 = fmaxf(m2, a[j] * k2);
                        }
#pragma unroll
                    for (int j = 0; j < kSC; ++j)
                        if (j < cnt) s2 += ex2_approx(__fmaf_rn(a[j], k2, -m2));
                }
            }
            cm2[sidx] = m2;
            cs2[sidx] = s2;
            M2loc = fmaxf(M2loc, m2);
        }
        float wmx = mxl, wmn = mnl, wm2 = M2loc;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            wmx = fmaxf(wmx, __shfl_xor_sync(kFullMask, wmx, o));
            wmn = fminf(wmn, __shfl_xor_sync(kFullMask, wmn, o));
            wm2 = fmaxf(wm2, __shfl_xor_sync(kFullMask, wm2, o));
        }
        if (lane == 0) {
            sm.red_a[warp] = wmx;
            sm.red_b[warp] = wmn;
            sm.red_c[warp] = wm2;
        }
        if (tid == 0) {
            sm.n_alt = 0;
            sm.n_side = 0;
            sm.flag = 0;
            sm.dbin = -1;
            sm.sort_next = 0;
        }
        for (int b = tid; b < kBins; b += kST) sm.hist[b] = 0;
        __syncthreads();
        float MX = -INFINITY, MN = INFINITY, M2 = -3.4e38f;
#pragma unroll
        for (int w = 0; w < kSW; ++w) {
            MX = fmaxf(MX, sm.red_a[w]);
            MN = fminf(MN, sm.red_b[w]);
            M2 = fmaxf(M2, sm.red_c[w]);
        }
        // red_* are reused by the scans below
        if (__syncthreads_or(has_nan)) {
            // sample_debug (llama2_cublas.cu:5071-5085): token 1, no coin, the
            // buffer keeps the logits
            if (p.probs_out) {
                const float4* src4 = reinterpret_cast<const float4*>(c.src);
                float4* dst4 = reinterpret_cast<float4*>(p.probs_out + (long long)row * V);
                for (int g = tid; g < V / 4; g += kST) dst4[g] = __ldg(src4 + g);
            }
            if (tid == 0) {
                p.out_ids[row] = 1;
                if (p.row_flags) p.row_flags[row] = kFlagNan;
            }
            continue;
        }
        c.max_x = c.unit ? MX : (c.T > 0.0f ? __fdiv_rn(MX, c.T) : __fdiv_rn(MN, c.T));
        // Rows this kernel takes: x = l/T by the unguarded Markstein division,
        // correctly rounded for |T| in [2^-10, 2^10] and |l| in [2^-60, 2^60]
        // (and for l = 0).  A nonzero |l| < 2^-60 gives |x| < 2^-49, below
        // half an ulp of max_x when |max_x| >= 2^-24, so d = fl(x - max_x) =
        // -max_x whatever the quotient's last bits.  Other rows (huge logits,
        // extreme temperatures, a tiny row maximum) go to the general kernel.
        {
            const float aT = fabsf(c.T);
            const bool lean = aT >= 0x1p-10f && aT <= 0x1p10f && fmaxf(fabsf(MX), fabsf(MN)) <= 0x1p60f &&
                              fabsf(c.max_x) >= 0x1p-24f;
            if (!lean) {
                if (tid == 0) defer_row_s(p, row);
                continue;
            }
        }
        // approximate chunk sums in units of exp(x - max); exclusive prefix in
        // chunk order (strip-major)
        float sig[kStrips], gss[kStrips];
        float strip_off = 0.0f;
#pragma unroll
        for (int sidx = 0; sidx < kStrips; ++sidx) {
            sig[sidx] = cs2[sidx] * ex2_approx(cm2[sidx] - M2);
            const ScanF sc = block_scan_f(sig[sidx], sm);
            gss[sidx] = strip_off + sc.excl;
            strip_off += sc.total;
        }
        const float s_approx = strip_off;

        // ---- pass 2: exact e where it matters, chunk functions, histogram
        const float cutoff = __fdiv_rn(__fsub_rn(1.0f, topp), (float)(V - 1));  // llama2.c:1024
        // candidates counted in the histogram: e >= e_min (none for
        // sample_mult rows, whose cutoff would count every element)
        const float e_min = mult ? INFINITY : cutoff * s_approx * 0.9921875f;
        const float d_cand = (e_min > 0.0f) ? __logf(e_min) - 1e-3f : -INFINITY;
        // every d = fl(x - max) lies in [fl(min_x - max_x), 0]: rows whose
        // range stays inside the fast exp range skip the range check
        const float min_x = c.unit ? MN : (c.T > 0.0f ? __fdiv_rn(MN, c.T) : __fdiv_rn(MX, c.T));
        const bool wide = !(__fsub_rn(min_x, c.max_x) >= xm::kExpFastMin);
        // a NaN logit makes the approximate sum NaN (ex2.approx(NaN) = NaN),
        // and the reference's softmax then yields all-NaN probabilities: such
        // rows skip pass 2 (whose fast exp does not carry NaN through)
        const bool nan_row = isnan(s_approx);
        bool nan_any = false;
        // guaranteed nucleus mass the selected candidates must carry: topp plus
        // the fp32 drift bound, against S_approx scaled up by the 2^-7 margin
        // that bounds its distance to the exact serial S
        const float target = (topp + 4096.0f * 0x1p-24f + 1e-5f) * s_approx * 1.0078125f;

#pragma unroll 1
        for (int sidx = 0; sidx < (nan_row ? 0 : kStrips); ++sidx) {
            const int t = sidx * kST + tid;
            const bool valid = t < nch;
            const int cnt = valid ? min(kSC, V - t * kSC) : 0;
            uint32_t alt = 0u;
            const uint32_t eb = valid ? xm::chain_guess_primary(gss[sidx], sig[sidx], alt) : 0u;
            // chunks whose binade is unknown or near a boundary keep their
            // values for a possible serial replay
            float* keep = nullptr;
            int keep_idx = -1;
            if (valid && (eb == 0u || alt != 0u)) {
                keep_idx = atomicAdd(&sm.n_side, 1);
                if (keep_idx < kSideCap) keep = sm.side[keep_idx];
                else keep_idx = -1;
            }
            const float lo = __uint_as_float(eb << 23), lo1 = __uint_as_float((eb << 23) | 1u);
            const float alo = __uint_as_float(alt << 23), alo1 = __uint_as_float((alt << 23) | 1u);
            float v0 = lo, v1 = lo1, w0 = alo, w1 = alo1;
            const float* cp = c.src + t * kSC;
            const bool warp_alt = __any_sync(kFullMask, alt != 0u);
            if (cnt == kSC && !wide) {
                if (warp_alt)
                    pass2_chunk<false, true>(cp, cnt, c, sm, e_min, keep, v0, v1, w0, w1);
                else
                    pass2_chunk<false, false>(cp, cnt, c, sm, e_min, keep, v0, v1, w0, w1);
            } else if (valid) {
                pass2_chunk<true, true>(cp, cnt, c, sm, e_min, keep, v0, v1, w0, w1);
            }
            nan_any |= isnan(v0);
            // chunk functions (primary and alternative binade)
            const bool clean = valid && eb != 0u && (__float_as_uint(v0) >> 23) == eb && (__float_as_uint(v1) >> 23) == eb;
            const bool aclean = valid && alt != 0u && (__float_as_uint(w0) >> 23) == alt && (__float_as_uint(w1) >> 23) == alt;
            const xm::ChainFn f{__fsub_rn(v0, lo), __fsub_rn(v1, lo1),
                                (__float_as_uint(v0) & 1u) | ((__float_as_uint(v1) & 1u) << 1)};
            uint32_t z = (clean ? (f.pbits | kFClean) : 0u) | (valid ? kFValid : 0u);
            if (aclean) {
                const int ai = atomicAdd(&sm.n_alt, 1);
                if (ai < kAltCap) {
                    sm.alt[ai] = make_float4(__fsub_rn(w0, alo), __fsub_rn(w1, alo1),
                                             __uint_as_float((__float_as_uint(w0) & 1u) |
                                                             ((__float_as_uint(w1) & 1u) << 1) | kFClean),
                                             __uint_as_float(alt));
                    z |= kFAlt | ((uint32_t)ai << 8);
                }
            }
            if (keep_idx >= 0) z |= (uint32_t)(keep_idx + 1) << 16;
            // run chunks take the composition to the end of their run; the
            // segment (= warp within the strip) function is lane 0's when all
            // 32 chunks form one run
            const bool runc = valid && clean && !(z & kFAlt);
            const bool runc_n = __shfl_down_sync(kFullMask, (int)runc, 1) != 0;
            const uint32_t eb_n = __shfl_down_sync(kFullMask, eb, 1);
            int run_end = lane;
            const xm::ChainFn F = warp_run_suffix(runc ? f : xm::chain_identity(),
                                                  runc && lane < 31 && runc_n && eb_n == eb, run_end);
            if (runc) z = (z & ~3u) | F.pbits | kFRun | ((uint32_t)run_end << 24);
            if (valid)
                sm.fn[t] = make_float4(runc ? F.L0 : f.L0, runc ? F.L1 : f.L1, __uint_as_float(z), __uint_as_float(eb));
            const uint32_t eb0 = __shfl_sync(kFullMask, eb, 0);
            const bool uni = __all_sync(kFullMask, !valid || (runc && eb == eb0));
            if (lane == 0)
                sm.wfn[sidx * kSW + warp] =
                    make_float4(F.L0, F.L1, __uint_as_float(F.pbits | (uni ? kFClean : 0u)), __uint_as_float(eb0));
        }
        const bool row_nan = (__syncthreads_or(nan_any) != 0) || nan_row;

        // ---- coin (drawn before the walk, llama2.c:1094); state committed at the end
        unsigned long long st = 0;
        float coin = 0.0f;
        if (p.coins) {
            coin = p.coins[row];
        } else {
            st = p.rng_state[row];
            coin = draw_coin(st);
        }
        int flags = 0, id = 0;
        bool defer = false;
        if (mult) {
            if (row_nan) {
                defer = true;  // NaN rows of sample_mult: the general kernel
            } else {
                if (warp == 0) {
                    const float S = resolve_S(sm, c);
                    if (lane == 0) sm.fval = S;
                }
                __syncthreads();
                const float S = sm.fval;
                build_cdf_fns(sm, c, S, gss, sig, p.probs_out ? p.probs_out + (long long)row * V : nullptr);
                if (warp == 0) {
                    const float rS = __frcp_rn(S);
                    float cdf = 0.0f;
                    const int k = walk_fns(sm, V, coin, cdf, [&](int i) { return p_of(c, sm, __ldg(c.src + i), S, rS); });
                    if (lane == 0) sm.result = (k < V) ? k : V - 1;  // llama2.c:1004
                }
                __syncthreads();
                id = sm.result;
            }
        } else if (row_nan) {
            if (p.probs_out) defer = true;  // the general kernel writes the NaN probabilities
            flags = kFlagNan | kFlagNoCand;
        } else {
            int K = 0, D = kBins - 1;
            bool all_cand = false, fits = true;
            unsigned long long* kb = sm.kbuf;
            {
            // ---- nucleus bins from the histogram: guaranteed mass of bins 0..D
            // against the target mass (checked after the walk: a miss defers
            // the row)
            int h[kBinsPerThread];
            int hc = 0;
            float hm = 0.0f;
#pragma unroll
            for (int q = 0; q < kBinsPerThread; ++q) {
                const int b = tid * kBinsPerThread + q;
                h[q] = sm.hist[b];
                hc += h[q];
                hm += (float)h[q] * bin_lo(b);
            }
            const ScanF ms = block_scan_f(hm, sm);
            int ctot;
            const int cex = block_scan_i(hc, sm, ctot) - hc;
            if (ms.incl >= target && ms.excl < target) {
                float m = ms.excl;
                int cc = cex, d = tid * kBinsPerThread + kBinsPerThread - 1;
#pragma unroll
                for (int q = 0; q < kBinsPerThread; ++q) {
                    cc += h[q];
                    m += (float)h[q] * bin_lo(tid * kBinsPerThread + q);
                    if (m >= target) {
                        d = tid * kBinsPerThread + q;
                        break;
                    }
                }
                sm.dbin = d;
                sm.ksel = cc;
            }
            __syncthreads();
            D = sm.dbin;
            K = sm.ksel;
            all_cand = D < 0;
            if (all_cand) {
                D = kBins - 1;
                K = ctot;
            }
            // the nucleus lives on chip, or in the CTA's L2 scratch
            kb = (K <= kKCap) ? sm.kbuf : super;
            // the L2 scratch holds any nucleus (ws_stride >= V + 4096 keys)
            fits = K <= p.ws_stride;
            if (fits) {
                // bin offsets (hist becomes the scatter cursor)
                int run = cex;
#pragma unroll
                for (int q = 0; q < kBinsPerThread; ++q) {
                    const int b = tid * kBinsPerThread + q;
                    if (b <= D) {
                        sm.bstart[b] = (unsigned short)run;
                        sm.hist[b] = run;
                        run += h[q];
                    }
                }
            }
            __syncthreads();
            if (warp == 0) {
                // ---- exact S (overlaps the extraction below)
                const float S = resolve_S(sm, c);
                if (lane == 0) sm.fval = S;
            } else if (fits) {
                // ---- re-read the row (L2) and place the elements of bins
                // 0..D, then sort each bin by (e desc, index asc)
                // Logit-space pre-filter: every element of bins 0..D has
                // e >= e_x = max(lower edge of bin D, e_min), so d >= ln(e_x) -
                // eps; d = fl(fl(l/T) - max) is monotone in l, and l beyond
                // l_lo (T > 0: below; T < 0: above) by a relative 2^-20 plus
                // the absolute 1e-3 margin cannot be one of them.
                const float e_x = fmaxf(bin_lo(D), e_min);
                const float d_x = (e_x > 0.0f) ? __logf(e_x) - 1e-3f : -INFINITY;
                const float tl = __fmul_rn(c.T, __fadd_rn(c.max_x, d_x));
                const float l_lo = (c.T > 0.0f) ? (tl - fabsf(tl) * 0x1p-20f - fabsf(c.T) * 5e-4f)
                                                : (tl + fabsf(tl) * 0x1p-20f + fabsf(c.T) * 5e-4f);
                const float sg = (c.T > 0.0f) ? 1.0f : -1.0f;
                const float l_cmp = sg * l_lo;
                const int u = tid - 32, nu = kST - 32;
                const float4* row4 = reinterpret_cast<const float4*>(c.src);
                const int ng = V / 4;
                for (int g0 = u; g0 < ng; g0 += 4 * nu) {
                    float4 q[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        q[k] = (g0 + k * nu < ng) ? __ldg(row4 + g0 + k * nu)
                                                  : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
                    uint32_t m = 0u;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        m |= (sg * q[k].x < l_cmp) ? 0u : (1u << (4 * k));
                        m |= (sg * q[k].y < l_cmp) ? 0u : (2u << (4 * k));
                        m |= (sg * q[k].z < l_cmp) ? 0u : (4u << (4 * k));
                        m |= (sg * q[k].w < l_cmp) ? 0u : (8u << (4 * k));
                    }
                    // padding (-inf * sg) never passes for T > 0; for T < 0 it
                    // is excluded by the granule bound below
                    // two elements per round: independent chains overlap
                    auto take = [&](int& idx, float& e) {
                        idx = -1;
                        e = 0.0f;
                        if (!m) return;
                        const int j = __ffs(m) - 1;
                        m &= m - 1;
                        const int gi = g0 + (j >> 2) * nu;
                        if (gi < ng) idx = 4 * gi + (j & 3);
                    };
                    while (m) {
                        int i1, i2;
                        float e1, e2;
                        take(i1, e1);
                        take(i2, e2);
                        const float l1 = (i1 >= 0) ? __ldg(c.src + i1) : 0.0f;
                        const float l2 = (i2 >= 0) ? __ldg(c.src + i2) : 0.0f;
                        const float d1 = __fsub_rn(div_lean(l1, c), c.max_x);
                        const float d2 = __fsub_rn(div_lean(l2, c), c.max_x);
                        if (i1 >= 0 && d1 >= d_cand) e1 = xm::exp_f32(d1, sm.exptab);
                        if (i2 >= 0 && d2 >= d_cand) e2 = xm::exp_f32(d2, sm.exptab);
                        if (i1 >= 0 && e1 >= e_min) {
                            const int b = bin_of(e1);
                            if (b <= D) {
                                const int pos = atomicAdd(&sm.hist[b], 1);
                                if (pos < K) kb[pos] = cand_key(e1, i1);
                            }
                        }
                        if (i2 >= 0 && e2 >= e_min) {
                            const int b = bin_of(e2);
                            if (b <= D) {
                                const int pos = atomicAdd(&sm.hist[b], 1);
                                if (pos < K) kb[pos] = cand_key(e2, i2);
                            }
                        }
                    }
                }
                named_bar(1, kST - 32);
                sort_bins(sm, kb, D, K, V);
            }
            __syncthreads();
            }
            // this row is no longer re-read: bring the next one into L2 for
            // its first pass (streamed rows: V % 4 == 0, 16-byte aligned)
            if (tid == 0) {
                const int nr = sm.next_row[(it + 1) & 1];
                if (nr < p.batch) prefetch_row_l2(p.logits + (long long)nr * p.ld, V);
            }
            const float S = sm.fval;
            if (p.probs_out && !(!fits || sm.flag)) {
                // the softmax sample() leaves in the buffer: p = fl(e/S) for
                // every element (V is a multiple of 4 on this kernel)
                const float rS = __frcp_rn(S);
                const float4* src4 = reinterpret_cast<const float4*>(c.src);
                float4* dst4 = reinterpret_cast<float4*>(p.probs_out + (long long)row * V);
                for (int g = tid; g < V / 4; g += kST) {
                    const float4 q = __ldg(src4 + g);
                    dst4[g] = make_float4(p_of(c, sm, q.x, S, rS), p_of(c, sm, q.y, S, rS), p_of(c, sm, q.z, S, rS),
                                          p_of(c, sm, q.w, S, rS));
                }
            }
            if (!fits || sm.flag) {
                defer = true;
            } else {
                // p = fl(e/S) in place of e (Markstein division: correctly
                // rounded for S in [1, 2^15] and e >= 2^-60).  The same pass
                // finds the end of the candidates proper (p >= cutoff form a
                // prefix) from each key's successor, and whether any equal-p
                // run exists.  Four keys per thread in flight.
                const float rS = __frcp_rn(S);
                auto to_p = [&](float e) {
                    const float q = __fmul_rn(e, rS);
                    return __fmaf_rn(__fmaf_rn(-q, S, e), rS, q);
                };
                if (tid == 0) {
                    sm.n0 = 0;
                    sm.n_pairs = 0;
                }
                __syncthreads();
                for (int base = 0; base < K; base += 4 * kST) {  // uniform trip count (barrier inside)
                    const int i0 = base + tid;
                    unsigned long long k[4], kn[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int i = i0 + u * kST;
                        k[u] = (i < K) ? kb[i] : 0ull;
                        kn[u] = (i + 1 < K) ? kb[i + 1] : 0ull;
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int i = i0 + u * kST;
                        if (i < K) {
                            const float pv = to_p(key_prob(k[u]));
                            const bool has_next = i + 1 < K;
                            const float pn = has_next ? to_p(key_prob(kn[u])) : -1.0f;
                            if (pn == pv) {
                                const int q = atomicAdd(&sm.n_pairs, 1);
                                if (q < kPairCap) sm.pairs[q] = i;
                            }
                            if (pv >= cutoff && !(pn >= cutoff)) sm.n0 = i + 1;
                            k[u] = ((unsigned long long)__float_as_uint(pv) << 32) | (k[u] & 0xFFFFFFFFull);
                        }
                    }
                    __syncthreads();  // every key of this round read before any is rewritten
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int i = i0 + u * kST;
                        if (i < K) {
                            kb[i] = k[u];
                            if (kPadP && kb == sm.kbuf) sm.padp[(i >> 5) * (kSC + 1) + (i & 31)] = key_prob(k[u]);
                        }
                    }
                }
                // equal-p runs (sorted by e, so contiguous) go to index order,
                // glibc qsort's order for ties; runs are a few keys, found from
                // the recorded neighbour pairs (all positions if too many)
                __syncthreads();
                const int npairs = sm.n_pairs;
                if (npairs > 0) {
                    const bool listed = npairs <= kPairCap;
                    const int nscan = listed ? npairs : K - 1;
                    for (int q = tid; q < nscan; q += kST) {
                        const int i = listed ? sm.pairs[q] : q;
                        const unsigned long long a = kb[i];
                        if ((a >> 32) == (kb[i + 1] >> 32) && (i == 0 || (kb[i - 1] >> 32) != (a >> 32))) {
                            int j = i + 1;
                            while (j < K && (kb[j] >> 32) == (a >> 32)) ++j;
                            for (int x = i + 1; x < j; ++x) {  // insertion sort by index
                                const unsigned long long kx = kb[x];
                                int y = x - 1;
                                while (y >= i && key_index(kb[y]) > key_index(kx)) {
                                    kb[y + 1] = kb[y];
                                    --y;
                                }
                                kb[y + 1] = kx;
                            }
                        }
                    }
                    __syncthreads();
                }
                const int n0 = sm.n0;
                const bool all_c = all_cand;
                const bool big = n0 > kWalkDirect;
                if (big) build_walk_fns(sm, kb, (kPadP && kb == sm.kbuf) ? sm.padp : nullptr, n0);  // all threads
                if (warp == 0) {
                    int res = -1;
                    if (n0 == 0) {
                        res = all_c ? -2 : -1;
                    } else if (!big) {
                        // llama2.c:1036-1043 as written: one serial fp32 sum,
                        // run in every lane on broadcast reads (no shuffles);
                        // lane 0 records each partial sum.  The chunk table is
                        // free once S is resolved and holds up to 4 * kChunks
                        // sums.
                        // Groups of 8: the adds form one dependent chain (keys
                        // past n0 add +0); the sums only grow, so a group holds
                        // the crossing iff its last sum exceeds topp.
                        float* cdf = reinterpret_cast<float*>(sm.fn);
                        float cum = 0.0f;
                        int last = n0;
                        for (int i0 = 0; i0 < n0; i0 += 8) {
                            float c8[8];
#pragma unroll
                            for (int u = 0; u < 8; ++u) c8[u] = (i0 + u < n0) ? key_prob(kb[i0 + u]) : 0.0f;
#pragma unroll
                            for (int u = 0; u < 8; ++u) {
                                cum = __fadd_rn(cum, c8[u]);
                                c8[u] = cum;
                            }
                            if (lane == 0) {
                                float4* d4 = reinterpret_cast<float4*>(cdf + i0);  // i0 % 8 == 0
                                d4[0] = make_float4(c8[0], c8[1], c8[2], c8[3]);
                                d4[1] = make_float4(c8[4], c8[5], c8[6], c8[7]);
                            }
                            if (c8[7] > topp) {
                                int u = 7;
                                float cu = c8[7];
#pragma unroll
                                for (int v = 6; v >= 0; --v)
                                    if (c8[v] > topp) {
                                        u = v;
                                        cu = c8[v];
                                    }
                                if (i0 + u < n0) {
                                    last = i0 + u;
                                    cum = cu;
                                }
                                break;
                            }
                        }
                        if (last >= n0) last = all_c ? n0 - 1 : -1;  // llama2.c:1037
                        if (last >= 0) {
                            // llama2.c:1046-1055: the second loop adds the same
                            // p's in the same order, so its cdf values are the
                            // recorded sums; the answer is the first i <= last
                            // with r < cdf[i], else last
                            const float r = __fmul_rn(coin, cum);
                            __syncwarp();
                            int k = last;
                            for (int b = 0; b <= last; b += 32) {
                                const int i = b + lane;
                                const unsigned m = __ballot_sync(kFullMask, i <= last && cdf[i] > r);
                                if (m) {
                                    k = b + __ffs(m) - 1;
                                    break;
                                }
                            }
                            res = key_index(kb[k]);
                        }
                    } else {
                        // large nuclei: the same two walks over chunk functions
                        float cum = 0.0f;
                        // llama2.c:1036-1043
                        int last = walk_chunks(sm, kb, n0, topp, cum, sm.ck_s);
                        if (last >= n0) last = all_c ? n0 - 1 : -1;  // llama2.c:1037
                        if (last >= 0) {
                            const float r = __fmul_rn(coin, cum);  // llama2.c:1046
                            // llama2.c:1047-1054 adds the same p's in the same
                            // order as the first walk, so it resumes at the
                            // last segment checkpoint whose sum is <= r (no
                            // earlier cdf can exceed r)
                            __syncwarp();
                            const int seg_last = last / (32 * kSC);
                            const unsigned okm = __ballot_sync(kFullMask, lane <= seg_last && !(sm.ck_s[lane] > r));
                            const int seg0 = 31 - __clz(okm);  // segment 0 (sum 0) always qualifies
                            float s3 = 0.0f;
                            int k = walk_chunks(sm, kb, last + 1, r, s3, nullptr, seg0, sm.ck_s[seg0]);
                            if (k > last) k = last;  // llama2.c:1055
                            res = key_index(kb[k]);
                        }
                    }
                    if (lane == 0) sm.result = res;
                }
                __syncthreads();
                const int res = sm.result;
                if (res == -1) {
                    defer = true;
                } else if (res == -2) {
                    flags |= kFlagNoCand;
                    id = 0;
                } else {
                    id = res;
                }
            }
        }
        if (tid == 0) {
            if (defer) {
                defer_row_s(p, row);
            } else {
                p.out_ids[row] = id;
                if (p.row_flags) p.row_flags[row] = flags;
                if (!p.coins) p.rng_state[row] = st;
            }
        }
        __syncthreads();
    }
}

}  // namespace

size_t smem_bytes() { return sizeof(StreamSmem); }

int launch(const RowLaunch& p, int num_ctas, cudaStream_t stream) {
    static std::atomic<unsigned long long> attr_done{0};
    int dev = 0;
    cudaError_t e0 = cudaGetDevice(&dev);
    if (e0 != cudaSuccess) return -(int)e0;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_done.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(row_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sizeof(StreamSmem));
        if (e != cudaSuccess) return -(int)e;
        attr_done.fetch_or(bit);
    }
    row_stream_kernel<<<num_ctas, kST, sizeof(StreamSmem), stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -(int)e;
}

}  // namespace RS_NS
