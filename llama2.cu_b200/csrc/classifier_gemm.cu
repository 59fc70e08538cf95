// classifier_gemm.cu -- the classifier projection of the fused variant:
// logits[B, V] = H[B, D] . Wcls[V, D]^T in bf16 with fp32 accumulation, on
// the 5th-generation tensor cores (tcgen05.mma, accumulator in TMEM), with
// an epilogue that also emits the per-chunk statistics the streaming sampler
// would otherwise compute in its first pass over the logits.
//
// It replaces the reference's classifier matmul followed by the host sampler
// (llama2_cublas.cu:5825-5826 cublasSgemv of wcls, llama2_cublas_bf16.cu:411
// the bf16 GemmEx form), at batch B instead of one token.
//
// Two persistent tensor-core kernels: for batches above 128 rows, CTA pairs
// with 256 x 256 tiles (tcgen05 cta_group::2, described with that kernel
// below); for 3 to 128 rows, one 256-thread CTA per SM with tile 128 (rows of
// H) x 256 (vocabulary entries), K step 64:
//   warp 0     TMA producer: A [128 x 64] and B [256 x 64] bf16 boxes, 128-byte
//              swizzle, into a 4-stage ring (48 KB a stage)
//   warp 1     MMA issuer (one thread): four tcgen05.mma (M128 N256 K16) per
//              stage, tcgen05.commit releases the stage; the accumulator is
//              double-buffered in TMEM (2 x 256 columns)
//   warp 2     TMEM allocation / release
//   warps 4-7  epilogue: tcgen05.ld of 32 columns at a time (one row per
//              thread), fp32 logits to HBM and, per 32-column chunk, the
//              statistics (max, min, approximate sum of exp((l - max)/T))
// One or two rows take a CUDA-core GEMV (below) that streams W at the HBM
// rate.  Every CTA loads its own tiles from this GPU's memory with plain TMA loads
// (the kernels also run on every GPU of a multi-GPU job).  Every mbarrier
// wait is bounded; a timeout sets the error word and drains the pipeline.
#include "device_common.cuh"
#include "sampler_kernels.cuh"

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

namespace b2s {
namespace {

constexpr int kGM = 128;      // rows of H per tile (TMEM lanes)
constexpr int kGN = 256;      // vocabulary entries per tile (TMEM columns)
constexpr int kGK = 64;       // K per stage: 128 bytes of bf16, one swizzle span
constexpr int kStages = 4;
constexpr int kGThreads = 256;
constexpr int kABytes = kGM * kGK * 2;  // 16 KB
constexpr int kBBytes = kGN * kGK * 2;  // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kTmemCols = 2 * kGN;      // two accumulators
constexpr int kGroupM = 16;             // M blocks swept together (L2 reuse of W)

struct GemmSmem {
    uint8_t a[kStages][kABytes];  // 1024-byte aligned (the swizzle atom)
    uint8_t b[kStages][kBBytes];
    unsigned long long full[kStages];
    unsigned long long empty[kStages];
    unsigned long long tmem_full[2];
    unsigned long long tmem_empty[2];
    unsigned long long drain;
    uint32_t tmem_base;
    int abort;
};
constexpr size_t kGemmSmemBytes = sizeof(GemmSmem) + 1024;  // + alignment slack

// ---- tcgen05 wrappers ------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulator)
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives on `bar` once every tcgen05 operation this thread issued so far is done.
__device__ __forceinline__ void tc_commit(unsigned long long* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored as rows of
// 128 bytes with the 128-byte swizzle (the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B): start address >> 4 in bits 0-13, leading
// byte offset (unused for swizzled K-major; 1) in 16-29, stride byte offset
// between 8-row groups (1024 B) >> 4 in 32-45, descriptor version 1 in
// 46-47, swizzle mode 2 (128 B) in 61-63.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), A and
// B bf16 (bits 7-9 = 1, 10-12 = 1), both K-major (bits 15, 16 = 0),
// N >> 3 in bits 17-22, M >> 4 in bits 24-28.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kGN >> 3) << 17) |
                            ((uint32_t)(kGM >> 4) << 24);

__device__ __forceinline__ bool aborted(const GemmSmem& sm) { return *(const volatile int*)&sm.abort != 0; }

__device__ __forceinline__ bool wait_or_abort(unsigned long long* bar, unsigned parity, GemmSmem& sm,
                                              int* error_word) {
    if (mbar_wait_bounded(bar, parity)) return true;
    sm.abort = 1;
    atomicOr(error_word, 2);
    return false;
}

__device__ __forceinline__ void tile_coords(int tile, int mt, int nt, int& m_blk, int& n_blk) {
    const int per_group = kGroupM * nt;
    const int g = tile / per_group;
    const int r = tile - g * per_group;
    const int gm = min(kGroupM, mt - g * kGroupM);  // M blocks in this group
    n_blk = r / gm;
    m_blk = g * kGroupM + (r - n_blk * gm);
}

// Statistics of one 32-column chunk of a row (the streaming sampler's pass 1
// on the same values): max l, min l, and the approximate sum of
// exp2(l*k2 - max(l*k2)) with k2 = log2(e)/T, in column order (0 when T = 0).
__device__ __forceinline__ float4 chunk_stats(const float (&v)[32], float T) {
    float mx = v[0], mn = v[0];
#pragma unroll
    for (int j = 1; j < 32; ++j) {
        mx = fmaxf(mx, v[j]);
        mn = fminf(mn, v[j]);
    }
    float s2 = 0.0f;
    if (T != 0.0f) {
        const float k2 = __frcp_rn(T) * 1.4426950408889634f;
        float m2 = -3.4e38f;
#pragma unroll
        for (int j = 0; j < 32; ++j) m2 = fmaxf(m2, v[j] * k2);
#pragma unroll
        for (int j = 0; j < 32; ++j) s2 += ex2_approx(__fmaf_rn(v[j], k2, -m2));
    }
    return make_float4(mx, mn, s2, 0.0f);
}

// Epilogue of one warp: 256 accumulator columns of this thread's TMEM lane
// (row `row`, vocabulary columns col0 ..), 32 at a time: fp32 logits to HBM
// and, per 32-column chunk, the streaming sampler's pass-1 statistics.
__device__ __forceinline__ void epilogue_rows(const GemmLaunch& p, uint32_t lane_addr, int row, int col0) {
    const bool row_ok = row < p.batch;
    float T = p.temperature;
    if (p.temperature_rows && row_ok) T = p.temperature_rows[row];
#pragma unroll 1
    for (int c = 0; c < kGN / 32; ++c) {
        float v[32];
        tmem_ld32(lane_addr + (uint32_t)(c * 32), v);
        const int col = col0 + c * 32;
        if (row_ok && col < p.vocab) {
            float4* dst = reinterpret_cast<float4*>(p.logits + (long long)row * p.ld + col);
#pragma unroll
            for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            if (p.stats) p.stats[(long long)row * p.stats_ld + col / 32] = chunk_stats(v, T);
        }
    }
}

__global__ void __launch_bounds__(kGThreads, 1)
    classifier_gemm_kernel(const __grid_constant__ CUtensorMap tmap_h, const __grid_constant__ CUtensorMap tmap_w,
                           GemmLaunch p) {
    extern __shared__ __align__(16) unsigned char gsm_raw[];
    GemmSmem& sm = *reinterpret_cast<GemmSmem*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = (p.batch + kGM - 1) / kGM;
    const int nt = (p.vocab + kGN - 1) / kGN;
    const int ntiles = mt * nt;
    const int ksteps = (p.dim + kGK - 1) / kGK;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&sm.tmem_full[a], 1);
            mbar_init(&sm.tmem_empty[a], 4);  // one arrival per epilogue warp
        }
        mbar_init(&sm.drain, 1);
        sm.abort = 0;
        fence_mbar_init();
    }
    if (warp == 2) {
        tmem_alloc(smem_addr(&sm.tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp == 0 && lane == 0) {
        // ---- TMA producer
        int stage = 0;
        unsigned phase = 0;
        for (int tile = blockIdx.x; tile < ntiles && !aborted(sm); tile += gridDim.x) {
            int mb, nb;
            tile_coords(tile, mt, nt, mb, nb);
            for (int k = 0; k < ksteps; ++k) {
                if (!wait_or_abort(&sm.empty[stage], phase ^ 1u, sm, p.error_word)) break;
                mbar_arrive_expect_tx(&sm.full[stage], kStageBytes);
                tma_load_2d(sm.a[stage], &tmap_h, k * kGK, mb * kGM, &sm.full[stage]);
                tma_load_2d(sm.b[stage], &tmap_w, k * kGK, nb * kGN, &sm.full[stage]);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        // drain: every stage this thread filled completes before the CTA exits
        for (int s = 0; s < kStages; ++s) {
            if (!mbar_wait_bounded(&sm.empty[stage], phase ^ 1u)) break;
            if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        int stage = 0;
        unsigned phase = 0;
        int it = 0;
        for (int tile = blockIdx.x; tile < ntiles && !aborted(sm); tile += gridDim.x, ++it) {
            const int acc = it & 1;
            const unsigned acc_phase = (unsigned)(it >> 1) & 1u;
            if (!wait_or_abort(&sm.tmem_empty[acc], acc_phase ^ 1u, sm, p.error_word)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem + (uint32_t)(acc * kGN);
            bool ok = true;
            for (int k = 0; k < ksteps; ++k) {
                if (!wait_or_abort(&sm.full[stage], phase, sm, p.error_word)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_addr(sm.a[stage]), b0 = smem_addr(sm.b[stage]);
#pragma unroll
                for (int kk = 0; kk < kGK / 16; ++kk) {
                    // K advances 16 bf16 = 32 bytes inside the swizzled 128-byte row
                    tc_mma(d_tmem, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32), kIdesc,
                           (k | kk) != 0 ? 1u : 0u);
                }
                tc_commit(&sm.empty[stage]);  // frees the stage when these MMAs are done
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            tc_commit(&sm.tmem_full[acc]);  // accumulator ready
            if (!ok) break;
        }
        // every MMA this thread issued is complete before TMEM is released
        tc_commit(&sm.drain);
        mbar_wait_bounded(&sm.drain, 0);
    } else if (warp >= 4) {
        // ---- epilogue: warp w reads TMEM lanes 32*(w-4) .. +31
        const int q = warp - 4;
        int it = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
            const int acc = it & 1;
            const unsigned acc_phase = (unsigned)(it >> 1) & 1u;
            bool got = false;
            if (lane == 0) got = wait_or_abort(&sm.tmem_full[acc], acc_phase, sm, p.error_word);
            got = __shfl_sync(kFullMask, got ? 1 : 0, 0) != 0;
            if (!got || aborted(sm)) break;
            tc_fence_after();
            int mb, nb;
            tile_coords(tile, mt, nt, mb, nb);
            const int row = mb * kGM + q * 32 + lane;
            epilogue_rows(p, tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kGN), row, nb * kGN);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.tmem_empty[acc]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M256 N256 K16).  Each CTA stages 128 rows of H
// and 128 rows of W per K step (32 KB, half the single-CTA ring's bytes per
// FLOP) and holds the 128 x 256 fp32 accumulator of its rows in its own TMEM,
// double-buffered.  The even CTA issues the MMAs.  Both CTAs' TMA loads
// (.cta_group::2, each into its own CTA's memory) complete on the even CTA's
// stage barrier; the
// even CTA's commits release the stage and hand over the accumulator in both
// CTAs (one commit per CTA, to that CTA's barrier), and every epilogue warp
// of the pair arrives on the even CTA's accumulator-free barrier.
// ---------------------------------------------------------------------------
constexpr int kPM = 256;              // rows of H per pair tile
constexpr int kPN = 256;              // vocabulary entries per pair tile
constexpr int kPHalf = 128;           // rows of each operand staged per CTA
constexpr int kPStages = 6;
constexpr int kPABytes = kPHalf * kGK * 2;  // 16 KB
constexpr int kPBBytes = kPHalf * kGK * 2;  // 16 KB
constexpr int kPGroupM = 16;          // pair M blocks swept together (L2 reuse of W)

struct PairSmem {
    uint8_t a[kPStages][kPABytes];
    uint8_t b[kPStages][kPBBytes];
    unsigned long long full[kPStages];   // even CTA: both halves landed
    unsigned long long empty[kPStages];  // this CTA's stage free
    unsigned long long tmem_full[2];     // this CTA's accumulator ready
    unsigned long long tmem_empty[2];    // even CTA: all eight epilogue warps done
    unsigned long long drain;
    uint32_t tmem_base;
    int abort;
};
constexpr size_t kPairSmemBytes = sizeof(PairSmem) + 1024;

constexpr uint32_t kPairIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPN >> 3) << 17) |
                                ((uint32_t)(kPM >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_mma2(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives on the barrier at `cluster_addr` (this CTA's or the peer's) once the
// pair's tcgen05 operations issued so far by this thread are done.
__device__ __forceinline__ void tc_commit2(uint32_t cluster_addr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
                 : "memory");
}
// TMA load into this CTA's shared memory completing on the even CTA's barrier.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, int x, int y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}

__device__ __forceinline__ bool pair_aborted(const PairSmem& sm) { return *(const volatile int*)&sm.abort != 0; }
__device__ __forceinline__ bool pair_wait(unsigned long long* bar, unsigned parity, PairSmem& sm, int* error_word) {
    if (mbar_wait_bounded(bar, parity)) return true;
    sm.abort = 1;
    atomicOr(error_word, 2);
    return false;
}

__device__ __forceinline__ void pair_tile_coords(int tile, int mt, int nt, int& m_blk, int& n_blk) {
    const int per_group = kPGroupM * nt;
    const int g = tile / per_group;
    const int r = tile - g * per_group;
    const int gm = min(kPGroupM, mt - g * kPGroupM);
    n_blk = r / gm;
    m_blk = g * kPGroupM + (r - n_blk * gm);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGThreads, 1)
    classifier_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_h, const __grid_constant__ CUtensorMap tmap_w,
                                GemmLaunch p) {
    extern __shared__ __align__(16) unsigned char psm_raw[];
    PairSmem& sm = *reinterpret_cast<PairSmem*>((reinterpret_cast<uintptr_t>(psm_raw) + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();
    const bool even = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int mt = (p.batch + kPM - 1) / kPM;
    const int nt = (p.vocab + kPN - 1) / kPN;
    const int ntiles = mt * nt;
    const int ksteps = (p.dim + kGK - 1) / kGK;

    if (tid == 0) {
        for (int s = 0; s < kPStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&sm.tmem_full[a], 1);
            mbar_init(&sm.tmem_empty[a], 8);  // the pair's eight epilogue warps
        }
        mbar_init(&sm.drain, 1);
        sm.abort = 0;
        fence_mbar_init();
    }
    if (warp == 2) {
        tmem_alloc2(smem_addr(&sm.tmem_base), kTmemCols);
        tmem_relinquish2();
    }
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised before any remote use
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp == 0 && lane == 0) {
        // ---- TMA producer (both CTAs): this CTA's halves, completing on the even CTA's barrier
        int stage = 0;
        unsigned phase = 0;
        for (int tile = pair; tile < ntiles && !pair_aborted(sm); tile += npairs) {
            int mb, nb;
            pair_tile_coords(tile, mt, nt, mb, nb);
            for (int k = 0; k < ksteps; ++k) {
                if (!pair_wait(&sm.empty[stage], phase ^ 1u, sm, p.error_word)) break;
                if (even) mbar_arrive_expect_tx(&sm.full[stage], 2 * (kPABytes + kPBBytes));
                const uint32_t fb = map_to_rank(&sm.full[stage], 0);
                tma_load_2d_pair(sm.a[stage], &tmap_h, k * kGK, mb * kPM + (int)rank * kPHalf, fb);
                tma_load_2d_pair(sm.b[stage], &tmap_w, k * kGK, nb * kPN + (int)rank * kPHalf, fb);
                if (++stage == kPStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        // drain: the stages this thread filled are consumed before the CTA exits
        for (int s = 0; s < kPStages; ++s) {
            if (!mbar_wait_bounded(&sm.empty[stage], phase ^ 1u)) break;
            if (++stage == kPStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
    } else if (warp == 1 && lane == 0 && even) {
        // ---- MMA issuer (even CTA)
        int stage = 0;
        unsigned phase = 0;
        int it = 0;
        for (int tile = pair; tile < ntiles && !pair_aborted(sm); tile += npairs, ++it) {
            const int acc = it & 1;
            const unsigned acc_phase = (unsigned)(it >> 1) & 1u;
            if (!pair_wait(&sm.tmem_empty[acc], acc_phase ^ 1u, sm, p.error_word)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem + (uint32_t)(acc * kPN);
            bool ok = true;
            for (int k = 0; k < ksteps; ++k) {
                if (!pair_wait(&sm.full[stage], phase, sm, p.error_word)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_addr(sm.a[stage]), b0 = smem_addr(sm.b[stage]);
#pragma unroll
                for (int kk = 0; kk < kGK / 16; ++kk)
                    tc_mma2(d_tmem, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32), kPairIdesc,
                            (k | kk) != 0 ? 1u : 0u);
                tc_commit2(map_to_rank(&sm.empty[stage], 0));
                tc_commit2(map_to_rank(&sm.empty[stage], 1));
                if (++stage == kPStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            tc_commit2(map_to_rank(&sm.tmem_full[acc], 0));
            tc_commit2(map_to_rank(&sm.tmem_full[acc], 1));
            if (!ok) break;
        }
        tc_commit2(map_to_rank(&sm.drain, 0));
        mbar_wait_bounded(&sm.drain, 0);
    } else if (warp >= 4) {
        // ---- epilogue (both CTAs): warp w reads TMEM lanes 32*(w-4) .. +31 of this CTA
        const int q = warp - 4;
        const uint32_t empty_bar = map_to_rank(&sm.tmem_empty[0], 0);
        int it = 0;
        for (int tile = pair; tile < ntiles; tile += npairs, ++it) {
            const int acc = it & 1;
            const unsigned acc_phase = (unsigned)(it >> 1) & 1u;
            bool got = false;
            if (lane == 0) got = pair_wait(&sm.tmem_full[acc], acc_phase, sm, p.error_word);
            got = __shfl_sync(kFullMask, got ? 1 : 0, 0) != 0;
            if (!got || pair_aborted(sm)) break;
            tc_fence_after();
            int mb, nb;
            pair_tile_coords(tile, mt, nt, mb, nb);
            const int row = mb * kPM + (int)rank * kPHalf + q * 32 + lane;
            epilogue_rows(p, tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * kPN), row, nb * kPN);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) remote_arrive(empty_bar + (uint32_t)(acc * sizeof(unsigned long long)));
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while its peer may still signal its barriers
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc2(tmem, kTmemCols);
    }
}

// ---- decode batches: a bandwidth-bound GEMV -------------------------------------
// With B <= kGemvMaxBatch rows the classifier is a stream of W (V*D*2 bytes,
// 262 MB at 32000 x 4096) with B multiply-adds per element: no operand reuse
// for the tensor cores to exploit, so CUDA cores read W once, with 16-byte
// streaming loads, at the HBM rate (B = 1: about 45 us for 262 MB, against
// about 58 us for the single-CTA tensor-core kernel's 128-row tile).  One CTA
// of kVWarps warps per 32 vocabulary rows (one statistics chunk), all CTAs
// resident at once: warp w takes the 256-element K steps w, w + kVWarps, ..
// of kVRows rows at a time, two steps (2 x kVRows 16-byte loads) in flight
// per lane.  Lane partial sums are reduced across the warp (reduce-scatter,
// then butterfly) and then across the warps in a fixed order; warp 0 writes
// the logits and the chunk statistics exactly as the tensor-core epilogue
// does.
#ifndef B2S_GEMV_MAX_BATCH
#define B2S_GEMV_MAX_BATCH 2
#endif
constexpr int kGemvMaxBatch = B2S_GEMV_MAX_BATCH;
static_assert(kGemvMaxBatch >= 0 && kGemvMaxBatch <= 2, "the GEMV kernel takes up to two rows");
constexpr int kVWarps = 4;
constexpr int kVRows = 4;  // rows of W per pass of a warp

// d = a * b + c for bf16 halves a, b of packed words (fma.rn.f32.bf16: the
// product of two bf16 values is exact in fp32, so this equals the fp32 FMA of
// the widened values).
__device__ __forceinline__ float fma_bf16_lo(uint32_t a2, uint32_t b2, float c) {
    float d;
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, al, bl, %3;\n\t}" : "=f"(d) : "r"(a2), "r"(b2), "f"(c));
    return d;
}
__device__ __forceinline__ float fma_bf16_hi(uint32_t a2, uint32_t b2, float c) {
    float d;
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, ah, bh, %3;\n\t}" : "=f"(d) : "r"(a2), "r"(b2), "f"(c));
    return d;
}

// acc[r][b] += W[row r, 8 elements] . H[b, same 8 elements] for one K step,
// element by element in K order.  H in global memory, or in shared memory
// when the kernel formed it (the folded RMSNorm).
template <int NB, bool kSharedH>
__device__ __forceinline__ void gemv_step(float (&acc)[kVRows][NB], const uint4 (&w)[kVRows], const uint4* h,
                                          long long rs, int batch) {
    uint32_t hq[NB][4];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        const uint4 q = (b < batch) ? (kSharedH ? h[b * rs] : __ldg(h + b * rs)) : make_uint4(0u, 0u, 0u, 0u);
        hq[b][0] = q.x;
        hq[b][1] = q.y;
        hq[b][2] = q.z;
        hq[b][3] = q.w;
    }
#pragma unroll
    for (int r = 0; r < kVRows; ++r) {
        const uint32_t wq[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                acc[r][b] = fma_bf16_lo(wq[e], hq[b][e], acc[r][b]);
                acc[r][b] = fma_bf16_hi(wq[e], hq[b][e], acc[r][b]);
            }
    }
}

constexpr int kNormThreads = 256;  // the RMSNorm kernel's CTA (its summation order)
constexpr int kFoldMaxDim = 16384;  // RMSNorm folded into the GEMV up to this dim

// The bf16 operand rows bf16(w * (r * x)), r = 1/sqrt(mean(x^2) + 1e-5), of
// `nb` fp32 rows into shared memory, by a CTA of kVWarps warps, with the
// arithmetic of rmsnorm_bf16_kernel in the same order: each thread plays the
// kNormThreads/(kVWarps*32) threads of that kernel with its index modulo
// kVWarps*32 (fma over j = t, t + 256, ..), then the same warp and block sums.
template <int NB>
__device__ void fold_rmsnorm_rows(const float* x, const float* w, int dim, int nb, __nv_bfloat16* hs) {
    constexpr int kPlay = kNormThreads / (kVWarps * 32);  // threads of the norm kernel each thread plays
    __shared__ float red[NB][kNormThreads / 32];
    __shared__ float rr[NB];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int b = 0; b < nb; ++b) {
        const float* xr = x + (long long)b * dim;
        float ss[kPlay];
#pragma unroll
        for (int k = 0; k < kPlay; ++k) {
            ss[k] = 0.0f;
            for (int j = tid + k * kVWarps * 32; j < dim; j += kNormThreads) ss[k] = __fmaf_rn(xr[j], xr[j], ss[k]);
#pragma unroll
            for (int o = 16; o; o >>= 1) ss[k] += __shfl_xor_sync(kFullMask, ss[k], o);
            if (lane == 0) red[b][warp + k * kVWarps] = ss[k];
        }
    }
    __syncthreads();
    if (tid < nb) {
        float tot = 0.0f;
#pragma unroll
        for (int i = 0; i < kNormThreads / 32; ++i) tot += red[tid][i];
        rr[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)dim), 1e-5f)));
    }
    __syncthreads();
    for (int b = 0; b < nb; ++b) {
        const float* xr = x + (long long)b * dim;
        const float r = rr[b];
        for (int j = tid; j < dim; j += kVWarps * 32)
            hs[(long long)b * dim + j] = __float2bfloat16_rn(__fmul_rn(w[j], __fmul_rn(r, xr[j])));
    }
    __syncthreads();
}

template <int NB, bool kFold>
__global__ void __launch_bounds__(kVWarps * 32, 8) classifier_gemv_kernel(GemmLaunch p) {
    __shared__ float part[kVWarps][NB][32];
    extern __shared__ __align__(16) unsigned char gemv_dyn[];  // the folded operand rows (kFold)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int v0 = blockIdx.x * 32;
    const long long rs = p.dim >> 3;  // uint4 per row (dim % 8 == 0)
    const int steps = (p.dim + 255) >> 8;
    const uint4* W = reinterpret_cast<const uint4*>(p.w);
    if (kFold) fold_rmsnorm_rows<NB>(p.x_f32, p.norm_w, p.dim, p.batch, reinterpret_cast<__nv_bfloat16*>(gemv_dyn));
    const uint4* H = reinterpret_cast<const uint4*>(kFold ? static_cast<const void*>(gemv_dyn) : p.h) + lane;
    const int b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1;
    float mine[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) mine[b] = 0.0f;
#pragma unroll 1
    for (int g = 0; g < 32 / kVRows; ++g) {
        const uint4* wr = W + (long long)(v0 + g * kVRows) * rs + lane;
        float acc[kVRows][NB];
#pragma unroll
        for (int r = 0; r < kVRows; ++r)
#pragma unroll
            for (int b = 0; b < NB; ++b) acc[r][b] = 0.0f;
#pragma unroll 1
        for (int s = warp; s < steps; s += 2 * kVWarps) {
            const int s2 = s + kVWarps;
            const bool ok1 = s * 32 + lane < rs;
            const bool ok2 = s2 < steps && s2 * 32 + lane < rs;
            uint4 w1[kVRows], w2[kVRows];
#pragma unroll
            for (int r = 0; r < kVRows; ++r) {
                w1[r] = ok1 ? __ldcs(wr + r * rs + s * 32) : make_uint4(0u, 0u, 0u, 0u);
                w2[r] = ok2 ? __ldcs(wr + r * rs + s2 * 32) : make_uint4(0u, 0u, 0u, 0u);
            }
            if (ok1) gemv_step<NB, kFold>(acc, w1, H + s * 32, rs, p.batch);
            if (ok2) gemv_step<NB, kFold>(acc, w2, H + s2 * 32, rs, p.batch);
        }
        // rows r of this pass: lanes with bits (4, 3) = (r >> 1, r & 1) end
        // with the warp's full sum of row r
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            float k0 = b4 ? acc[2][b] : acc[0][b], k1 = b4 ? acc[3][b] : acc[1][b];
            const float x0 = b4 ? acc[0][b] : acc[2][b], x1 = b4 ? acc[1][b] : acc[3][b];
            k0 += __shfl_xor_sync(kFullMask, x0, 16);
            k1 += __shfl_xor_sync(kFullMask, x1, 16);
            float kk = b3 ? k1 : k0;
            kk += __shfl_xor_sync(kFullMask, b3 ? k0 : k1, 8);
            kk += __shfl_xor_sync(kFullMask, kk, 4);
            kk += __shfl_xor_sync(kFullMask, kk, 2);
            kk += __shfl_xor_sync(kFullMask, kk, 1);
            if ((lane & 7) == g) mine[b] = kk;
        }
    }
    const int j = kVRows * (lane & 7) + 2 * b4 + b3;  // the vocabulary row this lane holds
#pragma unroll
    for (int b = 0; b < NB; ++b) part[warp][b][j] = mine[b];
    __syncthreads();
    if (warp != 0) return;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        float v = part[0][b][lane];
#pragma unroll
        for (int w = 1; w < kVWarps; ++w) v = __fadd_rn(v, part[w][b][lane]);
        part[0][b][lane] = v;
        if (b < p.batch) p.logits[(long long)b * p.ld + v0 + lane] = v;
    }
    __syncwarp();
    if (p.stats && lane < NB && lane < p.batch) {
        float v[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = part[0][lane][c];
        const float T = p.temperature_rows ? p.temperature_rows[lane] : p.temperature;
        p.stats[(long long)lane * p.stats_ld + blockIdx.x] = chunk_stats(v, T);
    }
}

// ---- host: tensor maps -------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

// 2-D bf16 K-major tensor [rows, dim] (row stride dim*2 bytes), box [box_rows, 64].
bool make_tmap(CUtensorMap* m, const void* base, int rows, int dim, int box_rows) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)dim, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)dim * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kGK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---- final RMSNorm prologue ---------------------------------------------------
// o = weight * (x * 1/sqrt(mean(x^2) + 1e-5)) per row (the reference's
// rmsnorm, llama2.c:422-433, applied to the final hidden state at
// llama2_cublas.cu:5809-5815), rounded to bf16: the classifier GEMM's A
// operand.  One 256-thread CTA per row; the sum of squares is a tree sum
// (the reference's is serial), so o can differ from the reference's in the
// last bit of the fp32 value before the bf16 rounding.

__global__ void __launch_bounds__(kNormThreads) rmsnorm_bf16_kernel(const float* x, const float* w, int dim,
                                                                    __nv_bfloat16* out) {
    __shared__ float red[kNormThreads / 32];
    const float* xr = x + (long long)blockIdx.x * dim;
    float ss = 0.0f;
    for (int j = threadIdx.x; j < dim; j += kNormThreads) ss = __fmaf_rn(xr[j], xr[j], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(kFullMask, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)dim), 1e-5f)));
    __nv_bfloat16* orow = out + (long long)blockIdx.x * dim;
    for (int j = threadIdx.x; j < dim; j += kNormThreads) orow[j] = __float2bfloat16_rn(__fmul_rn(w[j], __fmul_rn(r, xr[j])));
}

// ---- next-token input: embedding rows of the sampled ids ------------------------
// x[b, :] = table[ids[b], :] (llama2.c:636-637, the first step of the next
// forward), so a decode loop feeds the sampled ids back without a host
// round trip.  One CTA per row, 16-byte copies.
__global__ void __launch_bounds__(256) gather_rows_kernel(const float* table, int rows, int dim, const int* ids,
                                                          float* out) {
    const int b = blockIdx.x;
    const int id = ids[b];
    float* dst = out + (long long)b * dim;
    if (id < 0 || id >= rows) {  // an invalid id gives a zero row
        for (int j = threadIdx.x; j < dim; j += 256) dst[j] = 0.0f;
        return;
    }
    const float* src = table + (long long)id * dim;
    if ((dim & 3) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (int j = threadIdx.x; j < dim / 4; j += 256) d4[j] = __ldg(s4 + j);
    } else {
        for (int j = threadIdx.x; j < dim; j += 256) dst[j] = __ldg(src + j);
    }
}

}  // namespace

int launch_rmsnorm_bf16(const float* x, const float* weight, int batch, int dim, void* out, cudaStream_t stream) {
    rmsnorm_bf16_kernel<<<batch, kNormThreads, 0, stream>>>(x, weight, dim, static_cast<__nv_bfloat16*>(out));
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -(int)e;
}

int launch_gather_rows(const float* table, int rows, int dim, const int* ids, int batch, float* out,
                       cudaStream_t stream) {
    gather_rows_kernel<<<batch, 256, 0, stream>>>(table, rows, dim, ids, out);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -(int)e;
}

size_t gemm_smem_bytes() { return kGemmSmemBytes; }

int launch_classifier_gemm_pair(const GemmLaunch& p, int num_sms, cudaStream_t stream) {
    CUtensorMap th, tw;
    if (!make_tmap(&th, p.h, p.batch, p.dim, kPHalf) || !make_tmap(&tw, p.w, p.vocab, p.dim, kPHalf))
        return -(int)cudaErrorInvalidValue;
    static std::atomic<unsigned long long> attr_done{0};
    int dev = 0;
    cudaError_t e0 = cudaGetDevice(&dev);
    if (e0 != cudaSuccess) return -(int)e0;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_done.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(classifier_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kPairSmemBytes);
        if (e != cudaSuccess) return -(int)e;
        attr_done.fetch_or(bit);
    }
    const int mt = (p.batch + kPM - 1) / kPM, nt = (p.vocab + kPN - 1) / kPN;
    int pairs = num_sms / 2;
    if (pairs > mt * nt) pairs = mt * nt;
    classifier_gemm_pair_kernel<<<2 * pairs, kGThreads, kPairSmemBytes, stream>>>(th, tw, p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -(int)e;
}

bool gemm_folds_rmsnorm(int batch, int dim) { return batch >= 1 && batch <= kGemvMaxBatch && dim <= kFoldMaxDim; }

int launch_classifier_gemv(const GemmLaunch& p, cudaStream_t stream) {
    const bool fold = p.x_f32 != nullptr;
    if (p.batch < 1 || p.batch > kGemvMaxBatch || (p.dim & 7) || (p.vocab & 31) ||
        ((reinterpret_cast<uintptr_t>(fold ? nullptr : p.h) | reinterpret_cast<uintptr_t>(p.w)) & 15) ||
        (fold && (!p.norm_w || p.dim > kFoldMaxDim)))
        return -(int)cudaErrorInvalidValue;
    const int grid = p.vocab / 32;
    const size_t dyn = fold ? (size_t)p.batch * p.dim * 2 : 0;
    if (fold && dyn > 48 * 1024) {  // above the default: opt in once per device and shape
        static std::atomic<unsigned long long> attr_done{0};
        int dev = 0;
        cudaError_t e0 = cudaGetDevice(&dev);
        if (e0 != cudaSuccess) return -(int)e0;
        const unsigned long long bit = 1ull << (dev & 63);
        if (!(attr_done.load() & bit)) {
            const int mx = 2 * kFoldMaxDim * 2;
            cudaError_t e1 = cudaFuncSetAttribute(classifier_gemv_kernel<1, true>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
            cudaError_t e2 = cudaFuncSetAttribute(classifier_gemv_kernel<2, true>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
            if (e1 != cudaSuccess) return -(int)e1;
            if (e2 != cudaSuccess) return -(int)e2;
            attr_done.fetch_or(bit);
        }
    }
    if (p.batch == 1) {
        if (fold) classifier_gemv_kernel<1, true><<<grid, kVWarps * 32, dyn, stream>>>(p);
        else classifier_gemv_kernel<1, false><<<grid, kVWarps * 32, 0, stream>>>(p);
    } else {
        if (fold) classifier_gemv_kernel<2, true><<<grid, kVWarps * 32, dyn, stream>>>(p);
        else classifier_gemv_kernel<2, false><<<grid, kVWarps * 32, 0, stream>>>(p);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -(int)e;
}

int launch_classifier_gemm(const GemmLaunch& p, int num_sms, cudaStream_t stream) {
    if (p.x_f32 && !gemm_folds_rmsnorm(p.batch, p.dim)) return -(int)cudaErrorInvalidValue;
    // One or two rows stream W on CUDA cores.
    if (p.batch <= kGemvMaxBatch) return launch_classifier_gemv(p, stream);
    // Batches of more than one 128-row block use CTA pairs (half the staged
    // bytes per FLOP: 1386 vs 1297 TFLOP/s at 8192 x 4096 x 32000); a single
    // block (decode batches) is faster on single CTAs, whose 125 N tiles
    // spread the W stream over more SMs.
    if (p.batch > kGM) return launch_classifier_gemm_pair(p, num_sms, stream);
    CUtensorMap th, tw;
    if (!make_tmap(&th, p.h, p.batch, p.dim, kGM) || !make_tmap(&tw, p.w, p.vocab, p.dim, kGN))
        return -(int)cudaErrorInvalidValue;
    static std::atomic<unsigned long long> attr_done{0};
    int dev = 0;
    cudaError_t e0 = cudaGetDevice(&dev);
    if (e0 != cudaSuccess) return -(int)e0;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_done.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(classifier_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kGemmSmemBytes);
        if (e != cudaSuccess) return -(int)e;
        attr_done.fetch_or(bit);
    }
    const int mt = (p.batch + kGM - 1) / kGM, nt = (p.vocab + kGN - 1) / kGN;
    int grid = num_sms;
    if (grid > mt * nt) grid = mt * nt;
    classifier_gemm_kernel<<<grid, kGThreads, kGemmSmemBytes, stream>>>(th, tw, p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 1 : -(int)e;
}

}  // namespace b2s
