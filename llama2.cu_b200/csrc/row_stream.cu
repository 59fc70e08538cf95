// row_stream.cu -- the streaming top-p kernel (the fast path for sample()).
//
// Two CTA shapes, both persistent with one row per CTA at a time.  Batches
// larger than the SM count: four 256-thread CTAs per SM -- while one CTA is
// in a sequential phase (the exact serial-sum resolution, the nucleus walk),
// the other CTAs on the SM keep its pipes and the HBM busy; the row
// (V <= 32768, 1024 chunks of 32) is walked in four strips, thread t owning
// chunk 256s + t of strip s; nuclei of up to 2048 keys stay in shared
// memory, larger ones go to the CTA's L2-resident scratch.  Batches up to
// the SM count (decode): one 1024-thread CTA per SM, one chunk per thread,
// so each row's parallel phases use a whole SM, and nuclei of up to 14336
// keys stay in its shared memory.  Rows past the first wave are handed out
// by a device counter.  A thread's 128-byte chunk is read as 32-byte
// vectors.
//
//   Pass 1 (HBM read): max/min of the logits and, per chunk, an approximate
//     sum of exp(x - max) (ex2.approx) -- used to guess which binade the
//     serial running sum sits in at every chunk, and as S_approx.
//   Pass 2 (the same bytes, now in L2; 8-float granules, two ahead): x = l/T
//     (Markstein division), d = x - max and the exact table-driven exp of
//     every element.  The binade-chain function of the chunk is built on the
//     fly (exact_math.cuh), plus an alternative for the neighbouring binade
//     when the guess lies near a boundary, and each warp composes its chunks
//     into run functions.  Possible top-p candidates (e >= cutoff*S_approx,
//     with margin) are counted in a histogram over the top bits of e.
//   Nucleus bins: the smallest prefix of histogram bins whose guaranteed mass
//     exceeds topp plus the fp32 drift bound, against S_approx scaled up by a
//     2^-7 margin.
//   Then, concurrently: warp 0 turns the run and chunk functions into the
//     exact serial softmax denominator S (chunks that straddle a binade are
//     replayed as 32 serial adds), while the other warps re-read the row from
//     L2, scatter the elements of the nucleus bins in bin order and sort each
//     bin by (e desc, index asc).
//   Walk: p = fl(e/S), equal-p runs put in index order (glibc qsort's
//     order), then the serial cumulative sum to topp and to r = coin*cum:
//     the reference's loop itself for nuclei of up to 1024 keys (the second
//     walk searches the recorded sums), chunk functions for larger ones.  A
//     walk that does not cross topp inside the selected bins (S_approx was
//     off by more than the margin) defers the row.
// sample_mult rows share the passes and the resolution of S, then walk the
// cdf by chunk functions of the exact probabilities.
// Rows this kernel does not finish (extreme temperatures or logits, NaN rows
// of sample_mult, bins of more than 256 keys, walks whose S_approx margin
// failed) are appended to the deferred-row list that the general row kernel
// processes next.
#include "device_common.cuh"
#include "exact_math.cuh"
#include "sampler_kernels.cuh"

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace b2s {

#define RS_THREADS 256
#define RS_CTAS_PER_SM 4
#define RS_SORT_GROUP 32
#define RS_KEY_CAP 2048
#define RS_NS rs256
#include "row_stream_impl.cuh"
#undef RS_NS
#undef RS_KEY_CAP
#undef RS_SORT_GROUP
#undef RS_CTAS_PER_SM
#undef RS_THREADS

#define RS_THREADS 1024
#define RS_CTAS_PER_SM 1
#define RS_SORT_GROUP 8
#define RS_KEY_CAP 14336
#define RS_NS rs1024
#include "row_stream_impl.cuh"
#undef RS_NS
#undef RS_KEY_CAP
#undef RS_SORT_GROUP
#undef RS_CTAS_PER_SM
#undef RS_THREADS

size_t stream_smem_bytes() { return rs256::smem_bytes() > rs1024::smem_bytes() ? rs256::smem_bytes() : rs1024::smem_bytes(); }
int stream_ctas_per_sm() { return 4; }

int launch_row_stream(const RowLaunch& p, int num_sms, cudaStream_t stream) {
    if (p.batch <= num_sms) return rs1024::launch(p, p.batch, stream);
    const int ctas = p.batch < 4 * num_sms ? p.batch : 4 * num_sms;
    return rs256::launch(p, ctas, stream);
}

}  // namespace b2s
