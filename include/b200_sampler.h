/*
 * b200_sampler.h -- C-ABI of the B200 (sm_100a) logits -> token sampler.
 *
 * Part 1 is the llama2.c Sampler surface, kept as a drop-in: the same type
 * layouts, names, arguments and return values as the reference, so code that
 * calls llama2.c's sampler links against libb200_sampler.so unchanged.  The
 * computation runs on the current CUDA device; the host buffers keep their
 * reference meaning (sample() overwrites `logits` with the probabilities when
 * temperature != 0).
 *
 * Part 2 adds what the reference does not have: a batched device entry point
 * over B independent rows with per-row xorshift state, the fused classifier
 * GEMM + sampling entry point, and multi-GPU helpers (row sharding and an
 * optional NCCL gather of the sampled ids).
 *
 * Reference citations are file:line within the reference project.
 * All Part-2 functions return 0 on success or a negative SAMPLER_E* code and
 * never exit the process.
 */
#ifndef B200_SAMPLER_H_
#define B200_SAMPLER_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------
 * Part 1: llama2.c Sampler surface
 * ---------------------------------------------------------------------- */

/* Replaces ProbIndex, llama2.c:968-971 (same 8-byte layout). */
typedef struct {
    float prob;
    int index;
} ProbIndex;

/* Replaces Sampler, llama2.c:973-979 (same layout). */
typedef struct {
    int vocab_size;
    ProbIndex* probindex; /* host scratch, allocated by build_sampler */
    float temperature;
    float topp;
    unsigned long long rng_state;
} Sampler;

/* Replaces build_sampler, llama2.c:1058-1065. */
void build_sampler(Sampler* sampler, int vocab_size, float temperature, float topp,
                   unsigned long long rng_seed);
/* Replaces free_sampler, llama2.c:1067-1069. */
void free_sampler(Sampler* sampler);
/* Replaces random_u32, llama2.c:1071-1077 (xorshift*, host integer math). */
unsigned int random_u32(unsigned long long* state);
/* Replaces random_f32, llama2.c:1078-1080. */
float random_f32(unsigned long long* state);
/* Replaces sample_argmax, llama2.c:981-992.  Host buffer, device compute. */
int sample_argmax(float* probabilities, int n);
/* Replaces sample_mult, llama2.c:994-1005.  Host buffer, device compute. */
int sample_mult(float* probabilities, int n, float coin);
/* Replaces sample_topp, llama2.c:1015-1056.  Host buffer, device compute.
 * `probindex` is accepted for signature compatibility and left untouched
 * (the reference uses it as sort scratch only). */
int sample_topp(float* probabilities, int n, float topp, ProbIndex* probindex, float coin);
/* Replaces sample, llama2.c:1082-1105.  `logits` is a host buffer of
 * vocab_size floats; when temperature != 0 it is overwritten with the
 * softmax probabilities and rng_state advances by one draw, as in the
 * reference.  Returns the token id (or -1 if the device call failed; see
 * sampler_last_error()). */
int sample(Sampler* sampler, float* logits);
/* Replaces sample_debug, llama2_cublas.cu:5067-5111 (the per-token call of
 * that translation unit, :5905): sample() except that a `logits` buffer
 * holding any NaN returns token 1 (no coin drawn, buffer left as it is) and
 * any temperature below 1e-6f (zero and negative ones included) takes the
 * argmax.  Its diagnostic printf lines are not reproduced. */
int sample_debug(Sampler* sampler, float* logits);
/* Replaces do_sample, llama2_cublas_fp16.cu:1178-1189 (static there; the same
 * function is llama2_cublas_bf16.cu:1183 and llama2_cublas_fp16tc.cu:1222):
 * sample() except that any temperature below 1e-6f takes the argmax. */
int do_sample(Sampler* sampler, float* logits);

/* ------------------------------------------------------------------------
 * Part 2: batched device API (no counterpart in the reference; it extends
 * the per-row sample() call above to B rows)
 * ---------------------------------------------------------------------- */

#define SAMPLER_OK 0
#define SAMPLER_E_INVALID (-1)      /* bad argument (null pointer, size, alignment) */
#define SAMPLER_E_UNSUPPORTED (-2)  /* vocab_size above the supported maximum */
#define SAMPLER_E_CUDA (-3)         /* a CUDA runtime call failed */
#define SAMPLER_E_WORKSPACE (-4)    /* caller workspace too small */
#define SAMPLER_E_NCCL (-5)         /* NCCL missing or a NCCL call failed */
#define SAMPLER_E_DEVICE (-6)       /* the device reported a bounded-wait timeout */

/* Row flags written to row_flags[] (when non-NULL). */
#define SAMPLER_ROW_NAN 1          /* NaN reached the softmax: probabilities are NaN */
#define SAMPLER_ROW_NO_CANDIDATE 2 /* top-p found no candidate (reference reads probindex[-1]); id 0 */
#define SAMPLER_ROW_SLOW_PATH 4    /* nucleus exceeded on-chip capacity; global-memory path used */
#define SAMPLER_ROW_SERIAL 8       /* input not a non-negative finite distribution; serial replay */
#define SAMPLER_ROW_TIMEOUT 16     /* a bounded device wait expired; result invalid */

/* Flags for SamplerBatchConfig.flags */
#define SAMPLER_FLAG_PROBS_IN 1 /* rows are probabilities: skip /T and softmax, go straight to
                                   sample_mult / sample_topp (the coin is still drawn) */
#define SAMPLER_FLAG_GREEDY_BELOW_1E6 2 /* a row whose temperature is below 1e-6f (zero and negative
                                           ones included) takes the argmax, as do_sample
                                           (llama2_cublas_fp16.cu:1179) and sample_debug
                                           (llama2_cublas.cu:5089) decide; without the flag only
                                           temperature == 0 does, as sample() (llama2.c:1085) */
#define SAMPLER_FLAG_NAN_TOKEN1 4 /* a row holding any NaN logit gets token 1, draws no coin, leaves
                                     probs_out as the logits and is flagged SAMPLER_ROW_NAN, as
                                     sample_debug does (llama2_cublas.cu:5071-5085) */
/* The per-row rules of the reference's two other per-token calls. */
#define SAMPLER_MODE_DO_SAMPLE SAMPLER_FLAG_GREEDY_BELOW_1E6
#define SAMPLER_MODE_SAMPLE_DEBUG (SAMPLER_FLAG_GREEDY_BELOW_1E6 | SAMPLER_FLAG_NAN_TOKEN1)

/* Largest vocabulary the on-chip row path supports (the row is staged whole
 * in shared memory). */
#define SAMPLER_MAX_VOCAB 32768

typedef struct {
    int vocab_size;    /* V, 2 <= V <= SAMPLER_MAX_VOCAB */
    float temperature; /* used for every row unless temperature_rows != NULL */
    float topp;        /* used for every row unless topp_rows != NULL */
    int flags;         /* SAMPLER_FLAG_* (PROBS_IN does not combine with the other two) */
} SamplerBatchConfig;

/* Bytes of device workspace sampler_batched needs for `batch` rows of
 * `vocab_size` (the global-memory sort scratch of the slow top-p path). */
size_t sampler_workspace_bytes(int batch, int vocab_size);

/* Batched sampling of `batch` rows on the device (all pointers are device
 * pointers; `stream` is a cudaStream_t or NULL for the default stream).
 *   logits           [batch, ld] fp32, row r at logits + r*ld (read only)
 *   temperature_rows [batch] or NULL (then cfg->temperature)
 *   topp_rows        [batch] or NULL (then cfg->topp)
 *   coins            [batch] or NULL: a given coin per row instead of a draw
 *                    from rng_state (rng_state is then neither read nor written)
 *   rng_state        [batch] xorshift states, advanced in place by one draw on
 *                    rows with temperature != 0 (may be NULL when coins given
 *                    or every row is greedy)
 *   out_ids          [batch] int32 token ids
 *   probs_out        [batch, vocab_size] or NULL: the probabilities sample()
 *                    leaves in its buffer (softmax output; logits when greedy)
 *   row_flags        [batch] or NULL: SAMPLER_ROW_* bits per row; the only
 *                    report of a device timeout (SAMPLER_ROW_TIMEOUT, id 0 on
 *                    every unfinished row), since the call does not synchronize
 *   workspace        NULL (library-managed: one workspace per stream, created
 *                    on the stream's first call and kept until the process
 *                    exits, so calls on different streams may overlap) or a
 *                    caller buffer >= sampler_workspace_bytes(), which calls
 *                    that may overlap on the GPU must not share
 * Per row it follows sample() (llama2.c:1082-1105) exactly: greedy when
 * temperature == 0, else /T, softmax, coin, then sample_mult when topp <= 0
 * or topp >= 1, else sample_topp (with SAMPLER_MODE_SAMPLE_DEBUG or
 * SAMPLER_MODE_DO_SAMPLE in cfg->flags: sample_debug's or do_sample's rules
 * instead).  Asynchronous on `stream`. */
int sampler_batched(const SamplerBatchConfig* cfg, const float* logits, int batch, long long ld,
                    const float* temperature_rows, const float* topp_rows, const float* coins,
                    unsigned long long* rng_state, int* out_ids, float* probs_out, int* row_flags,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Same as sampler_batched but every buffer is a HOST buffer; copies to and
 * from the device happen inside (pinned or pageable host memory).  The rows
 * are copied in up to 16 pieces back to back on one stream and sampled on
 * another as each piece lands, so the copies overlap the sampling.
 * rng_state (host) is advanced in place. */
int sampler_batched_host(const SamplerBatchConfig* cfg, const float* logits, int batch,
                         long long ld, const float* topp_rows, unsigned long long* rng_state,
                         int* out_ids);

/* rng_state[r] = rng_seed + row_offset + r for r < batch (device buffer):
 * the per-row seeding rule of the batched API (row r of the global batch is
 * seeded rng_seed + r). */
int sampler_seed_states(unsigned long long* rng_state, int batch, unsigned long long rng_seed,
                        long long row_offset, void* stream);

/* Number of kernel launches the last sampler_batched call on this thread
 * issued (diagnostic; used by the benchmark's launch count). */
int sampler_last_launch_count(void);

/* Human-readable text of the last error on this thread. */
const char* sampler_last_error(void);

/* Fused variant: the classifier projection and the sampling of its rows.
 * Replaces, per decode step, the classifier matmul of the final hidden state
 * (llama2_cublas.cu:5825-5826 cublasSgemv with wcls; the bf16 GemmEx form
 * llama2_cublas_bf16.cu:411) followed by sample() on the host
 * (llama2_cublas.cu:5831-5905), for `batch` rows at once:
 *   logits[b, v] = sum_k hidden[b, k] * wcls[v, k]   (bf16 in, fp32 accumulate)
 * on the sm_100a tensor cores (for one or two rows: a CUDA-core GEMV that
 * streams wcls once), whose epilogue also emits the per-row softmax
 * statistics the sampler needs, then per row exactly what sampler_batched()
 * does on those logits (same ids, states and flags).
 *   hidden     bf16 [batch, dim] row-major (16-byte aligned), dim % 8 == 0
 *   wcls       bf16 [vocab_size, dim] row-major (16-byte aligned)
 *   cfg        vocab_size % 32 == 0, <= SAMPLER_MAX_VOCAB; flags: no PROBS_IN
 *   logits_out fp32 [batch, vocab_size] or NULL (then library-managed)
 * Other arguments as in sampler_batched().  Asynchronous on `stream`.
 * The per-chunk statistics (and the logits when logits_out is NULL) live in
 * buffers the library keeps per stream (created on the stream's first call),
 * so fused calls on different streams may overlap. */
int classifier_sample_fused(const SamplerBatchConfig* cfg, const void* hidden, const void* wcls, int batch,
                            int dim, const float* temperature_rows, const float* topp_rows, const float* coins,
                            unsigned long long* rng_state, int* out_ids, float* logits_out, int* row_flags,
                            void* stream);

/* The classifier projection of classifier_sample_fused() alone:
 * logits_out[b, v] = sum_k hidden[b, k] * wcls[v, k] (bf16 in, fp32 out), the
 * batched replacement of llama2_cublas.cu:5825-5826.  Same layout rules;
 * vocab % 32 == 0 and no upper bound on vocab.  Asynchronous on `stream`. */
int classifier_logits(const void* hidden, const void* wcls, int batch, int dim, int vocab, float* logits_out,
                      void* stream);

/* The final RMSNorm of the last layer's output (llama2.c:422-433 rmsnorm,
 * applied at llama2_cublas.cu:5809-5815) as the classifier's prologue:
 * out_bf16[b, j] = bf16(norm_weight[j] * (x[b, j] / sqrt(mean_j(x[b, :]^2) + 1e-5)))
 * for fp32 x [batch, dim] and norm_weight [dim]; device buffers. */
int rmsnorm_bf16(const float* x, const float* norm_weight, int batch, int dim, void* out_bf16, void* stream);

/* The whole decode step from the last layer's fp32 output: rmsnorm_bf16 into
 * a library-managed buffer, then classifier_sample_fused (same arguments and
 * results).  For one or two rows with dim <= 16384 the normalization is done
 * inside the classifier kernel instead (one launch, no intermediate buffer),
 * with the same bits as the two-launch chain. */
int classifier_rmsnorm_sample_fused(const SamplerBatchConfig* cfg, const float* x, const float* norm_weight,
                                    const void* wcls, int batch, int dim, const float* temperature_rows,
                                    const float* topp_rows, const float* coins, unsigned long long* rng_state,
                                    int* out_ids, float* logits_out, int* row_flags, void* stream);

/* The next decode step's input without a host round trip:
 * out[b, :] = table[ids[b], :] for fp32 table [table_rows, dim] (the token
 * embedding lookup that starts the reference's forward, llama2.c:636-637),
 * ids the device ids a sampler call just wrote; an id outside the table
 * gives a zero row.  Device buffers; asynchronous on `stream`.  With the
 * library's buffers allocated by a first call, a whole decode step
 * (sampler_seed_states / classifier_sample_fused / sampler_gather_rows) can
 * be captured in a CUDA graph: a call captured on a stream that has no
 * library buffers of its own yet (nothing is allocated during a capture)
 * uses those of the last call made outside a capture, so replays of that
 * graph must not overlap calls on that call's stream. */
int sampler_gather_rows(const float* table, int table_rows, int dim, const int* ids, int batch, float* out,
                        void* stream);

/* Failure-detection self-test (no counterpart in the reference): runs the
 * row kernel on one row with its first bounded device wait made to run out
 * after `polls` polls (a barrier that no copy targets, so nothing is left in
 * flight), synchronizes, and reports it as a real timeout is reported:
 * returns SAMPLER_E_DEVICE and sets *row_flag to SAMPLER_ROW_TIMEOUT.  The
 * device stays usable; later calls run normally.  polls in [1, 2^24]. */
int sampler_selftest_wait_timeout(unsigned polls, int* row_flag);

/* Largest vocabulary sampler_batched_noalloc accepts. */
#define SAMPLER_NOALLOC_MAX_VOCAB 32768

/* The batched sampler for callers that cannot allocate device memory (an
 * inference server whose GPU memory belongs to its own arena or caching
 * allocator, or a decode loop that must not let cudaMalloc/cudaFree
 * synchronize the device).  No counterpart in the reference.  Same
 * arguments and per-row semantics as sampler_batched, without the workspace:
 * it allocates nothing (no cudaMalloc/cudaFree, no allocating library call)
 * and uses a fixed 8 MiB + 256 B array compiled into the library, present on
 * every GPU that loads it until the process exits.
 *  - vocab_size above SAMPLER_NOALLOC_MAX_VOCAB: returns SAMPLER_E_UNSUPPORTED.
 *  - The first call on each device looks up that device's copy of the array
 *    (cudaGetSymbolAddress) with the device current; make that first call
 *    before any stream capture.
 *  - Every call shares the array (it keeps the last call's contents), so
 *    calls that overlap on the GPU -- different streams, or threads using the
 *    same device -- race; serialize them.
 *  - Returns status codes only; sampler_last_error() is not updated.
 *  - The call does not synchronize, so a device timeout (a bounded wait that
 *    ran out) is reported only through row_flags: every row the kernel did
 *    not finish gets SAMPLER_ROW_TIMEOUT and id 0.  Callers that need to see
 *    it pass row_flags. */
int sampler_batched_noalloc(const SamplerBatchConfig* cfg, const float* logits, int batch, long long ld,
                            const float* temperature_rows, const float* topp_rows, const float* coins,
                            unsigned long long* rng_state, int* out_ids, float* probs_out, int* row_flags,
                            void* stream);

/* ------------------------------------------------------------------------
 * Multi-GPU helpers (no counterpart in the reference, which is single-GPU:
 * llama2_cublas.cu:6065 calls cudaSetDevice(0)).
 * ---------------------------------------------------------------------- */

/* Contiguous row shard of rank `rank` out of `world` for a global batch:
 * rows [*row_begin, *row_begin + *row_count). */
int sampler_shard_rows(int batch, int world, int rank, int* row_begin, int* row_count);

/* NCCL is loaded at run time (dlopen of libnccl.so.2); these return
 * SAMPLER_E_NCCL when it is absent.  The id is NCCL's 128-byte unique id. */
int sampler_nccl_get_unique_id(void* id128);
int sampler_nccl_comm_init(void** comm, int nranks, const void* id128, int rank);
/* All-gather of equal-sized int32 id shards (rows_per_rank each) into
 * ids_all [nranks * rows_per_rank] on every rank; device buffers. */
int sampler_nccl_allgather_ids(void* comm, const int* ids_local, int rows_per_rank, int* ids_all,
                               void* stream);
int sampler_nccl_comm_destroy(void* comm);

#ifdef __cplusplus
}
#endif

#endif /* B200_SAMPLER_H_ */
