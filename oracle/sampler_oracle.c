/*
 * oracle/sampler_oracle.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A CPU restatement of the llama2.c Sampler (logits -> token id), used only as
 * the checker by tests/, by __graft_entry__.smoke() and by bench.py's
 * cpu_baseline leg.  The product path (llama2.cu_b200/csrc) never links,
 * loads or calls anything in this file.
 *
 * Parity pin: there are no golden vectors for the sampler in the reference
 * repository.  This restatement is pinned against the reference's own
 * sampler compiled from its sources (oracle/_ref, built by oracle/Makefile
 * from llama2_cublas_fp16.c:561-670 with -DTESTING); tests/golden holds the
 * ids that build produced and tests/test_oracle.py checks both agree.
 *
 * Every function cites the reference lines whose behaviour it restates
 * (paths are relative to the reference project root).  Scalar semantics that
 * matter for bit-exactness are kept exactly: fp32 `logits /= T` division,
 * max-then-expf-then-serial-sum softmax, `>=` cutoff, strict `>` and `<` in
 * the cumulative loops, the `n-1` / `probindex[last_idx]` fallbacks and
 * glibc qsort with a comparator that returns 0 on ties.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct {
    float prob;
    int index;
} OracleProbIndex; /* same 8-byte layout as ProbIndex, llama2.c:968-971 */

/* xorshift* step, llama2.c:1071-1077 */
unsigned int oracle_random_u32(unsigned long long* state) {
    unsigned long long s = *state;
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    *state = s;
    return (unsigned int)((s * 0x2545F4914F6CDD1Dull) >> 32);
}

/* 24-bit uniform in [0,1), llama2.c:1078-1080 */
float oracle_random_f32(unsigned long long* state) {
    return (oracle_random_u32(state) >> 8) / 16777216.0f;
}

/* first index of the strict maximum, llama2.c:981-992 */
int oracle_argmax(const float* p, int n) {
    int best = 0;
    float best_val = p[0];
    for (int i = 1; i < n; ++i) {
        if (p[i] > best_val) {
            best_val = p[i];
            best = i;
        }
    }
    return best;
}

/* serial fp32 cdf walk, llama2.c:994-1005 */
int oracle_mult(const float* p, int n, float coin) {
    float cdf = 0.0f;
    for (int i = 0; i < n; ++i) {
        cdf += p[i];
        if (coin < cdf) return i;
    }
    return n - 1;
}

/* descending by prob, 0 on ties, llama2.c:1007-1013 */
static int oracle_cmp(const void* a, const void* b) {
    const OracleProbIndex* x = (const OracleProbIndex*)a;
    const OracleProbIndex* y = (const OracleProbIndex*)b;
    if (x->prob > y->prob) return -1;
    if (x->prob < y->prob) return 1;
    return 0;
}

/* Detailed top-p: returns the id and reports the intermediate quantities a
 * test needs to explain a mismatch (n0, last_idx, cumulative, r).
 * Behaviour follows llama2.c:1015-1056.  When n0 == 0 the reference reads
 * probindex[-1] (undefined); here the id is -1 so callers can see it. */
int oracle_topp_detail(const float* p, int n, float topp, OracleProbIndex* pi, float coin,
                       int* n0_out, int* last_out, float* cum_out, float* r_out) {
    const float cutoff = (1.0f - topp) / (n - 1);
    int n0 = 0;
    for (int i = 0; i < n; ++i) {
        if (p[i] >= cutoff) {
            pi[n0].index = i;
            pi[n0].prob = p[i];
            ++n0;
        }
    }
    qsort(pi, n0, sizeof(OracleProbIndex), oracle_cmp);
    float cum = 0.0f;
    int last = n0 - 1;
    for (int i = 0; i < n0; ++i) {
        cum += pi[i].prob;
        if (cum > topp) {
            last = i;
            break;
        }
    }
    const float r = coin * cum;
    if (n0_out) *n0_out = n0;
    if (last_out) *last_out = last;
    if (cum_out) *cum_out = cum;
    if (r_out) *r_out = r;
    if (n0 == 0) return -1;
    float cdf = 0.0f;
    for (int i = 0; i <= last; ++i) {
        cdf += pi[i].prob;
        if (r < cdf) return pi[i].index;
    }
    return pi[last].index;
}

int oracle_topp(const float* p, int n, float topp, OracleProbIndex* pi, float coin) {
    return oracle_topp_detail(p, n, topp, pi, coin, 0, 0, 0, 0);
}

/* max -> expf(x - max) with a serial fp32 sum -> divide, llama2.c:588-606 */
void oracle_softmax(float* x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; ++i)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    for (int i = 0; i < n; ++i) x[i] /= sum;
}

/* Serial fp32 sum of expf(x - max) only (the softmax denominator). */
float oracle_softmax_sum(const float* logits, int n, float temperature) {
    float mx = logits[0] / temperature;
    for (int i = 1; i < n; ++i) {
        float v = logits[i] / temperature;
        if (v > mx) mx = v;
    }
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) sum += expf(logits[i] / temperature - mx);
    return sum;
}

/* One sample() call, llama2.c:1082-1105.  `logits` is overwritten with the
 * probabilities when temperature != 0, exactly as the reference does. */
int oracle_sample(int n, float temperature, float topp, unsigned long long* state, float* logits,
                  OracleProbIndex* scratch) {
    if (temperature == 0.0f) return oracle_argmax(logits, n);
    for (int q = 0; q < n; ++q) logits[q] /= temperature;
    oracle_softmax(logits, n);
    const float coin = oracle_random_f32(state);
    if (topp <= 0 || topp >= 1) return oracle_mult(logits, n, coin);
    return oracle_topp(logits, n, topp, scratch, coin);
}

/* Mode bits of the other per-row calls in the reference's CUDA translation
 * units (the same values as the library's SAMPLER_FLAG_* bits). */
#define ORACLE_GREEDY_BELOW_1E6 2 /* T < 1e-6f is greedy: do_sample, llama2_cublas_fp16.cu:1179;
                                     sample_debug, llama2_cublas.cu:5089 */
#define ORACLE_NAN_TOKEN1 4       /* any NaN logit -> token 1: sample_debug, llama2_cublas.cu:5071-5085 */

/* sample() with the mode bits: mode 6 restates sample_debug
 * (llama2_cublas.cu:5067-5111, whose diagnostic printf calls are left out),
 * mode 2 restates do_sample (llama2_cublas_fp16.cu:1178-1189; its inlined
 * cdf loop is sample_mult's).  The NaN test looks at the logits before any
 * division; such a row returns 1 without drawing a coin or touching the
 * buffer.  The greedy test `T < 1e-6f` takes T == 0 and every negative T. */
int oracle_sample_mode(int n, float temperature, float topp, unsigned long long* state, float* logits,
                       OracleProbIndex* scratch, int mode) {
    if (mode & ORACLE_NAN_TOKEN1) {
        for (int i = 0; i < n; ++i)
            if (isnan(logits[i])) return 1;
    }
    if ((mode & ORACLE_GREEDY_BELOW_1E6) && temperature < 1e-6f) return oracle_argmax(logits, n);
    return oracle_sample(n, temperature, topp, state, logits, scratch);
}

/* ---------------------------------------------------------------------------
 * Batch drivers (the reference has none: they loop its per-row call).
 * ------------------------------------------------------------------------- */

static int clamp_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    return nthreads;
#else
    (void)nthreads;
    return 1;
#endif
}

/* B independent rows; row r uses its own state states[r] (advanced in place),
 * topp from topp_rows[r] when non-NULL.  probs_out (nullable, [B, V]) gets the
 * overwritten logits buffer of each row.  Returns 0. */
int oracle_sample_batch(const float* logits, int B, int V, long long ld, float temperature,
                        float topp, const float* topp_rows, unsigned long long* states,
                        int* ids, float* probs_out, int nthreads) {
    nthreads = clamp_threads(nthreads);
#pragma omp parallel num_threads(nthreads)
    {
        float* row = (float*)malloc((size_t)V * sizeof(float));
        OracleProbIndex* pi = (OracleProbIndex*)malloc((size_t)V * sizeof(OracleProbIndex));
#pragma omp for schedule(dynamic, 4)
        for (int r = 0; r < B; ++r) {
            memcpy(row, logits + (size_t)r * (size_t)ld, (size_t)V * sizeof(float));
            const float tp = topp_rows ? topp_rows[r] : topp;
            ids[r] = oracle_sample(V, temperature, tp, &states[r], row, pi);
            if (probs_out) memcpy(probs_out + (size_t)r * V, row, (size_t)V * sizeof(float));
        }
        free(row);
        free(pi);
    }
    return 0;
}

/* oracle_sample_batch with the mode bits of oracle_sample_mode. */
int oracle_sample_mode_batch(const float* logits, int B, int V, long long ld, float temperature, float topp,
                             const float* topp_rows, unsigned long long* states, int* ids, float* probs_out,
                             int nthreads, int mode) {
    nthreads = clamp_threads(nthreads);
#pragma omp parallel num_threads(nthreads)
    {
        float* row = (float*)malloc((size_t)V * sizeof(float));
        OracleProbIndex* pi = (OracleProbIndex*)malloc((size_t)V * sizeof(OracleProbIndex));
#pragma omp for schedule(dynamic, 4)
        for (int r = 0; r < B; ++r) {
            memcpy(row, logits + (size_t)r * (size_t)ld, (size_t)V * sizeof(float));
            const float tp = topp_rows ? topp_rows[r] : topp;
            ids[r] = oracle_sample_mode(V, temperature, tp, &states[r], row, pi, mode);
            if (probs_out) memcpy(probs_out + (size_t)r * V, row, (size_t)V * sizeof(float));
        }
        free(row);
        free(pi);
    }
    return 0;
}

/* The probabilities-in check: the coin is drawn from states[r] as sample()
 * would, then sample_mult / sample_topp run directly on the given rows. */
int oracle_sample_probs_batch(const float* probs, int B, int V, long long ld, float topp,
                              const float* topp_rows, unsigned long long* states, int* ids,
                              int nthreads) {
    nthreads = clamp_threads(nthreads);
#pragma omp parallel num_threads(nthreads)
    {
        OracleProbIndex* pi = (OracleProbIndex*)malloc((size_t)V * sizeof(OracleProbIndex));
#pragma omp for schedule(dynamic, 4)
        for (int r = 0; r < B; ++r) {
            const float* p = probs + (size_t)r * (size_t)ld;
            const float tp = topp_rows ? topp_rows[r] : topp;
            const float coin = oracle_random_f32(&states[r]);
            ids[r] = (tp <= 0 || tp >= 1) ? oracle_mult(p, V, coin) : oracle_topp(p, V, tp, pi, coin);
        }
        free(pi);
    }
    return 0;
}

/* One sampler advancing over `steps` consecutive rows (the generate loop's
 * pattern, llama2.c:1399-1411). */
int oracle_sample_sequence(const float* logits, int steps, int V, float temperature, float topp,
                           unsigned long long seed, int* ids) {
    float* row = (float*)malloc((size_t)V * sizeof(float));
    OracleProbIndex* pi = (OracleProbIndex*)malloc((size_t)V * sizeof(OracleProbIndex));
    unsigned long long state = seed;
    for (int s = 0; s < steps; ++s) {
        memcpy(row, logits + (size_t)s * V, (size_t)V * sizeof(float));
        ids[s] = oracle_sample(V, temperature, topp, &state, row, pi);
    }
    free(row);
    free(pi);
    return 0;
}

/* Diagnostics for the "mismatch is a boundary coin" rule.  For row r (given
 * the oracle's probabilities p and the coin it drew) returns the smallest
 * distance between the decision value and any cumulative value the reference
 * compares it against: coin vs the mult cdf, or topp vs the nucleus cumsum and
 * r vs the nucleus cdf. */
double oracle_boundary_distance(const float* p, int V, float topp, float coin) {
    double best = INFINITY;
    if (topp <= 0 || topp >= 1) {
        float cdf = 0.0f;
        for (int i = 0; i < V; ++i) {
            cdf += p[i];
            double d = fabs((double)coin - (double)cdf);
            if (d < best) best = d;
            if (cdf > coin + 1e-3f) break;
        }
        return best;
    }
    OracleProbIndex* pi = (OracleProbIndex*)malloc((size_t)V * sizeof(OracleProbIndex));
    int n0 = 0, last = 0;
    float cum = 0.0f, r = 0.0f;
    oracle_topp_detail(p, V, topp, pi, coin, &n0, &last, &cum, &r);
    float c = 0.0f;
    for (int i = 0; i < n0; ++i) {
        c += pi[i].prob;
        double d1 = fabs((double)c - (double)topp);
        double d2 = fabs((double)c - (double)r);
        if (d1 < best) best = d1;
        if (d2 < best) best = d2;
        if (i > last + 1) break;
    }
    free(pi);
    return best;
}
