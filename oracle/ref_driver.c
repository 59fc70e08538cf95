/*
 * oracle/ref_driver.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * Batch drivers around the reference's OWN sampler, linked by oracle/Makefile
 * with the object built from the reference source llama2_cublas_fp16.c
 * (compiled with -DTESTING, which fences its main() at :810-884).  The
 * reference's functions are declared here by the signatures it defines at
 * llama2_cublas_fp16.c:561-670 (identical to llama2.c:968-1105); nothing of
 * the reference is copied.  The result is oracle/_ref/libref_sampler.so,
 * used to pin the restatement in sampler_oracle.c and as the timed CPU
 * baseline ("kind": "reference").  Two more variants of the per-row call
 * come from the reference's CUDA translation units (cut out by line range at
 * build time, see oracle/Makefile): sample_debug (llama2_cublas.cu:5067-5111,
 * linked here as cu_sample_debug) and do_sample (llama2_cublas_fp16.cu:
 * 1178-1189, static there, reached through the fp16cu_do_sample wrapper).
 */
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Interface layouts of the reference, llama2_cublas_fp16.c:564-575. */
typedef struct {
    float prob;
    int index;
} ProbIndex;
typedef struct {
    int vocab_size;
    ProbIndex* probindex;
    float temperature;
    float topp;
    unsigned long long rng_state;
} Sampler;

/* Defined by the reference object this driver is linked with. */
void build_sampler(Sampler* sampler, int vocab_size, float temperature, float topp,
                   unsigned long long rng_seed);
void free_sampler(Sampler* sampler);
int sample(Sampler* sampler, float* logits);
int sample_mult(float* probabilities, int n, float coin);
int sample_topp(float* probabilities, int n, float topp, ProbIndex* probindex, float coin);
float random_f32(unsigned long long* state);
/* The reference's sample_debug (llama2_cublas.cu:5067) under its build-time name. */
int cu_sample_debug(Sampler* sampler, float* logits);
/* The reference's do_sample (llama2_cublas_fp16.cu:1178) through the build-time wrapper. */
int fp16cu_do_sample(Sampler* s, float* logits);

static int clamp_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    return nthreads;
#else
    (void)nthreads;
    return 1;
#endif
}

int ref_num_threads(void) { return clamp_threads(0); }

/* llama2.c sample() over B independent rows: one Sampler per row seeded
 * states[r] (advanced in place), a private copy of each row because sample()
 * overwrites its input.  probs_out (nullable) receives the overwritten rows. */
int ref_sample_batch(const float* logits, int B, int V, long long ld, float temperature, float topp,
                     const float* topp_rows, unsigned long long* states, int* ids,
                     float* probs_out, int nthreads) {
    nthreads = clamp_threads(nthreads);
#pragma omp parallel num_threads(nthreads)
    {
        float* row = (float*)malloc((size_t)V * sizeof(float));
#pragma omp for schedule(dynamic, 4)
        for (int r = 0; r < B; ++r) {
            Sampler s;
            build_sampler(&s, V, temperature, topp_rows ? topp_rows[r] : topp, states[r]);
            memcpy(row, logits + (size_t)r * (size_t)ld, (size_t)V * sizeof(float));
            ids[r] = sample(&s, row);
            states[r] = s.rng_state;
            if (probs_out) memcpy(probs_out + (size_t)r * V, row, (size_t)V * sizeof(float));
            free_sampler(&s);
        }
        free(row);
    }
    return 0;
}

/* The per-row call of another reference translation unit over B rows, as
 * ref_sample_batch does for sample(): mode 6 = sample_debug (NaN guard and
 * greedy below 1e-6), mode 2 = do_sample (greedy below 1e-6).  Returns -1 for
 * any other mode. */
int ref_sample_mode_batch(const float* logits, int B, int V, long long ld, float temperature, float topp,
                          const float* topp_rows, unsigned long long* states, int* ids, float* probs_out,
                          int nthreads, int mode) {
    if (mode != 6 && mode != 2) return -1;
    nthreads = clamp_threads(nthreads);
#pragma omp parallel num_threads(nthreads)
    {
        float* row = (float*)malloc((size_t)V * sizeof(float));
#pragma omp for schedule(dynamic, 4)
        for (int r = 0; r < B; ++r) {
            Sampler s;
            build_sampler(&s, V, temperature, topp_rows ? topp_rows[r] : topp, states[r]);
            memcpy(row, logits + (size_t)r * (size_t)ld, (size_t)V * sizeof(float));
            ids[r] = (mode == 6) ? cu_sample_debug(&s, row) : fp16cu_do_sample(&s, row);
            states[r] = s.rng_state;
            if (probs_out) memcpy(probs_out + (size_t)r * V, row, (size_t)V * sizeof(float));
            free_sampler(&s);
        }
        free(row);
    }
    return 0;
}

/* sample_mult / sample_topp on given probabilities, coin from states[r]. */
int ref_sample_probs_batch(const float* probs, int B, int V, long long ld, float topp,
                           const float* topp_rows, unsigned long long* states, int* ids,
                           int nthreads) {
    nthreads = clamp_threads(nthreads);
#pragma omp parallel num_threads(nthreads)
    {
        float* row = (float*)malloc((size_t)V * sizeof(float));
        ProbIndex* pi = (ProbIndex*)malloc((size_t)V * sizeof(ProbIndex));
#pragma omp for schedule(dynamic, 4)
        for (int r = 0; r < B; ++r) {
            memcpy(row, probs + (size_t)r * (size_t)ld, (size_t)V * sizeof(float));
            const float tp = topp_rows ? topp_rows[r] : topp;
            const float coin = random_f32(&states[r]);
            ids[r] = (tp <= 0 || tp >= 1) ? sample_mult(row, V, coin)
                                          : sample_topp(row, V, tp, pi, coin);
        }
        free(row);
        free(pi);
    }
    return 0;
}

/* One Sampler advancing across `steps` rows, as the generate loop uses it. */
int ref_sample_sequence(const float* logits, int steps, int V, float temperature, float topp,
                        unsigned long long seed, int* ids) {
    Sampler s;
    build_sampler(&s, V, temperature, topp, seed);
    float* row = (float*)malloc((size_t)V * sizeof(float));
    for (int t = 0; t < steps; ++t) {
        memcpy(row, logits + (size_t)t * V, (size_t)V * sizeof(float));
        ids[t] = sample(&s, row);
    }
    free(row);
    free_sampler(&s);
    return 0;
}
