// sampler_kernels.cuh -- launch interface between the C-ABI host code and the
// device kernels of the logits -> token path.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2s {

constexpr int kRowThreads = 1024;      // threads of the row kernel (one CTA per SM)
constexpr int kRowCPT = 32;            // row elements per thread chunk
constexpr int kRowCap = kRowThreads * kRowCPT;  // 32768 floats staged on chip
constexpr int kCandCap = 8192;         // nucleus candidates kept on chip

struct RowLaunch {
    const float* logits;  // [B, ld]
    long long ld;
    int batch;
    int vocab;
    float temperature;            // when temperature_rows == nullptr
    float topp;                   // when topp_rows == nullptr
    const float* temperature_rows;
    const float* topp_rows;
    const float* coins;           // optional given coins
    unsigned long long* rng_state;
    int* out_ids;
    float* probs_out;             // optional [B, vocab]
    int* row_flags;               // optional [B]
    unsigned long long* workspace;  // per-CTA slow-path scratch
    long long ws_stride;          // u64 entries per CTA (power of two >= vocab)
    int probs_in;                 // rows are probabilities
    int force_mode;               // 0: by topp as sample() does, 1: sample_mult, 2: sample_topp
    int greedy_eps;               // rows with temperature < 1e-6f are greedy (do_sample, sample_debug)
    int nan_token1;               // rows holding a NaN logit give token 1, no draw (sample_debug)
    int* error_word;              // device word, set on bounded-wait timeout
    // Failure-detection self-test only (0 otherwise): the first row's staging
    // issues no copy, so its bounded wait runs out after this many polls.
    unsigned wait_test;
    // streaming kernel: next row to take (rows handed out in order of demand
    // past the first gridDim.x); nullptr keeps the fixed stride
    int* row_counter;
    int vec32;  // every row starts on a 32-byte boundary (32-byte chunk loads)
    // deferred rows: the streaming kernel appends rows it leaves to the
    // general kernel; the general kernel then walks row_list[0..*row_count)
    int* defer_count;
    int* defer_rows;
    const int* row_list;
    const int* row_count;
    // optional per-chunk statistics of the rows (max l, min l, approximate
    // sum of exp2(l*k2 - max(l*k2)), unused), written by the classifier GEMM
    // epilogue: the streaming kernel then skips its first pass
    const float4* stats;
    long long stats_ld;  // float4 entries per row
};

// The classifier GEMM of the fused variant: logits[B, V] = H[B, D] . W[V, D]^T
// (bf16 in, fp32 out) plus the per-chunk statistics of each row.
struct GemmLaunch {
    const void* h;   // bf16 [batch, dim], row-major
    const void* w;   // bf16 [vocab, dim], row-major
    int batch;
    int dim;
    int vocab;       // multiple of 32
    float* logits;   // fp32 [batch, ld]
    long long ld;    // multiple of 4
    float4* stats;   // [batch, stats_ld] or nullptr
    long long stats_ld;
    float temperature;
    const float* temperature_rows;
    int* error_word;
    // Final RMSNorm folded into the one- or two-row classifier (GEMV): when
    // x_f32 is set, h is ignored and each CTA forms the bf16 operand
    // bf16(norm_w * (x / rms(x))) of the rows itself, bit-identical to
    // launch_rmsnorm_bf16's output.
    const float* x_f32;   // fp32 [batch, dim] or nullptr
    const float* norm_w;  // fp32 [dim]
};

struct ArgmaxLaunch {
    const float* logits;
    long long ld;
    int batch;
    int vocab;
    int* out_ids;
    float* probs_out;  // optional copy of the rows (sample() leaves logits untouched)
};

// Returns the number of kernels launched (>= 1) or a negative cudaError_t.
int launch_row_sampler(const RowLaunch& p, int num_ctas, cudaStream_t stream);
int launch_argmax(const ArgmaxLaunch& p, cudaStream_t stream);
int launch_seed_states(unsigned long long* st, int batch, unsigned long long seed,
                       long long offset, cudaStream_t stream);
size_t row_kernel_smem_bytes();
size_t stream_smem_bytes();
int stream_ctas_per_sm();
// The streaming kernel over all rows (greedy and top-p rows finish there;
// the rest go to the deferred list); it launches at most
// stream_ctas_per_sm() * num_sms CTAs, each with ws_stride >= vocab u64
// workspace entries.
int launch_row_stream(const RowLaunch& p, int num_sms, cudaStream_t stream);
// Persistent tcgen05 GEMM, one CTA per SM (at most num_sms CTAs).
int launch_classifier_gemm(const GemmLaunch& p, int num_sms, cudaStream_t stream);
// The same GEMM by CTA pairs (tcgen05 cta_group::2, 256 x 256 tiles).
int launch_classifier_gemm_pair(const GemmLaunch& p, int num_sms, cudaStream_t stream);
size_t gemm_smem_bytes();
// Whether launch_classifier_gemm folds the final RMSNorm (x_f32 / norm_w) in:
// the GEMV shapes (one or two rows) with dim up to 16384.
bool gemm_folds_rmsnorm(int batch, int dim);
// Final RMSNorm of `batch` fp32 rows into bf16 (the GEMM's A operand).
int launch_rmsnorm_bf16(const float* x, const float* weight, int batch, int dim, void* out, cudaStream_t stream);
// Embedding rows of the sampled ids (the next decode step's input).
int launch_gather_rows(const float* table, int rows, int dim, const int* ids, int batch, float* out,
                       cudaStream_t stream);

}  // namespace b2s
