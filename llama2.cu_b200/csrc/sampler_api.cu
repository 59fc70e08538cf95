// sampler_api.cu -- host side of the C-ABI declared in include/b200_sampler.h.
//
// The llama2.c entry points keep the reference's meaning (llama2.c:964-1105)
// and route the per-row work to the device kernels in sampler_kernels.cu.
// There is no CPU implementation of the sampling arithmetic here: if the
// device or the kernels are unavailable, calls fail (-1 / SAMPLER_E_*) with a
// message in sampler_last_error().
#include "../../include/b200_sampler.h"
#include "sampler_kernels.cuh"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>
#include <vector>

namespace {

thread_local std::string g_last_error;
thread_local int g_last_launches = 0;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

#define B2S_CUDA(call)                                                                      \
    do {                                                                                    \
        cudaError_t e_ = (call);                                                            \
        if (e_ != cudaSuccess)                                                              \
            return fail(SAMPLER_E_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));     \
    } while (0)

size_t next_pow2(size_t x) {
    size_t p = 1;
    while (p < x) p <<= 1;
    return p;
}

// Library-managed buffers of one (device, stream): calls on different
// streams never share scratch, so they may overlap on the GPU.
struct StreamBufs {
    cudaStream_t stream = nullptr;
    unsigned long long* workspace = nullptr;  // sampler_batched with workspace == NULL
    size_t workspace_bytes = 0;
    float* flogits = nullptr;  // fused classifier: logits when the caller passes none
    size_t flogits_cap = 0;
    float4* stats = nullptr;   // fused classifier: per-chunk statistics
    size_t stats_cap = 0;
    void* hnorm = nullptr;     // bf16 normalized hidden states
    size_t hnorm_cap = 0;
};

// Per-device state for the library-managed buffers.
struct DeviceCtx {
    // Serializes the host-buffer entry points on this device: they share the
    // staging buffers and streams below (distinct Samplers used from
    // different threads stay independent, as in the reference).
    std::mutex host_mu;
    int device = -1;
    int num_sms = 0;
    cudaStream_t stream = nullptr;   // used by the single-row llama2.c entry points
    cudaStream_t streams[2] = {nullptr, nullptr};  // host-buffer pipeline: [0] copies in, [1] samples
    cudaEvent_t piece_ready[16] = {};               // piece k of the pipeline is on the device
    int* error_word = nullptr;
    // single-row buffers (the llama2.c entry points, serialized by host_mu)
    unsigned long long* host_ws = nullptr;
    size_t host_ws_bytes = 0;
    float* d_row = nullptr;
    float* d_probs = nullptr;
    float* d_coin = nullptr;
    unsigned long long* d_state1 = nullptr;  // the Sampler's state when the device draws
    int* d_id = nullptr;
    int row_cap = 0;
    // host-pipeline buffers (sampler_batched_host, serialized by host_mu)
    unsigned long long* pipe_ws = nullptr;
    size_t pipe_ws_bytes = 0;
    float* d_logits = nullptr;
    size_t logits_cap = 0;
    float* d_topp = nullptr;
    unsigned long long* d_state = nullptr;
    int* d_ids = nullptr;
    int rows_cap = 0;
    // per-stream buffers, created on a stream's first call and kept until exit
    std::vector<StreamBufs*> per_stream;
    StreamBufs* last_eager = nullptr;  // the set the last call outside a stream capture used
};

std::mutex g_mu;
std::vector<DeviceCtx*> g_ctx;

int get_ctx(DeviceCtx** out) {
    int dev = 0;
    B2S_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_mu);
    if ((int)g_ctx.size() <= dev) g_ctx.resize(dev + 1, nullptr);
    if (!g_ctx[dev]) {
        DeviceCtx* c = new DeviceCtx();
        c->device = dev;
        B2S_CUDA(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, dev));
        B2S_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
        B2S_CUDA(cudaStreamCreateWithFlags(&c->streams[0], cudaStreamNonBlocking));
        B2S_CUDA(cudaStreamCreateWithFlags(&c->streams[1], cudaStreamNonBlocking));
        for (cudaEvent_t& e : c->piece_ready) B2S_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        B2S_CUDA(cudaMalloc(&c->error_word, sizeof(int)));
        B2S_CUDA(cudaMemset(c->error_word, 0, sizeof(int)));
        B2S_CUDA(cudaMalloc(&c->d_coin, 4 * sizeof(float)));
        B2S_CUDA(cudaMalloc(&c->d_id, 4 * sizeof(int)));
        B2S_CUDA(cudaMalloc(&c->d_state1, sizeof(unsigned long long)));
        g_ctx[dev] = c;
    }
    *out = g_ctx[dev];
    return SAMPLER_OK;
}

// Grows a library-managed buffer to at least `bytes` (callers hold g_mu).
// cudaFree waits for the device, so work still using the old buffer ends first.
template <class T>
int ensure_buf(T** ptr, size_t* cap, size_t bytes) {
    if (*cap >= bytes) return SAMPLER_OK;
    if (*ptr) cudaFree(*ptr);
    *ptr = nullptr;
    *cap = 0;
    B2S_CUDA(cudaMalloc(reinterpret_cast<void**>(ptr), bytes));
    *cap = bytes;
    return SAMPLER_OK;
}

// The buffers of `stream` on device context c (callers hold g_mu).
StreamBufs* stream_bufs(DeviceCtx* c, cudaStream_t stream) {
    for (StreamBufs* b : c->per_stream)
        if (b->stream == stream) return b;
    StreamBufs* b = new StreamBufs();
    b->stream = stream;
    c->per_stream.push_back(b);
    return b;
}

bool stream_capturing(cudaStream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    return cudaStreamIsCapturing(s, &st) == cudaSuccess && st != cudaStreamCaptureStatusNone;
}

// The set a call on `stream` uses (callers hold g_mu and then grow the member
// they need with ensure_buf, which allocates).  Nothing can be allocated while
// a stream is being captured into a CUDA graph, so a capturing stream whose
// own set is too small (torch captures on a side stream of its own) borrows
// the set of the last call made outside a capture, when that one is large
// enough: the graph's replays then use those buffers.  `fits` tells whether a
// set already holds what the call needs.  Returns nullptr when a capture finds
// no large enough set (make one eager call of the same size first).
template <class Fits>
StreamBufs* bufs_for_call(DeviceCtx* c, cudaStream_t stream, const Fits& fits) {
    StreamBufs* b = stream_bufs(c, stream);
    if (!stream_capturing(stream)) {
        c->last_eager = b;
        return b;
    }
    if (fits(b)) return b;
    if (c->last_eager && fits(c->last_eager)) return c->last_eager;
    return nullptr;
}

int ensure_row(DeviceCtx* c, int V) {
    if (c->row_cap >= V) return SAMPLER_OK;
    if (c->d_row) cudaFree(c->d_row);
    if (c->d_probs) cudaFree(c->d_probs);
    c->d_row = c->d_probs = nullptr;
    c->row_cap = 0;
    B2S_CUDA(cudaMalloc(&c->d_row, (size_t)V * sizeof(float)));
    B2S_CUDA(cudaMalloc(&c->d_probs, (size_t)V * sizeof(float)));
    c->row_cap = V;
    return SAMPLER_OK;
}

int row_ctas(const DeviceCtx* c, int batch) { return batch < c->num_sms ? batch : c->num_sms; }

// Workspace layout: [deferred-row count, row counter (16 B)][deferred rows: batch int32,
// padded to 16 B][general kernel: ctas x pow2(V) u64 sort scratch]
// [streaming kernel: stream_ctas x V u64 candidate lists].
size_t defer_bytes(int batch) { return 16 + (((size_t)batch * sizeof(int) + 15) & ~(size_t)15); }
size_t general_bytes(int ctas, int V) { return (size_t)ctas * next_pow2((size_t)V) * sizeof(unsigned long long); }
// per streaming CTA: the candidate list (<= V keys) and a nucleus spill area
size_t stream_stride(int V) { return (size_t)((V + 1) & ~1) + 4096; }
size_t stream_bytes(int sctas, int V) { return (size_t)sctas * stream_stride(V) * sizeof(unsigned long long); }
int stream_ctas(const DeviceCtx* c, int batch) {
    const int n = c->num_sms * b2s::stream_ctas_per_sm();
    return batch < n ? batch : n;
}
size_t workspace_for(const DeviceCtx* c, int V, int batch) {
    const int ctas = batch < c->num_sms ? batch : c->num_sms;
    return defer_bytes(batch) + general_bytes(ctas, V) + stream_bytes(stream_ctas(c, batch), V);
}

// Rows the streaming kernel can stage with 16-byte vector loads.
bool stream_layout_ok(const float* logits, int V, long long ld) {
    return (V % 4) == 0 && V <= SAMPLER_MAX_VOCAB && (ld % 4) == 0 && ((uintptr_t)logits & 15u) == 0;
}

// Core dispatcher shared by every entry point.  All pointers are device
// pointers.  force_mode: 0 = sample() dispatch by topp, 1 = sample_mult,
// 2 = sample_topp.
int dispatch(const SamplerBatchConfig* cfg, const float* logits, int batch, long long ld,
             const float* temperature_rows, const float* topp_rows, const float* coins,
             unsigned long long* rng_state, int* out_ids, float* probs_out, int* row_flags,
             void* workspace, size_t workspace_bytes, cudaStream_t stream, int force_mode,
             const float4* stats = nullptr, long long stats_ld = 0, bool allow_stream = true) {
    g_last_launches = 0;
    if (!cfg || !logits || !out_ids) return fail(SAMPLER_E_INVALID, "null config, logits or out_ids");
    const int V = cfg->vocab_size;
    if (batch < 0 || V < 1 || ld < V) return fail(SAMPLER_E_INVALID, "bad sizes: batch=%d vocab=%d ld=%lld", batch, V, ld);
    if (V > SAMPLER_MAX_VOCAB)
        return fail(SAMPLER_E_UNSUPPORTED, "vocab_size %d above SAMPLER_MAX_VOCAB %d", V, SAMPLER_MAX_VOCAB);
    if (batch == 0) return SAMPLER_OK;
    const int mode_bits = SAMPLER_FLAG_GREEDY_BELOW_1E6 | SAMPLER_FLAG_NAN_TOKEN1;
    if (cfg->flags & ~(SAMPLER_FLAG_PROBS_IN | mode_bits))
        return fail(SAMPLER_E_INVALID, "unknown bits in flags 0x%x", cfg->flags);
    const bool probs_in = (cfg->flags & SAMPLER_FLAG_PROBS_IN) != 0;
    if (probs_in && (cfg->flags & mode_bits))
        return fail(SAMPLER_E_INVALID, "PROBS_IN does not combine with GREEDY_BELOW_1E6 / NAN_TOKEN1");
    const bool greedy_eps = (cfg->flags & SAMPLER_FLAG_GREEDY_BELOW_1E6) != 0;
    const bool nan_token1 = (cfg->flags & SAMPLER_FLAG_NAN_TOKEN1) != 0;
    // every row greedy: one temperature for the batch at which the row rule takes the argmax
    const bool uniform_greedy = !probs_in && !temperature_rows && force_mode == 0 &&
                                (cfg->temperature == 0.0f || (greedy_eps && cfg->temperature < 1e-6f));
    // the argmax kernel has no NaN test: under NAN_TOKEN1 the row kernels take greedy rows too
    const bool all_greedy = uniform_greedy && !nan_token1;
    if (!uniform_greedy && !coins && !rng_state)
        return fail(SAMPLER_E_INVALID, "rng_state is NULL but rows need a coin");
    DeviceCtx* c = nullptr;
    int rc = get_ctx(&c);
    if (rc) return rc;

    if (all_greedy) {
        b2s::ArgmaxLaunch a{logits, ld, batch, V, out_ids, probs_out};
        const int n = b2s::launch_argmax(a, stream);
        if (n < 0) return fail(SAMPLER_E_CUDA, "argmax launch: %s", cudaGetErrorString((cudaError_t)(-n)));
        if (row_flags) B2S_CUDA(cudaMemsetAsync(row_flags, 0, (size_t)batch * sizeof(int), stream));
        g_last_launches = n + (row_flags ? 1 : 0);
        return SAMPLER_OK;
    }

    const int ctas = row_ctas(c, batch);
    const size_t need = workspace_for(c, V, batch);
    unsigned long long* ws = nullptr;
    if (workspace) {
        if (workspace_bytes < need)
            return fail(SAMPLER_E_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, need);
        if (((uintptr_t)workspace & 15u) != 0) return fail(SAMPLER_E_INVALID, "workspace not 16-byte aligned");
        ws = static_cast<unsigned long long*>(workspace);
    } else {
        std::lock_guard<std::mutex> lk(g_mu);
        StreamBufs* b = bufs_for_call(c, stream, [&](StreamBufs* x) { return x->workspace_bytes >= need; });
        if (!b) return fail(SAMPLER_E_WORKSPACE, "no library workspace of %zu bytes during a stream capture", need);
        rc = ensure_buf(&b->workspace, &b->workspace_bytes, need);
        if (rc) return rc;
        ws = b->workspace;
    }
    char* wsb = reinterpret_cast<char*>(ws);
    int* defer_count = reinterpret_cast<int*>(wsb);
    int* defer_rows = reinterpret_cast<int*>(wsb + 16);
    unsigned long long* general_ws = reinterpret_cast<unsigned long long*>(wsb + defer_bytes(batch));
    unsigned long long* stream_ws =
        reinterpret_cast<unsigned long long*>(wsb + defer_bytes(batch) + general_bytes(ctas, V));
    b2s::RowLaunch p{};
    p.logits = logits;
    p.ld = ld;
    p.batch = batch;
    p.vocab = V;
    p.temperature = cfg->temperature;
    p.topp = cfg->topp;
    p.temperature_rows = temperature_rows;
    p.topp_rows = topp_rows;
    p.coins = coins;
    p.rng_state = rng_state;
    p.out_ids = out_ids;
    p.probs_out = probs_out;
    p.row_flags = row_flags;
    p.workspace = general_ws;
    p.ws_stride = (long long)next_pow2((size_t)V);
    p.probs_in = probs_in ? 1 : 0;
    p.force_mode = force_mode;
    p.greedy_eps = greedy_eps ? 1 : 0;
    p.nan_token1 = nan_token1 ? 1 : 0;
    p.error_word = c->error_word;
    p.defer_count = defer_count;
    p.defer_rows = defer_rows;
    // Fast path: the streaming kernel takes greedy, top-p and sample_mult rows
    // (writing the probabilities when asked) and defers the rest to the
    // general kernel, which then walks the deferred list.  Probabilities in
    // and forced modes use the general kernel for every row.
    const bool streamed = allow_stream && !probs_in && force_mode == 0 && stream_layout_ok(logits, V, ld) &&
                          ((uintptr_t)probs_out & 15u) == 0;
    int launches = 0;
    if (streamed) {
        B2S_CUDA(cudaMemsetAsync(defer_count, 0, 2 * sizeof(int), stream));  // count and row counter
        b2s::RowLaunch q = p;
        q.row_counter = defer_count + 1;
        q.vec32 = (((uintptr_t)logits & 31u) == 0 && (ld % 8) == 0) ? 1 : 0;
        q.workspace = stream_ws;
        q.ws_stride = (long long)stream_stride(V);
        q.stats = stats;
        q.stats_ld = stats_ld;
        const int n = b2s::launch_row_stream(q, c->num_sms, stream);
        if (n < 0) return fail(SAMPLER_E_CUDA, "stream launch: %s", cudaGetErrorString((cudaError_t)(-n)));
        launches += n + 1;
        p.row_list = defer_rows;
        p.row_count = defer_count;
    }
    const int n = b2s::launch_row_sampler(p, ctas, stream);
    if (n < 0) return fail(SAMPLER_E_CUDA, "row sampler launch: %s", cudaGetErrorString((cudaError_t)(-n)));
    g_last_launches = launches + n;
    return SAMPLER_OK;
}

// Reads and clears the device error word after a synchronize.
int check_device_word(DeviceCtx* c) {
    int w = 0;
    B2S_CUDA(cudaMemcpy(&w, c->error_word, sizeof(int), cudaMemcpyDeviceToHost));
    if (w) {
        B2S_CUDA(cudaMemset(c->error_word, 0, sizeof(int)));
        return fail(SAMPLER_E_DEVICE, "a bounded device wait expired");
    }
    return SAMPLER_OK;
}

// One host row through the device: the shared body of the llama2.c
// single-row entry points.  Returns the id or -1.  With `state` (a host
// Sampler state) the device draws the coin when the row rule needs one and
// the state comes back advanced or not, as the reference leaves it;
// `mode_flags` are SAMPLER_FLAG_GREEDY_BELOW_1E6 / SAMPLER_FLAG_NAN_TOKEN1.
int host_row(float* row, int n, float temperature, float topp, const float* coin, int probs_in,
             int force_mode, bool write_back, unsigned long long* state = nullptr, int mode_flags = 0) {
    DeviceCtx* c = nullptr;
    if (get_ctx(&c)) return -1;
    std::lock_guard<std::mutex> host_lock(c->host_mu);
    if (n < 1 || n > SAMPLER_MAX_VOCAB) {
        fail(SAMPLER_E_UNSUPPORTED, "vocab_size %d outside [1, %d]", n, SAMPLER_MAX_VOCAB);
        return -1;
    }
    if (ensure_row(c, n)) return -1;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (ensure_buf(&c->host_ws, &c->host_ws_bytes, workspace_for(c, n, 1))) return -1;
    }
    cudaStream_t s = c->stream;
    if (cudaMemcpyAsync(c->d_row, row, (size_t)n * sizeof(float), cudaMemcpyHostToDevice, s) != cudaSuccess) {
        fail(SAMPLER_E_CUDA, "H2D copy failed");
        return -1;
    }
    if (coin && cudaMemcpyAsync(c->d_coin, coin, sizeof(float), cudaMemcpyHostToDevice, s) != cudaSuccess) {
        fail(SAMPLER_E_CUDA, "H2D coin copy failed");
        return -1;
    }
    if (state && cudaMemcpyAsync(c->d_state1, state, sizeof(*state), cudaMemcpyHostToDevice, s) != cudaSuccess) {
        fail(SAMPLER_E_CUDA, "H2D state copy failed");
        return -1;
    }
    SamplerBatchConfig cfg{n, temperature, topp, (probs_in ? SAMPLER_FLAG_PROBS_IN : 0) | mode_flags};
    // one row with its probabilities: the general kernel's single pass is the
    // lower latency here
    const int rc = dispatch(&cfg, c->d_row, 1, n, nullptr, nullptr, coin ? c->d_coin : nullptr,
                            state ? c->d_state1 : nullptr, c->d_id, write_back ? c->d_probs : nullptr, nullptr,
                            c->host_ws, c->host_ws_bytes, s, force_mode, nullptr, 0, !write_back);
    if (rc) return -1;
    int id = -1;
    if (cudaMemcpyAsync(&id, c->d_id, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) {
        fail(SAMPLER_E_CUDA, "D2H id copy failed");
        return -1;
    }
    unsigned long long st_back = 0;
    if (state && cudaMemcpyAsync(&st_back, c->d_state1, sizeof(st_back), cudaMemcpyDeviceToHost, s) != cudaSuccess) {
        fail(SAMPLER_E_CUDA, "D2H state copy failed");
        return -1;
    }
    if (write_back &&
        cudaMemcpyAsync(row, c->d_probs, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost, s) != cudaSuccess) {
        fail(SAMPLER_E_CUDA, "D2H probabilities copy failed");
        return -1;
    }
    if (cudaStreamSynchronize(s) != cudaSuccess) {
        fail(SAMPLER_E_CUDA, "stream synchronize failed: %s", cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    if (check_device_word(c)) return -1;
    if (state) *state = st_back;
    return id;
}

// ---------------------------------------------------------------------------
// NCCL, loaded at run time
// ---------------------------------------------------------------------------
struct NcclApi {
    bool tried = false;
    void* lib = nullptr;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};
NcclApi g_nccl;
std::mutex g_nccl_mu;

int nccl_load() {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.lib) return SAMPLER_OK;
    if (g_nccl.tried) return fail(SAMPLER_E_NCCL, "libnccl.so.2 could not be loaded");
    g_nccl.tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return fail(SAMPLER_E_NCCL, "dlopen libnccl.so.2: %s", dlerror());
    g_nccl.get_unique_id = (decltype(&ncclGetUniqueId))dlsym(h, "ncclGetUniqueId");
    g_nccl.comm_init_rank = (decltype(&ncclCommInitRank))dlsym(h, "ncclCommInitRank");
    g_nccl.all_gather = (decltype(&ncclAllGather))dlsym(h, "ncclAllGather");
    g_nccl.comm_destroy = (decltype(&ncclCommDestroy))dlsym(h, "ncclCommDestroy");
    g_nccl.error_string = (decltype(&ncclGetErrorString))dlsym(h, "ncclGetErrorString");
    if (!g_nccl.get_unique_id || !g_nccl.comm_init_rank || !g_nccl.all_gather || !g_nccl.comm_destroy)
        return fail(SAMPLER_E_NCCL, "libnccl.so.2 lacks a required symbol");
    g_nccl.lib = h;
    return SAMPLER_OK;
}

int nccl_fail(ncclResult_t r, const char* what) {
    return fail(SAMPLER_E_NCCL, "%s: %s", what, g_nccl.error_string ? g_nccl.error_string(r) : "nccl error");
}

}  // namespace

// ===========================================================================
// Part 1: llama2.c Sampler surface
// ===========================================================================
extern "C" {

void build_sampler(Sampler* sampler, int vocab_size, float temperature, float topp,
                   unsigned long long rng_seed) {
    sampler->vocab_size = vocab_size;
    sampler->temperature = temperature;
    sampler->topp = topp;
    sampler->rng_state = rng_seed;
    // host scratch with the reference's size (llama2.c:1064); the device path
    // does not need it but callers may rely on it existing
    sampler->probindex = (ProbIndex*)malloc((size_t)vocab_size * sizeof(ProbIndex));
}

void free_sampler(Sampler* sampler) {
    free(sampler->probindex);
    sampler->probindex = nullptr;
}

unsigned int random_u32(unsigned long long* state) {
    unsigned long long s = *state;
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    *state = s;
    return (unsigned int)((s * 0x2545F4914F6CDD1Dull) >> 32);
}

float random_f32(unsigned long long* state) { return (random_u32(state) >> 8) / 16777216.0f; }

int sample_debug(Sampler* sampler, float* logits) {
    // Whether the coin is drawn depends on the NaN test, so the device draws
    // it from a copy of the state (llama2_cublas.cu:5071-5100).  A greedy
    // row (T < 1e-6f) and a NaN row leave the buffer as it is.
    const bool greedy = sampler->temperature < 1e-6f;
    return host_row(logits, sampler->vocab_size, sampler->temperature, sampler->topp, nullptr, 0, 0, !greedy,
                    &sampler->rng_state, SAMPLER_MODE_SAMPLE_DEBUG);
}

int do_sample(Sampler* sampler, float* logits) {
    // llama2_cublas_fp16.cu:1179: any temperature below 1e-6f is greedy
    if (sampler->temperature < 1e-6f)
        return host_row(logits, sampler->vocab_size, 0.0f, sampler->topp, nullptr, 0, 0, false);
    const float coin = random_f32(&sampler->rng_state);
    return host_row(logits, sampler->vocab_size, sampler->temperature, sampler->topp, &coin, 0, 0, true);
}

int sample_argmax(float* probabilities, int n) {
    return host_row(probabilities, n, 0.0f, 0.0f, nullptr, 0, 0, false);
}

int sample_mult(float* probabilities, int n, float coin) {
    return host_row(probabilities, n, 1.0f, 1.0f, &coin, 1, 1, false);
}

int sample_topp(float* probabilities, int n, float topp, ProbIndex* probindex, float coin) {
    (void)probindex;
    return host_row(probabilities, n, 1.0f, topp, &coin, 1, 2, false);
}

int sample(Sampler* sampler, float* logits) {
    if (sampler->temperature == 0.0f)
        return host_row(logits, sampler->vocab_size, 0.0f, sampler->topp, nullptr, 0, 0, false);
    // The coin comes from the Sampler's own state exactly as llama2.c:1094
    // draws it (host integer arithmetic), then the device does the rest.
    const float coin = random_f32(&sampler->rng_state);
    return host_row(logits, sampler->vocab_size, sampler->temperature, sampler->topp, &coin, 0, 0, true);
}

// ===========================================================================
// Part 2: batched API
// ===========================================================================
size_t sampler_workspace_bytes(int batch, int vocab_size) {
    DeviceCtx* c = nullptr;
    if (get_ctx(&c) != SAMPLER_OK || !c) return 0;
    return workspace_for(c, vocab_size < 1 ? 1 : vocab_size, batch < 1 ? 1 : batch);
}

int sampler_batched(const SamplerBatchConfig* cfg, const float* logits, int batch, long long ld,
                    const float* temperature_rows, const float* topp_rows, const float* coins,
                    unsigned long long* rng_state, int* out_ids, float* probs_out, int* row_flags,
                    void* workspace, size_t workspace_bytes, void* stream) {
    return dispatch(cfg, logits, batch, ld, temperature_rows, topp_rows, coins, rng_state, out_ids, probs_out,
                    row_flags, workspace, workspace_bytes, (cudaStream_t)stream, 0);
}

}  // extern "C"

namespace {
// The fused call: classifier GEMM (tcgen05) with the statistics epilogue,
// then the streaming sampler fed by those statistics.  With x_f32 (one or two
// rows), the final RMSNorm of x is folded into the classifier kernel and
// `hidden` is not used.
int fused_call(const SamplerBatchConfig* cfg, const void* hidden, const float* x_f32, const float* norm_w,
               const void* wcls, int batch, int dim, const float* temperature_rows, const float* topp_rows,
               const float* coins, unsigned long long* rng_state, int* out_ids, float* logits_out, int* row_flags,
               void* stream) {
    g_last_launches = 0;
    if (!cfg || !(hidden || x_f32) || !wcls || !out_ids)
        return fail(SAMPLER_E_INVALID, "null config, hidden, wcls or out_ids");
    const int V = cfg->vocab_size;
    if (batch < 0 || dim < 8 || (dim % 8) != 0 || V < 32 || (V % 32) != 0)
        return fail(SAMPLER_E_INVALID, "bad sizes: batch=%d dim=%d (multiple of 8) vocab=%d (multiple of 32)", batch,
                    dim, V);
    if (V > SAMPLER_MAX_VOCAB)
        return fail(SAMPLER_E_UNSUPPORTED, "vocab_size %d above SAMPLER_MAX_VOCAB %d", V, SAMPLER_MAX_VOCAB);
    if (cfg->flags & SAMPLER_FLAG_PROBS_IN) return fail(SAMPLER_E_INVALID, "PROBS_IN does not apply to the fused call");
    if (((uintptr_t)hidden & 15u) || ((uintptr_t)wcls & 15u) || ((uintptr_t)logits_out & 15u))
        return fail(SAMPLER_E_INVALID, "hidden, wcls and logits_out must be 16-byte aligned");
    if (batch == 0) return SAMPLER_OK;
    if (x_f32 && (!norm_w || !b2s::gemm_folds_rmsnorm(batch, dim)))
        return fail(SAMPLER_E_INVALID, "the folded RMSNorm takes one or two rows of dim <= 16384");
    DeviceCtx* c = nullptr;
    int rc = get_ctx(&c);
    if (rc) return rc;
    const size_t nlog = (size_t)batch * (size_t)V;
    const long long sld = V / 32;
    const size_t nst = (size_t)batch * (size_t)sld;
    float* logits = logits_out;
    float4* stats = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        StreamBufs* b = bufs_for_call(c, (cudaStream_t)stream, [&](StreamBufs* x) {
            return x->stats_cap >= nst * sizeof(float4) && (logits || x->flogits_cap >= nlog * sizeof(float));
        });
        if (!b) return fail(SAMPLER_E_WORKSPACE, "no library buffers for %d rows during a stream capture", batch);
        if (!logits) {
            rc = ensure_buf(&b->flogits, &b->flogits_cap, nlog * sizeof(float));
            if (rc) return rc;
            logits = b->flogits;
        }
        rc = ensure_buf(&b->stats, &b->stats_cap, nst * sizeof(float4));
        if (rc) return rc;
        stats = b->stats;
    }
    b2s::GemmLaunch g{};
    g.h = hidden;
    g.w = wcls;
    g.batch = batch;
    g.dim = dim;
    g.vocab = V;
    g.logits = logits;
    g.ld = V;
    g.stats = stats;
    g.stats_ld = sld;
    g.temperature = cfg->temperature;
    g.temperature_rows = temperature_rows;
    g.error_word = c->error_word;
    g.x_f32 = x_f32;
    g.norm_w = norm_w;
    const int n = b2s::launch_classifier_gemm(g, c->num_sms, (cudaStream_t)stream);
    if (n < 0) return fail(SAMPLER_E_CUDA, "classifier GEMM launch: %s", cudaGetErrorString((cudaError_t)(-n)));
    rc = dispatch(cfg, logits, batch, V, temperature_rows, topp_rows, coins, rng_state, out_ids, nullptr, row_flags,
                  nullptr, 0, (cudaStream_t)stream, 0, stats, sld);
    g_last_launches += n;
    return rc;
}
}  // namespace

extern "C" {

int classifier_sample_fused(const SamplerBatchConfig* cfg, const void* hidden, const void* wcls, int batch, int dim,
                            const float* temperature_rows, const float* topp_rows, const float* coins,
                            unsigned long long* rng_state, int* out_ids, float* logits_out, int* row_flags,
                            void* stream) {
    if (!hidden) return fail(SAMPLER_E_INVALID, "null hidden");
    return fused_call(cfg, hidden, nullptr, nullptr, wcls, batch, dim, temperature_rows, topp_rows, coins, rng_state,
                      out_ids, logits_out, row_flags, stream);
}

// Final RMSNorm prologue alone: out_bf16[b, :] = bf16(weight * (x[b, :] / rms)).
int rmsnorm_bf16(const float* x, const float* norm_weight, int batch, int dim, void* out_bf16, void* stream) {
    g_last_launches = 0;
    if (!x || !norm_weight || !out_bf16) return fail(SAMPLER_E_INVALID, "null x, norm_weight or out_bf16");
    if (batch < 0 || dim < 1) return fail(SAMPLER_E_INVALID, "bad sizes: batch=%d dim=%d", batch, dim);
    if (batch == 0) return SAMPLER_OK;
    const int n = b2s::launch_rmsnorm_bf16(x, norm_weight, batch, dim, out_bf16, (cudaStream_t)stream);
    if (n < 0) return fail(SAMPLER_E_CUDA, "rmsnorm launch: %s", cudaGetErrorString((cudaError_t)(-n)));
    g_last_launches = n;
    return SAMPLER_OK;
}

// The decode step from the last layer's fp32 output: final RMSNorm, classifier
// GEMM with the statistics epilogue, sampling.
int classifier_rmsnorm_sample_fused(const SamplerBatchConfig* cfg, const float* x, const float* norm_weight,
                                    const void* wcls, int batch, int dim, const float* temperature_rows,
                                    const float* topp_rows, const float* coins, unsigned long long* rng_state,
                                    int* out_ids, float* logits_out, int* row_flags, void* stream) {
    g_last_launches = 0;
    if (!x || !norm_weight) return fail(SAMPLER_E_INVALID, "null x or norm_weight");
    if (batch < 0 || dim < 8 || (dim % 8) != 0) return fail(SAMPLER_E_INVALID, "bad sizes: batch=%d dim=%d", batch, dim);
    if (batch == 0) return SAMPLER_OK;
    // one or two rows (decode): the classifier kernel forms the normalized
    // operand itself -- one launch fewer, the same bits
    if (b2s::gemm_folds_rmsnorm(batch, dim))
        return fused_call(cfg, nullptr, x, norm_weight, wcls, batch, dim, temperature_rows, topp_rows, coins,
                          rng_state, out_ids, logits_out, row_flags, stream);
    DeviceCtx* c = nullptr;
    int rc = get_ctx(&c);
    if (rc) return rc;
    const size_t need = (size_t)batch * (size_t)dim * 2;
    void* h = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        StreamBufs* b = bufs_for_call(c, (cudaStream_t)stream, [&](StreamBufs* x) { return x->hnorm_cap >= need; });
        if (!b) return fail(SAMPLER_E_WORKSPACE, "no library buffers for %d rows during a stream capture", batch);
        rc = ensure_buf(&b->hnorm, &b->hnorm_cap, need);
        if (rc) return rc;
        h = b->hnorm;
    }
    const int n = b2s::launch_rmsnorm_bf16(x, norm_weight, batch, dim, h, (cudaStream_t)stream);
    if (n < 0) return fail(SAMPLER_E_CUDA, "rmsnorm launch: %s", cudaGetErrorString((cudaError_t)(-n)));
    rc = classifier_sample_fused(cfg, h, wcls, batch, dim, temperature_rows, topp_rows, coins, rng_state, out_ids,
                                 logits_out, row_flags, stream);
    g_last_launches += n;
    return rc;
}

// Next decode step's input rows from the sampled ids, on the device.
int sampler_gather_rows(const float* table, int table_rows, int dim, const int* ids, int batch, float* out,
                        void* stream) {
    g_last_launches = 0;
    if (!table || !ids || !out) return fail(SAMPLER_E_INVALID, "null table, ids or out");
    if (batch < 0 || dim < 1 || table_rows < 1) return fail(SAMPLER_E_INVALID, "bad sizes");
    if (batch == 0) return SAMPLER_OK;
    if ((dim & 3) == 0 && (((uintptr_t)table | (uintptr_t)out) & 15u))
        return fail(SAMPLER_E_INVALID, "table and out must be 16-byte aligned");
    const int n = b2s::launch_gather_rows(table, table_rows, dim, ids, batch, out, (cudaStream_t)stream);
    if (n < 0) return fail(SAMPLER_E_CUDA, "gather launch: %s", cudaGetErrorString((cudaError_t)(-n)));
    g_last_launches = n;
    return SAMPLER_OK;
}

// The classifier GEMM alone (no statistics, no sampling).
int classifier_logits(const void* hidden, const void* wcls, int batch, int dim, int vocab, float* logits_out,
                      void* stream) {
    g_last_launches = 0;
    if (!hidden || !wcls || !logits_out) return fail(SAMPLER_E_INVALID, "null hidden, wcls or logits_out");
    if (batch < 0 || dim < 8 || (dim % 8) != 0 || vocab < 32 || (vocab % 32) != 0)
        return fail(SAMPLER_E_INVALID, "bad sizes: batch=%d dim=%d (multiple of 8) vocab=%d (multiple of 32)", batch,
                    dim, vocab);
    if (((uintptr_t)hidden & 15u) || ((uintptr_t)wcls & 15u) || ((uintptr_t)logits_out & 15u))
        return fail(SAMPLER_E_INVALID, "hidden, wcls and logits_out must be 16-byte aligned");
    if (batch == 0) return SAMPLER_OK;
    DeviceCtx* c = nullptr;
    const int rc = get_ctx(&c);
    if (rc) return rc;
    b2s::GemmLaunch g{};
    g.h = hidden;
    g.w = wcls;
    g.batch = batch;
    g.dim = dim;
    g.vocab = vocab;
    g.logits = logits_out;
    g.ld = vocab;
    g.temperature = 1.0f;
    g.error_word = c->error_word;
    const int n = b2s::launch_classifier_gemm(g, c->num_sms, (cudaStream_t)stream);
    if (n < 0) return fail(SAMPLER_E_CUDA, "classifier GEMM launch: %s", cudaGetErrorString((cudaError_t)(-n)));
    g_last_launches = n;
    return SAMPLER_OK;
}

int sampler_batched_host(const SamplerBatchConfig* cfg, const float* logits, int batch, long long ld,
                         const float* topp_rows, unsigned long long* rng_state, int* out_ids) {
    g_last_launches = 0;
    if (!cfg || !logits || !out_ids) return fail(SAMPLER_E_INVALID, "null config, logits or out_ids");
    const int V = cfg->vocab_size;
    if (batch < 0 || V < 1 || ld < V) return fail(SAMPLER_E_INVALID, "bad sizes");
    if (batch == 0) return SAMPLER_OK;
    DeviceCtx* c = nullptr;
    int rc = get_ctx(&c);
    if (rc) return rc;
    std::lock_guard<std::mutex> host_lock(c->host_mu);
    const bool all_greedy = !(cfg->flags & SAMPLER_FLAG_PROBS_IN) &&
                            (cfg->temperature == 0.0f ||
                             ((cfg->flags & SAMPLER_FLAG_GREEDY_BELOW_1E6) && cfg->temperature < 1e-6f));
    if (!all_greedy && !rng_state) return fail(SAMPLER_E_INVALID, "rng_state is NULL");
    // Pipeline: one stream copies in -- the per-row inputs first, then the
    // logits in up to 16 pieces back to back (pieces of tens of MB keep the
    // host-to-device engine at its full rate, where one large copy runs
    // slower and small copies or kernels between pieces leave it idle) -- and
    // one stream samples each piece once it has landed and copies its ids and
    // states back (the other direction's engine).  One stream samples, so one
    // workspace serves every piece.
    constexpr int kPieces = 16;
    int piece = (batch + kPieces - 1) / kPieces;
    if (piece < 1) piece = 1;
    const size_t ws_bytes = (workspace_for(c, V, piece) + 255) & ~(size_t)255;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        rc = ensure_buf(&c->pipe_ws, &c->pipe_ws_bytes, ws_bytes);
        if (rc) return rc;
        const size_t need = (size_t)batch * (size_t)V;
        if (c->logits_cap < need) {
            if (c->d_logits) cudaFree(c->d_logits);
            c->d_logits = nullptr;
            c->logits_cap = 0;
            B2S_CUDA(cudaMalloc(&c->d_logits, need * sizeof(float)));
            c->logits_cap = need;
        }
        if (c->rows_cap < batch) {
            if (c->d_topp) cudaFree(c->d_topp);
            if (c->d_state) cudaFree(c->d_state);
            if (c->d_ids) cudaFree(c->d_ids);
            c->d_topp = nullptr;
            c->d_state = nullptr;
            c->d_ids = nullptr;
            c->rows_cap = 0;
            B2S_CUDA(cudaMalloc(&c->d_topp, (size_t)batch * sizeof(float)));
            B2S_CUDA(cudaMalloc(&c->d_state, (size_t)batch * sizeof(unsigned long long)));
            B2S_CUDA(cudaMalloc(&c->d_ids, (size_t)batch * sizeof(int)));
            c->rows_cap = batch;
        }
    }
    cudaStream_t cs = c->streams[0], ks = c->streams[1];
    if (topp_rows)
        B2S_CUDA(cudaMemcpyAsync(c->d_topp, topp_rows, (size_t)batch * sizeof(float), cudaMemcpyHostToDevice, cs));
    if (!all_greedy)
        B2S_CUDA(cudaMemcpyAsync(c->d_state, rng_state, (size_t)batch * sizeof(unsigned long long),
                                 cudaMemcpyHostToDevice, cs));
    // every upload is queued before any copy back: a copy into pageable host
    // memory returns only once done, and would hold back the next upload
    for (int r0 = 0, k = 0; r0 < batch; r0 += piece, ++k) {
        const int rows = (batch - r0) < piece ? (batch - r0) : piece;
        float* dl = c->d_logits + (size_t)r0 * V;
        if (ld == V) {
            B2S_CUDA(cudaMemcpyAsync(dl, logits + (size_t)r0 * V, (size_t)rows * V * sizeof(float),
                                     cudaMemcpyHostToDevice, cs));
        } else {
            B2S_CUDA(cudaMemcpy2DAsync(dl, (size_t)V * sizeof(float), logits + (size_t)r0 * ld,
                                       (size_t)ld * sizeof(float), (size_t)V * sizeof(float), rows,
                                       cudaMemcpyHostToDevice, cs));
        }
        B2S_CUDA(cudaEventRecord(c->piece_ready[k], cs));
    }
    int launches = 0;
    for (int r0 = 0, k = 0; r0 < batch; r0 += piece, ++k) {
        const int rows = (batch - r0) < piece ? (batch - r0) : piece;
        float* dl = c->d_logits + (size_t)r0 * V;
        B2S_CUDA(cudaStreamWaitEvent(ks, c->piece_ready[k], 0));
        rc = dispatch(cfg, dl, rows, V, nullptr, topp_rows ? c->d_topp + r0 : nullptr, nullptr,
                      all_greedy ? nullptr : c->d_state + r0, c->d_ids + r0, nullptr, nullptr, c->pipe_ws, ws_bytes,
                      ks, 0);
        if (rc) return rc;
        launches += g_last_launches;
        B2S_CUDA(cudaMemcpyAsync(out_ids + r0, c->d_ids + r0, rows * sizeof(int), cudaMemcpyDeviceToHost, ks));
        if (!all_greedy)
            B2S_CUDA(cudaMemcpyAsync(rng_state + r0, c->d_state + r0, rows * sizeof(unsigned long long),
                                     cudaMemcpyDeviceToHost, ks));
    }
    B2S_CUDA(cudaStreamSynchronize(c->streams[0]));
    B2S_CUDA(cudaStreamSynchronize(c->streams[1]));
    g_last_launches = launches;
    return check_device_word(c);
}

// Failure-detection self-test: the row kernel on one zero row whose staging
// issues no copy, so its first bounded wait runs out after `polls` polls; the
// timeout is reported the way a real one is.
int sampler_selftest_wait_timeout(unsigned polls, int* row_flag) {
    g_last_launches = 0;
    if (polls == 0 || polls > (1u << 24) || !row_flag)
        return fail(SAMPLER_E_INVALID, "polls must be in [1, 2^24] and row_flag non-NULL");
    DeviceCtx* c = nullptr;
    int rc = get_ctx(&c);
    if (rc) return rc;
    std::lock_guard<std::mutex> host_lock(c->host_mu);
    constexpr int V = 64;
    if (ensure_row(c, V)) return SAMPLER_E_CUDA;
    cudaStream_t s = c->stream;
    int* d_flag = c->d_id + 1;  // d_id holds 4 ints: [0] the id, [1] the row flag
    B2S_CUDA(cudaMemsetAsync(c->d_row, 0, V * sizeof(float), s));
    B2S_CUDA(cudaMemsetAsync(c->d_id, 0xFF, 2 * sizeof(int), s));
    b2s::RowLaunch p{};
    p.logits = c->d_row;
    p.ld = V;
    p.batch = 1;
    p.vocab = V;
    p.temperature = 0.0f;
    p.topp = 0.9f;
    p.out_ids = c->d_id;
    p.row_flags = d_flag;
    p.error_word = c->error_word;
    p.wait_test = polls;
    const int n = b2s::launch_row_sampler(p, 1, s);
    if (n < 0) return fail(SAMPLER_E_CUDA, "row sampler launch: %s", cudaGetErrorString((cudaError_t)(-n)));
    g_last_launches = n;
    B2S_CUDA(cudaMemcpyAsync(row_flag, d_flag, sizeof(int), cudaMemcpyDeviceToHost, s));
    B2S_CUDA(cudaStreamSynchronize(s));
    return check_device_word(c);
}

int sampler_seed_states(unsigned long long* rng_state, int batch, unsigned long long rng_seed,
                        long long row_offset, void* stream) {
    if (!rng_state || batch < 0) return fail(SAMPLER_E_INVALID, "bad arguments");
    if (batch == 0) return SAMPLER_OK;
    const int n = b2s::launch_seed_states(rng_state, batch, rng_seed, row_offset, (cudaStream_t)stream);
    if (n < 0) return fail(SAMPLER_E_CUDA, "seed launch: %s", cudaGetErrorString((cudaError_t)(-n)));
    return SAMPLER_OK;
}

int sampler_last_launch_count(void) { return g_last_launches; }

const char* sampler_last_error(void) { return g_last_error.c_str(); }

// ===========================================================================
// Multi-GPU helpers
// ===========================================================================
int sampler_shard_rows(int batch, int world, int rank, int* row_begin, int* row_count) {
    if (batch < 0 || world < 1 || rank < 0 || rank >= world || !row_begin || !row_count)
        return fail(SAMPLER_E_INVALID, "bad shard arguments");
    const int base = batch / world, rem = batch % world;
    *row_begin = rank * base + (rank < rem ? rank : rem);
    *row_count = base + (rank < rem ? 1 : 0);
    return SAMPLER_OK;
}

int sampler_nccl_get_unique_id(void* id128) {
    if (!id128) return fail(SAMPLER_E_INVALID, "null id buffer");
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId id;
    const ncclResult_t r = g_nccl.get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id128, &id, sizeof(id));
    return SAMPLER_OK;
}

int sampler_nccl_comm_init(void** comm, int nranks, const void* id128, int rank) {
    if (!comm || !id128) return fail(SAMPLER_E_INVALID, "null argument");
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId id;
    memcpy(&id, id128, sizeof(id));
    ncclComm_t cm = nullptr;
    const ncclResult_t r = g_nccl.comm_init_rank(&cm, nranks, id, rank);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    *comm = cm;
    return SAMPLER_OK;
}

int sampler_nccl_allgather_ids(void* comm, const int* ids_local, int rows_per_rank, int* ids_all, void* stream) {
    if (!comm || !ids_local || !ids_all || rows_per_rank < 0) return fail(SAMPLER_E_INVALID, "bad arguments");
    int rc = nccl_load();
    if (rc) return rc;
    const ncclResult_t r = g_nccl.all_gather(ids_local, ids_all, (size_t)rows_per_rank, ncclInt32,
                                             (ncclComm_t)comm, (cudaStream_t)stream);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    return SAMPLER_OK;
}

int sampler_nccl_comm_destroy(void* comm) {
    if (!comm) return SAMPLER_OK;
    int rc = nccl_load();
    if (rc) return rc;
    const ncclResult_t r = g_nccl.comm_destroy((ncclComm_t)comm);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommDestroy");
    return SAMPLER_OK;
}

}  // extern "C"
