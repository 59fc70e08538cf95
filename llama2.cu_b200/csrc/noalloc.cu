// noalloc.cu -- the batched sampler without any device allocation.
//
// Some callers cannot call cudaMalloc: an inference server whose device
// memory is owned by its own arena or caching allocator (a foreign
// cudaMalloc would bypass its accounting and can fail once it has reserved
// the card), or a decode loop where cudaMalloc/cudaFree would implicitly
// synchronize the device.  sampler_batched() allocates its workspace on
// first use; this entry point instead runs the general row kernel with its
// scratch (the per-CTA sort area of the nucleus slow path and the device
// error word) in a fixed array compiled into the library.  The array exists
// on every GPU that loads the library, until the process exits.
#include "../../include/b200_sampler.h"
#include "sampler_kernels.cuh"

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace {

// 256 bytes of header (the device error word) + 8 MiB of slow-path scratch:
// 32 CTAs x 32768 keys x 8 bytes at the maximum vocabulary.
constexpr size_t kHeaderBytes = 256;
constexpr size_t kScratchBytes = (size_t)8 << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kHeaderBytes + kScratchBytes];

constexpr int kMaxDevices = 64;
struct DevScratch {
    unsigned char* base = nullptr;  // device address of g_noalloc_scratch on that device
    int num_sms = 0;
};
DevScratch g_dev[kMaxDevices];
std::mutex g_setup_mu;

size_t pow2_at_least(size_t x) {
    size_t p = 1;
    while (p < x) p <<= 1;
    return p;
}

// Once per device, with that device current: the device address of the
// array (in host code its name is only a host-side stand-in).
int setup_device(int dev, DevScratch** out) {
    if (dev < 0 || dev >= kMaxDevices) return SAMPLER_E_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_setup_mu);
    DevScratch& d = g_dev[dev];
    if (!d.base) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return SAMPLER_E_CUDA;
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
            return SAMPLER_E_CUDA;
        d.num_sms = sms;
        d.base = static_cast<unsigned char*>(ptr);
    }
    *out = &d;
    return SAMPLER_OK;
}

}  // namespace

extern "C" int sampler_batched_noalloc(const SamplerBatchConfig* cfg, const float* logits, int batch,
                                       long long ld, const float* temperature_rows, const float* topp_rows,
                                       const float* coins, unsigned long long* rng_state, int* out_ids,
                                       float* probs_out, int* row_flags, void* stream) {
    if (!cfg || !logits || !out_ids) return SAMPLER_E_INVALID;
    const int V = cfg->vocab_size;
    if (batch < 0 || V < 1 || ld < V) return SAMPLER_E_INVALID;
    if (V > SAMPLER_NOALLOC_MAX_VOCAB) return SAMPLER_E_UNSUPPORTED;
    if (batch == 0) return SAMPLER_OK;
    const int mode_bits = SAMPLER_FLAG_GREEDY_BELOW_1E6 | SAMPLER_FLAG_NAN_TOKEN1;
    if (cfg->flags & ~(SAMPLER_FLAG_PROBS_IN | mode_bits)) return SAMPLER_E_INVALID;
    const bool probs_in = (cfg->flags & SAMPLER_FLAG_PROBS_IN) != 0;
    if (probs_in && (cfg->flags & mode_bits)) return SAMPLER_E_INVALID;
    const bool greedy_eps = (cfg->flags & SAMPLER_FLAG_GREEDY_BELOW_1E6) != 0;
    const bool any_draw = probs_in || temperature_rows ||
                          !(cfg->temperature == 0.0f || (greedy_eps && cfg->temperature < 1e-6f));
    if (any_draw && !coins && !rng_state) return SAMPLER_E_INVALID;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return SAMPLER_E_CUDA;
    DevScratch* d = nullptr;
    const int rc = setup_device(dev, &d);
    if (rc) return rc;

    // as many CTAs as the scratch holds slow-path areas for (32 at V = 32768)
    const size_t stride = pow2_at_least((size_t)V);
    int ctas = (int)(kScratchBytes / (stride * sizeof(unsigned long long)));
    if (ctas > d->num_sms) ctas = d->num_sms;
    if (ctas > batch) ctas = batch;

    // The error word starts each call at zero (a stream-ordered memset of the
    // array's header; no allocation).  Its value is not read back: the call
    // does not synchronize, so a timeout shows only in row_flags.
    if (cudaMemsetAsync(d->base, 0, sizeof(int), (cudaStream_t)stream) != cudaSuccess) return SAMPLER_E_CUDA;

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
    p.error_word = reinterpret_cast<int*>(d->base);
    p.workspace = reinterpret_cast<unsigned long long*>(d->base + kHeaderBytes);
    p.ws_stride = (long long)stride;
    p.probs_in = probs_in ? 1 : 0;
    p.force_mode = 0;
    p.greedy_eps = greedy_eps ? 1 : 0;
    p.nan_token1 = (cfg->flags & SAMPLER_FLAG_NAN_TOKEN1) ? 1 : 0;
    const int n = b2s::launch_row_sampler(p, ctas, (cudaStream_t)stream);
    return n < 0 ? SAMPLER_E_CUDA : SAMPLER_OK;
}
