// Host model of the device algorithms in llama2.cu_b200/csrc/exact_math.cuh,
// compiled with g++ by tests/test_exact_math.py.  It runs the SAME scalar
// functions the kernels use (exp_f32, chain_build/compose/apply,
// chain_guess_binade) and replays the block/warp orchestration of the
// chain engine sequentially, then checks:
//   exp  : against glibc expf on a strided sample of every float in [-104, 0]
//   chain: bit-exact equality with the serial fp32 loop on many row kinds
#include "../../llama2.cu_b200/csrc/exact_math.cuh"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

using namespace xm;

static int check_exp(long stride) {
    ExpTableEntry tab[kExpTableSize];
    for (int j = 0; j < kExpTableSize; ++j) tab[j] = exp_table_entry(j);
    long long tot = 0, mis = 0, big = 0;
    const uint32_t lo = xm_f2u_host(-0.0f), hi = xm_f2u_host(-104.0f);
    for (long long b = lo; b <= hi; b += stride) {
        const float d = xm_u2f_host((uint32_t)b);
        const float a = exp_f32(d, tab), g = expf(d);
        ++tot;
        if (a != g) {
            ++mis;
            const long long df = (long long)xm_f2u_host(a) - (long long)xm_f2u_host(g);
            if (df > 1 || df < -1) ++big;
        }
    }
    // exp(0) must be exactly 1 (the max element of a softmax row)
    if (exp_f32(0.0f, tab) != 1.0f) big++;
    printf("exp: %lld samples, %lld differ from expf (%.4f%%), %lld by more than 1 ulp\n", tot, mis,
           100.0 * mis / tot, big);
    return (big == 0 && mis * 10000 < tot * 3) ? 0 : 1;  // < 0.03% and never > 1 ulp
}

// Sequential replay of chain_run: chunks of CPT, 32-chunk warps.
template <int CPT>
static float engine(const std::vector<float>& a, float s_init, std::vector<float>& chunk_s) {
    const int n = (int)a.size(), nch = (n + CPT - 1) / CPT, nw = (nch + 31) / 32;
    std::vector<std::array<float, CPT>> ch(nch);
    for (int t = 0; t < nch; ++t)
        for (int j = 0; j < CPT; ++j) ch[t][j] = (t * CPT + j < n) ? a[t * CPT + j] : 0.0f;
    std::vector<float> sig(nch), g(nch);
    for (int t = 0; t < nch; ++t) {
        float s = 0.0f;
        for (int j = 0; j < CPT; ++j) s += ch[t][j];
        sig[t] = s;
    }
    float acc = 0.0f;
    for (int t = 0; t < nch; ++t) {
        g[t] = acc + s_init;
        acc += sig[t];
    }
    std::vector<uint32_t> eb(nch);
    std::vector<int> clean(nch, 0);
    std::vector<ChainFn> f(nch, chain_identity());
    for (int t = 0; t < nch; ++t) {
        eb[t] = chain_guess_binade(g[t], sig[t]);
        if (eb[t]) {
            float tmp[CPT];
            for (int j = 0; j < CPT; ++j) tmp[j] = ch[t][j];
            clean[t] = chain_build(tmp, eb[t], f[t]);
        }
    }
    std::vector<int> uni(nw, 0);
    std::vector<uint32_t> web(nw, 0);
    std::vector<ChainFn> wf(nw, chain_identity()), excl(nch, chain_identity());
    for (int w = 0; w < nw; ++w) {
        int u = 1;
        const uint32_t e0 = eb[w * 32];
        for (int l = 0; l < 32 && w * 32 + l < nch; ++l) {
            const int t = w * 32 + l;
            if (!clean[t] || eb[t] != e0) u = 0;
        }
        uni[w] = u;
        web[w] = e0;
        if (u) {
            ChainFn c = chain_identity();
            for (int l = 0; l < 32 && w * 32 + l < nch; ++l) {
                excl[w * 32 + l] = c;
                c = chain_compose(c, f[w * 32 + l]);
            }
            wf[w] = c;
        }
    }
    chunk_s.assign(nch + 1, 0.0f);
    std::vector<float> ws(nw, NAN);
    float s = s_init;
    for (int w = 0; w < nw; ++w) {
        if (uni[w]) {
            float s2 = s;
            if (chain_apply(s2, web[w], wf[w])) {
                ws[w] = s;
                s = s2;
                continue;
            }
        }
        for (int l = 0; l < 32 && w * 32 + l < nch; ++l) {
            const int t = w * 32 + l;
            chunk_s[t] = s;
            float s2 = s;
            if (clean[t] && chain_apply(s2, eb[t], f[t])) {
                s = s2;
            } else {
                for (int j = 0; j < CPT; ++j) s = s + ch[t][j];
            }
        }
    }
    chunk_s[nch] = s;
    for (int w = 0; w < nw; ++w)
        if (!std::isnan(ws[w]))
            for (int l = 0; l < 32 && w * 32 + l < nch; ++l) {
                const int t = w * 32 + l;
                chunk_s[t] = ws[w] + ((xm_f2u_host(ws[w]) & 1u) ? excl[t].L1 : excl[t].L0);
            }
    return s;
}

template <int CPT>
static bool check_row(const std::vector<float>& a, float s_init) {
    std::vector<float> cs;
    const float tot = engine<CPT>(a, s_init, cs);
    float s = s_init;
    for (size_t i = 0; i < a.size(); ++i) {
        if (i % CPT == 0 && cs[i / CPT] != s) return false;
        s += a[i];
    }
    return s == tot;
}

// Markstein division q = RN(x*r), q' = RN(q + RN(x - q*d)*r) with r = RN(1/d)
// (P. Markstein, IBM J. Res. Dev. 34(1), 1990) against IEEE division, on the
// two ranges the kernels use it for: x = l/T with |T| in [2^-10, 2^10] and
// |l| in [2^-60, 2^60], and p = e/S with S in [1, 2^15] and e in [2^-60, 1].
static float markstein(float x, float d, float r) {
    const float q = x * r;
    return fmaf(fmaf(-q, d, x), r, q);
}

static int check_div(long stride) {
    std::mt19937_64 rng(777);
    std::uniform_real_distribution<double> U(0, 1);
    long long n = 0, bad = 0;
    for (int range = 0; range < 2; ++range) {
        std::vector<float> ds = range == 0 ? std::vector<float>{0.7f, 0.8f, 1.0f, 0x1p-10f, 0x1.fffffep9f, -0.5f}
                                           : std::vector<float>{1.0f, 1.5f, 32000.0f, 0x1.fffffep14f, 12345.678f};
        while (ds.size() < 64) {
            const double m = 1.0 + U(rng);
            ds.push_back(range == 0 ? (float)ldexp(m, (int)(U(rng) * 20) - 10) : (float)ldexp(m, (int)(U(rng) * 15)));
        }
        const uint32_t lo = xm_f2u_host(0x1p-60f), hi = xm_f2u_host(range == 0 ? 0x1p60f : 1.0f);
        for (float d : ds) {
            const float r = 1.0f / d;
            for (uint64_t b = lo; b <= hi; b += (uint64_t)stride * 101) {
                for (int sg = 0; sg < (range == 0 ? 2 : 1); ++sg) {
                    const float x = xm_u2f_host((uint32_t)b | (sg ? 0x80000000u : 0u));
                    ++n;
                    if (xm_f2u_host(markstein(x, d, r)) != xm_f2u_host(x / d)) ++bad;
                }
            }
        }
    }
    printf("division: %lld quotients, %lld differ from IEEE division\n", n, bad);
    return bad != 0;
}

int main(int argc, char** argv) {
    const long stride = argc > 1 ? atol(argv[1]) : 97;
    int rc = check_exp(stride) | check_div(stride);
    std::mt19937_64 rng(12345);
    std::normal_distribution<double> N(0, 1);
    std::uniform_real_distribution<double> U(0, 1);
    int rows = 0, bad = 0;
    for (int kind = 0; kind < 10; ++kind) {
        for (int r = 0; r < 12; ++r) {
            const int n = (kind == 8) ? 8192 : (kind == 9 ? 1000 + 37 * r : 32000);
            std::vector<float> x(n), e(n);
            float T = 1.0f;
            for (int i = 0; i < n; ++i) {
                double v;
                switch (kind) {
                    case 0: v = 2 * N(rng); break;
                    case 1: v = 3 * N(rng); T = 0.8f; break;
                    case 2: v = -log(-log(U(rng))) + 12 * U(rng) * pow(1 + (int)(U(rng) * n), -1.1); T = 0.7f; break;
                    case 3: v = 0.01 * N(rng); break;
                    case 4: v = 0.0; break;
                    default: v = 30 * N(rng); break;
                }
                x[i] = (float)v;
            }
            if (kind <= 5 || kind == 9) {
                float mx = x[0] / T;
                for (int i = 0; i < n; ++i) mx = std::max(mx, x[i] / T);
                for (int i = 0; i < n; ++i) e[i] = expf(x[i] / T - mx);
            } else if (kind == 6) {  // absorbed values and exact half-ulp ties
                e[0] = 1.0f;
                for (int i = 1; i < n; ++i) e[i] = ldexpf(i % 3 == 0 ? 1.0f : (i % 3 == 1 ? 1.0f : 3.0f), i % 3 == 0 ? -24 : -25);
            } else if (kind == 7) {  // softmax probabilities
                float s = 0.0f;
                for (int i = 0; i < n; ++i) e[i] = expf((float)N(rng));
                for (int i = 0; i < n; ++i) s += e[i];
                for (int i = 0; i < n; ++i) e[i] /= s;
            } else {  // descending nucleus
                for (int i = 0; i < n; ++i) e[i] = (float)(0.2 * pow(i + 1, -1.3));
            }
            ++rows;
            bool ok = (n == 8192) ? check_row<8>(e, 0.0f) : check_row<32>(e, 0.0f);
            if (kind == 7) ok = ok && check_row<8>(e, 0.25f);  // engine started mid-chain
            if (!ok) ++bad;
        }
    }
    printf("chain: %d rows, %d mismatches with the serial fp32 loop\n", rows, bad);
    return rc | (bad != 0);
}
