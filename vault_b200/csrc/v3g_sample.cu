// Top-k + temperature sampling of logit rows on the device: the reference's v3_sample_topk
// (runtime/vault3.c:3204-3230, declared runtime/vault3.h:221), one CTA per row.
//
//   temp <= 0 or k <= 1: the greedy token (first maximum, v3_argmax, runtime/vault3.c:3198-3202);
//   otherwise, with k capped at 64: the k largest logits, ordered by value (descending) and, among equal values, by
//   index (ascending) -- the order the reference's insertion list produces -- then
//     p[j] = expf_ref((val[j] - val[0]) / temp),  sum = p[0] + p[1] + ... (in order),
//     x = xorshift64(rng) (13, 7, 17; a zero state starts from 0x9E3779B97F4A7C15), rng <- x,
//     r = ((x >> 40) & 0xFFFFFF) / 2^24 * sum, and the first j with (r -= p[j]) <= 0 gives the token.
// expf_ref is the reference's own exponential (v3_expf, runtime/vault3.c:104-114: Cody-Waite reduction with a
// degree-7 polynomial) restated with explicitly rounded operations; the whole draw runs on one thread in the
// reference's operation order.
//
// Selection: every logit becomes the 64-bit key (order-preserving float bits << 32) | (2^32 - 1 - index), the key
// of the greedy token in k_argmax_partial, so "larger key" = "larger value, or equal value and smaller index"
// (-0.0 equals +0.0, NaN is never a candidate).  The k-th largest key is found by an 8-pass radix select (8 bits
// per pass, shared-memory histograms); the k keys at or above it are collected and ranked in shared memory.  No
// global scratch: the CTA's shared memory holds all of it.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/vault_b200.h"
#include "v3g.cuh"
#include "v3g_internal.h"

namespace v3g {

constexpr int SAMPLE_THREADS = 512;
constexpr int SAMPLE_KMAX = 64;

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// v3_expf of runtime/vault3.c:104-114, every operation rounded on its own (no contraction)
__device__ float expf_ref(float x) {
    if (x > 88.72f) return u2f(0x7F800000u);
    if (x < -103.9f) return 0.0f;
    const float kf = __fmul_rn(x, 1.44269504088896341f);
    const int k = (int)__fadd_rn(kf, kf >= 0.0f ? 0.5f : -0.5f);   // C conversion: truncation toward zero
    const float fk = (float)k;
    const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(fk, 0.693145751953125f)), __fmul_rn(fk, 1.428606765330187e-06f));
    float p = __fadd_rn(1.3888889e-3f, __fmul_rn(r, 1.9841270e-4f));
    p = __fadd_rn(8.3333338e-3f, __fmul_rn(r, p));
    p = __fadd_rn(4.1666668e-2f, __fmul_rn(r, p));
    p = __fadd_rn(1.6666667e-1f, __fmul_rn(r, p));
    p = __fadd_rn(0.5f, __fmul_rn(r, p));
    p = __fadd_rn(1.0f, __fmul_rn(r, p));
    p = __fadd_rn(1.0f, __fmul_rn(r, p));
    if (k > 127) return __fmul_rn(__fmul_rn(p, u2f(254u << 23)), 2.0f);
    if (k < -126) return __fmul_rn(__fmul_rn(p, u2f((uint32_t)(k + 126 + 127) << 23)), u2f(1u << 23));
    return __fmul_rn(p, u2f((uint32_t)(k + 127) << 23));
}

__device__ __forceinline__ uint64_t logit_key(float v, uint32_t i) {
    return ((uint64_t)float_key(v) << 32) | (uint64_t)(0xFFFFFFFFu - i);
}

// tokens[row] gets the draw; out (when not null) also gets it at out[row * out_ld] (the generation token sink)
__global__ void __launch_bounds__(SAMPLE_THREADS) k_sample_topk(const float *logits, uint32_t vocab, uint64_t ld,
                                                               uint32_t k, float temp, uint64_t *rng,
                                                               int32_t *tokens, int32_t *out, int64_t out_ld) {
    const int tid = threadIdx.x, nt = blockDim.x;
    auto emit = [&](int32_t tok) {
        tokens[blockIdx.x] = tok;
        if (out) out[(int64_t)blockIdx.x * out_ld] = tok;
    };
    const float *lg = logits + (size_t)blockIdx.x * ld;
    __shared__ unsigned int hist[256];
    __shared__ uint64_t sel[SAMPLE_KMAX], sorted[SAMPLE_KMAX];
    __shared__ unsigned long long best;
    __shared__ uint64_t prefix;
    __shared__ int need, cnt;
    const bool greedy = temp <= 0.0f || k <= 1;
    if (greedy) {   // first maximum, NaN never selected
        if (tid == 0) best = 0ull;
        __syncthreads();
        unsigned long long b = 0ull;
        for (uint32_t i = tid; i < vocab; i += nt) {
            const float v = lg[i];
            if (v == v) {
                const unsigned long long key = logit_key(v, i);
                b = key > b ? key : b;
            }
        }
        atomicMax(&best, b);
        __syncthreads();
        if (tid == 0) emit(best ? (int32_t)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu)) : 0);
        return;
    }
    const uint32_t kk = k > (uint32_t)SAMPLE_KMAX ? (uint32_t)SAMPLE_KMAX : k;
    if (tid == 0) {
        prefix = 0ull;
        need = (int)kk;
        cnt = 0;
    }
    // radix select of the need-th largest key, 8 bits per pass from the top
    for (int pass = 0; pass < 8; ++pass) {
        const int shift = 56 - 8 * pass;
        for (int b = tid; b < 256; b += nt) hist[b] = 0u;
        __syncthreads();
        const uint64_t pre = prefix;
        for (uint32_t i = tid; i < vocab; i += nt) {
            const float v = lg[i];
            if (v != v) continue;
            const uint64_t key = logit_key(v, i);
            if (pass == 0 || (key >> (shift + 8)) == (pre >> (shift + 8)))
                atomicAdd(&hist[(unsigned)(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            if (pass == 0) {   // fewer non-NaN logits than k: take them all
                unsigned int total = 0u;
                for (int b = 0; b < 256; ++b) total += hist[b];
                if ((unsigned)need > total) need = (int)total;
            }
            int digit = 0;
            if (need > 0) {
                unsigned int cum = 0u;
                for (int b = 255; b >= 0; --b) {
                    if (cum + hist[b] >= (unsigned)need) {
                        digit = b;
                        need -= (int)cum;
                        break;
                    }
                    cum += hist[b];
                }
            }
            prefix = pre | ((uint64_t)digit << shift);
        }
        __syncthreads();
    }
    // the keys at or above the selected one: exactly min(k, non-NaN logits) of them (keys are distinct)
    const uint64_t kth = prefix;
    const bool any = need > 0;
    for (uint32_t i = tid; i < vocab && any; i += nt) {
        const float v = lg[i];
        if (v != v) continue;
        const uint64_t key = logit_key(v, i);
        if (key >= kth) {
            const int slot = atomicAdd(&cnt, 1);
            if (slot < SAMPLE_KMAX) sel[slot] = key;
        }
    }
    __syncthreads();
    const int n = cnt < SAMPLE_KMAX ? cnt : SAMPLE_KMAX;
    if (tid < n) {   // rank by counting larger keys
        const uint64_t mine = sel[tid];
        int rank = 0;
        for (int j = 0; j < n; ++j) rank += sel[j] > mine ? 1 : 0;
        sorted[rank] = mine;
    }
    __syncthreads();
    if (tid != 0) return;
    if (n == 0) {   // no finite logit
        emit(0);
        return;
    }
    float p[SAMPLE_KMAX];
    int32_t idx[SAMPLE_KMAX];
    float sum = 0.0f;
    const float v0 = lg[0xFFFFFFFFu - (uint32_t)(sorted[0] & 0xFFFFFFFFu)];
    for (int j = 0; j < n; ++j) {
        idx[j] = (int32_t)(0xFFFFFFFFu - (uint32_t)(sorted[j] & 0xFFFFFFFFu));
        p[j] = expf_ref(__fdiv_rn(__fsub_rn(lg[idx[j]], v0), temp));
        sum = __fadd_rn(sum, p[j]);
    }
    uint64_t x = rng[blockIdx.x] ? rng[blockIdx.x] : 0x9E3779B97F4A7C15ull;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    rng[blockIdx.x] = x;
    float r = __fmul_rn(__fdiv_rn((float)((x >> 40) & 0xFFFFFFull), 16777216.0f), sum);
    int32_t tok = idx[n - 1];
    for (int j = 0; j < n; ++j) {
        r = __fsub_rn(r, p[j]);
        if (r <= 0.0f) {
            tok = idx[j];
            break;
        }
    }
    emit(tok);
}

cudaError_t launch_sample_topk(const float *logits, uint32_t rows, uint32_t vocab, uint64_t ld, uint32_t k, float temp,
                               uint64_t *rng, int32_t *tokens, int32_t *out, int64_t out_ld, cudaStream_t st) {
    k_sample_topk<<<rows, SAMPLE_THREADS, 0, st>>>(logits, vocab, ld, k, temp, rng, tokens, out, out_ld);
    return cudaGetLastError();
}

}  // namespace v3g

using namespace v3g;

extern "C" int v3g_sample_topk(const float *dev_logits, uint32_t rows, uint32_t vocab, uint64_t ld, uint32_t k,
                               float temp, uint64_t *dev_rng, int32_t *dev_tokens, void *stream) {
    if (!dev_logits || !dev_tokens || (!dev_rng && !(temp <= 0.0f || k <= 1)))
        return v3g_fail(V3G_E_ARG, "v3g_sample_topk: null pointer");
    if (vocab == 0 || ld < vocab) return v3g_fail(V3G_E_ARG, "v3g_sample_topk: vocab must be > 0 and <= ld");
    if (rows == 0) return V3G_OK;
    const cudaError_t e = launch_sample_topk(dev_logits, rows, vocab, ld, k, temp, dev_rng, dev_tokens, nullptr, 0,
                                             (cudaStream_t)stream);
    return e == cudaSuccess ? V3G_OK : v3g_fail(V3G_E_CUDA, cudaGetErrorString(e));
}
