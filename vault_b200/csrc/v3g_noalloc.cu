// Greedy-token selection for callers that cannot allocate device memory.
//
// v3g_step picks each sequence's next token with a multi-CTA argmax whose per-row 64-bit keys live in the
// state arena.  Some callers of this library have logits but no state arena and may not call cudaMalloc: a
// serving runtime whose caching allocator owns every byte of device memory (a side allocation breaks its
// accounting and, through the implicit device synchronisation of cudaMalloc / cudaFree, stalls every other
// stream), or a sampling loop that must not pay allocator latency per token.  v3g_argmax_noalloc gives them the
// same selection with its scratch keys in a fixed file-scope device array instead.
//
// Limits: at most V3G_NOALLOC_MAX_ROWS rows per call (the array is 8 bytes per row and is held by every GPU that
// loads the library until the process exits).  All calls share the array: calls that overlap on the GPU race and
// give wrong tokens, so calls must be ordered (one stream, or events between streams).
#include <mutex>

#include "../../include/vault_b200.h"
#include "v3g_internal.h"

namespace v3g {

constexpr int NOALLOC_MAX_DEVICES = 64;
constexpr int NOALLOC_CTAS_PER_ROW = 32;

// per-row best key: (order-preserving float key << 32) | (~index), so the largest key is the first maximum
static __device__ __align__(256) unsigned long long g_noalloc_keys[V3G_NOALLOC_MAX_ROWS];

__global__ void k_noalloc_clear(unsigned long long *keys, int rows) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) keys[i] = 0ull;
}

// row blockIdx.y, vocab slice blockIdx.x: the same selection rule as the step's argmax (NaN never wins; -0.0 and
// +0.0 tie, the first index wins; a row without a non-NaN value keeps key 0 and yields token 0)
__global__ void __launch_bounds__(256) k_noalloc_argmax(const float *logits, int vocab, size_t ld,
                                                        unsigned long long *keys) {
    const int b = blockIdx.y, tid = threadIdx.x;
    const float *lg = logits + (size_t)b * ld;
    // 64-bit slice bounds: vocab may be as large as 2^31 - 1, where i0 + per and i + blockDim.x leave int range
    const int64_t per = ((int64_t)vocab + gridDim.x - 1) / gridDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * per, i1 = i0 + per < vocab ? i0 + per : (int64_t)vocab;
    unsigned long long best = 0ull;
    for (int64_t i = i0 + tid; i < i1; i += blockDim.x) {
        const float v = lg[i];
        if (v == v) {
            const unsigned long long key = ((unsigned long long)float_key(v) << 32) | (0xFFFFFFFFu - (uint32_t)i);
            best = key > best ? key : best;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    __shared__ unsigned long long sb[8];
    if ((tid & 31) == 0) sb[tid >> 5] = best;
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (int)blockDim.x / 32; ++w) best = sb[w] > best ? sb[w] : best;
        atomicMax(&keys[b], best);
    }
}

__global__ void k_noalloc_tokens(const unsigned long long *keys, int rows, int32_t *out) {
    for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < rows; b += gridDim.x * blockDim.x) {
        const unsigned long long key = keys[b];
        out[b] = key ? (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu)) : 0;
    }
}

// device address of g_noalloc_keys on the current device, looked up once per device
static cudaError_t noalloc_keys(unsigned long long **out) {
    static std::mutex mu;
    static unsigned long long *addr[NOALLOC_MAX_DEVICES] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_keys);
        if (e != cudaSuccess) return e;
        addr[dev] = static_cast<unsigned long long *>(p);
    }
    *out = addr[dev];
    return cudaSuccess;
}

}  // namespace v3g

using namespace v3g;

extern "C" int v3g_argmax_noalloc(const float *dev_logits, uint32_t rows, uint32_t vocab, uint64_t ld,
                                  int32_t *dev_tokens, void *stream) {
    if (!dev_logits || !dev_tokens || rows == 0 || vocab == 0 || ld < vocab || vocab > 0x7FFFFFFFu)
        return v3g_fail(V3G_E_ARG, "v3g_argmax_noalloc: null pointer, zero size or ld < vocab");
    if (rows > V3G_NOALLOC_MAX_ROWS)
        return v3g_fail(V3G_E_LIMIT, "v3g_argmax_noalloc: more rows than V3G_NOALLOC_MAX_ROWS (4096) per call");
    unsigned long long *keys = nullptr;
    cudaError_t e = noalloc_keys(&keys);
    if (e != cudaSuccess) return v3g_fail(V3G_E_CUDA, std::string("v3g_argmax_noalloc set-up: ") + cudaGetErrorString(e));
    cudaStream_t st = (cudaStream_t)stream;
    const int r = (int)rows;
    k_noalloc_clear<<<(r + 255) / 256, 256, 0, st>>>(keys, r);   // the keys must start at zero every call
    k_noalloc_argmax<<<dim3(NOALLOC_CTAS_PER_ROW, r), 256, 0, st>>>(dev_logits, (int)vocab, (size_t)ld, keys);
    k_noalloc_tokens<<<(r + 255) / 256, 256, 0, st>>>(keys, r, dev_tokens);
    e = cudaGetLastError();
    if (e != cudaSuccess) return v3g_fail(V3G_E_CUDA, std::string("v3g_argmax_noalloc launch: ") + cudaGetErrorString(e));
    return V3G_OK;
}
