// Standalone decode-attention kernel (one launch per layer, used when the persistent decode kernel is not) and the
// lm-head argmax / end-of-step kernels.
#include <math.h>

#include "v3g_attn.cuh"
#include "v3g_internal.h"

namespace v3g {

// one work item per CTA: `tps` 64-key tiles of (sequence blockIdx.z, KV head blockIdx.y), split blockIdx.x
template <int D>
__global__ void __launch_bounds__(ATT_THREADS) k_attention(const ModelDev *mp, const StateDev *sp, int layer,
                                                           float scale, int tps) {
    __shared__ __align__(16) AttnSmemSpan<D> sm;
    griddep_wait();
    griddep_launch();
    const int64_t pos = __ldcg(&sp->step->pos);
    (void)mp;
    const KeySpan ks = key_span(*sp, blockIdx.z, pos);
    attn_span<D>(*sp, ks, layer, scale, blockIdx.x, tps, blockIdx.y, blockIdx.z, pos, sm, blockDim.x);
}

// greedy next token = first index of the largest logit (v3_argmax, runtime/vault3.c:3198-3202; torch.argmax):
// each CTA reduces a slice and folds (value, ~index) into one 64-bit atomicMax per sequence
__global__ void __launch_bounds__(256) k_argmax_partial(const ModelDev *mp, const StateDev *sp) {
    griddep_wait();
    griddep_launch();
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int b = blockIdx.y, tid = threadIdx.x;
    const float *lg = s.logits + (size_t)b * m.vocab;
    const int per = (m.vocab + gridDim.x - 1) / gridDim.x;
    const int i0 = blockIdx.x * per, i1 = min(m.vocab, i0 + per);
    unsigned long long best = 0ull;
    for (int i = i0 + tid; i < i1; i += blockDim.x) {
        const float v = __ldcg(&lg[i]);
        if (v == v) {   // NaN never wins
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
        atomicMax(&s.amax[b], best);
    }
}

// finish the step: next token per sequence (tok_in for greedy chaining, optional token sink), advance pos
__global__ void k_finish(const StateDev *sp, int want_lm) {
    griddep_wait();
    griddep_launch();
    const StateDev &s = *sp;
    StepCtl &sc = *s.step;
    for (int b = threadIdx.x; b < s.B && want_lm; b += blockDim.x) {
        const unsigned long long key = __ldcg(&s.amax[b]);
        const int tok = key ? (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu)) : 0;
        s.tok_in[b] = tok;
        if (sc.out_tokens) sc.out_tokens[(int64_t)b * sc.out_ld + sc.out_idx] = tok;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        sc.pos += 1;
        if (sc.ids) sc.ids_idx += 1;
        if (sc.out_tokens && want_lm) sc.out_idx += 1;
    }
}

// tiles per split: enough splits to give the SMs about four items each at the state's longest key span, at most
// 16 tiles (1,024 keys) per item
template <int D>
static cudaError_t launch_attention_d(const v3g_model *m, v3g_state *s, int layer, bool pdl, cudaStream_t st) {
    const int64_t work = (int64_t)s->host.max_splits * m->host.G * s->B;   // 64-key tiles at the longest span
    int tps = (int)(work / (4 * (int64_t)m->n_sm));
    tps = tps < 1 ? 1 : (tps > 16 ? 16 : tps);
    dim3 grid((s->host.max_splits + tps - 1) / tps, m->host.G, s->B);
    return launch_k(pdl, k_attention<D>, grid, dim3(ATT_THREADS), 0, st, (const ModelDev *)m->dev,
                    (const StateDev *)s->dev, layer, (float)(1.0 / sqrt((double)D)), tps);
}

cudaError_t launch_attention(const v3g_model *m, v3g_state *s, int layer, bool pdl, cudaStream_t st) {
    switch (m->host.D) {
        case 16: return launch_attention_d<16>(m, s, layer, pdl, st);
        case 32: return launch_attention_d<32>(m, s, layer, pdl, st);
        case 64: return launch_attention_d<64>(m, s, layer, pdl, st);
        case 128: return launch_attention_d<128>(m, s, layer, pdl, st);
        default: return cudaErrorInvalidValue;   // head_dim is checked at load time
    }
}

cudaError_t launch_argmax_only(const v3g_model *m, v3g_state *s, cudaStream_t st) {
    return launch_k(false, k_argmax_partial, dim3(32, s->B), dim3(256), 0, st, (const ModelDev *)m->dev,
                    (const StateDev *)s->dev);
}

cudaError_t launch_argmax_finish(const v3g_model *m, v3g_state *s, bool want_lm, bool pdl, cudaStream_t st) {
    cudaError_t e = cudaSuccess;
    if (want_lm) e = launch_k(pdl, k_argmax_partial, dim3(32, s->B), dim3(256), 0, st, (const ModelDev *)m->dev,
                              (const StateDev *)s->dev);
    if (e != cudaSuccess) return e;
    return launch_k(pdl, k_finish, dim3(1), dim3(256), 0, st, (const StateDev *)s->dev, want_lm ? 1 : 0);
}

}  // namespace v3g
