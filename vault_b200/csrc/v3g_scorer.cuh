// SegmentScorer v2 with habituation (src/vault_v3_model.py:870-883 SegmentScorer, :2294-2305 step form,
// :1198-1247 chunk form; runtime/vault3.c:961-977, :2201-2216), shared by the decode step (one token per sequence)
// and the chunked prefill (every token of a piece), so both give bit-identical scores and bank selections.
//
//   raw = fc2(gelu(fc1(LN(f)))),  hab = fc2(gelu(fc1(LN(f - 0.65 ema_prev))))
//   score = raw + 0.35 relu(hab - raw)   (raw alone for a stream's first token),   ema = 0.985 ema + 0.015 f
//
// f is the concatenation of the residual streams entering the feature layers.  The element-wise arithmetic uses
// explicitly rounded fp32 operations (no fused multiply-add contraction), the same sequence as the reference's fp32
// tensors, and both callers reduce in one fixed order (256 threads, warp partials summed in warp order).
#pragma once
#include "v3g.cuh"

namespace v3g {

constexpr int SCORER_THREADS = 256;

__device__ __forceinline__ float sc_hab_in(float f, float e) { return __fsub_rn(f, __fmul_rn(0.65f, e)); }
__device__ __forceinline__ float sc_ema_next(float e, float f) {
    return __fadd_rn(__fmul_rn(0.985f, e), __fmul_rn(0.015f, f));
}
__device__ __forceinline__ float sc_ln(float v, float mu, float inv, float lw, float lb) {
    return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, mu), inv), lw), lb);
}

// LayerNorm statistics of the raw (in0) and habituated (in1) feature rows over fd features (eps 1e-5), one 256-thread
// CTA: stat = {mean0, mean1, 1/std0, 1/std1} on every thread.  Thread tid sums features tid, tid + 256, ..., the warp
// sums reduce by butterfly and thread 0 adds the 8 warp partials in warp order.
template <class In0, class In1>
__device__ void scorer_ln_stats_block(int fd, const In0 &in0, const In1 &in1, float (&stat)[4]) {
    const int tid = threadIdx.x, nt = SCORER_THREADS;
    __shared__ float red[4][32];
    __shared__ float sh[4];
    float a0 = 0.f, a1 = 0.f;
    for (int k = tid; k < fd; k += nt) {
        a0 = __fadd_rn(a0, in0(k));
        a1 = __fadd_rn(a1, in1(k));
    }
    a0 = warp_sum(a0);
    a1 = warp_sum(a1);
    if ((tid & 31) == 0) {
        red[0][tid >> 5] = a0;
        red[1][tid >> 5] = a1;
    }
    __syncthreads();
    if (tid == 0) {
        float x0 = 0.f, x1 = 0.f;
        for (int w = 0; w < nt / 32; ++w) {
            x0 = __fadd_rn(x0, red[0][w]);
            x1 = __fadd_rn(x1, red[1][w]);
        }
        sh[0] = __fdiv_rn(x0, (float)fd);
        sh[1] = __fdiv_rn(x1, (float)fd);
    }
    __syncthreads();
    const float mu0 = sh[0], mu1 = sh[1];
    float v0 = 0.f, v1 = 0.f;
    for (int k = tid; k < fd; k += nt) {
        const float d0 = __fsub_rn(in0(k), mu0), d1 = __fsub_rn(in1(k), mu1);
        v0 = __fadd_rn(v0, __fmul_rn(d0, d0));
        v1 = __fadd_rn(v1, __fmul_rn(d1, d1));
    }
    v0 = warp_sum(v0);
    v1 = warp_sum(v1);
    if ((tid & 31) == 0) {
        red[2][tid >> 5] = v0;
        red[3][tid >> 5] = v1;
    }
    __syncthreads();
    if (tid == 0) {
        float x0 = 0.f, x1 = 0.f;
        for (int w = 0; w < nt / 32; ++w) {
            x0 = __fadd_rn(x0, red[2][w]);
            x1 = __fadd_rn(x1, red[3][w]);
        }
        sh[2] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(x0, (float)fd), 1e-5f)));
        sh[3] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(x1, (float)fd), 1e-5f)));
    }
    __syncthreads();
    stat[0] = mu0;
    stat[1] = mu1;
    stat[2] = sh[2];
    stat[3] = sh[3];
}

// fc1 dot product of hidden unit u with one LayerNorm'd input row, as lane `lane` of a warp: the lane adds
// w1[u][k] * ln(k) over k = lane, lane + 32, ... in increasing k, then the warp sums by butterfly.  Callers that
// tile k or tokens keep this per-lane order, so every path gives the same bits.
__device__ __forceinline__ float sc_fc1_term(float acc, float wk, float lnk) { return __fadd_rn(acc, __fmul_rn(wk, lnk)); }

// fc1 pre-activations of the raw features (in0) and the habituated ones (in1) for hidden units [u0, u0 + 8): one
// 256-thread CTA, one warp per unit.  z0[u], z1[u] receive fc1 outputs plus bias.  in0(k) / in1(k) return feature k.
template <class In0, class In1>
__device__ void scorer_fc1_block(const ModelDev &m, int fd, const In0 &in0, const In1 &in1, int u0, float *z0,
                                 float *z1) {
    float st[4];
    scorer_ln_stats_block(fd, in0, in1, st);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int u = u0 + warp;
    if (u >= m.seg_hidden) return;
    const float *w1 = m.sc_w1 + (size_t)u * fd;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 4
    for (int k = lane; k < fd; k += 32) {   // unrolled: the loads of 4 steps in flight, the sums still in k order
        const float lw = m.sc_ln_w[k], lb = m.sc_ln_b[k], wk = w1[k];
        s0 = sc_fc1_term(s0, wk, sc_ln(in0(k), st[0], st[2], lw, lb));
        s1 = sc_fc1_term(s1, wk, sc_ln(in1(k), st[1], st[3], lw, lb));
    }
    s0 = warp_sum(s0);
    s1 = warp_sum(s1);
    if (lane == 0) {
        z0[u] = __fadd_rn(s0, m.sc_b1[u]);
        z1[u] = __fadd_rn(s1, m.sc_b1[u]);
    }
}

__device__ __forceinline__ bool sc_contains(const uint8_t *buf, int n, const char *lit, int ln) {
    for (int i = 0; i + ln <= n; ++i) {
        int k = 0;
        while (k < ln && buf[i + k] == (uint8_t)lit[k]) ++k;
        if (k == ln) return true;
    }
    return false;
}

// GELU + fc2 of both pre-activation rows, the habituated score (ready: the stream's EMA existed before this token)
// and the authority-spoof quarantine over the last <= 24 tokens ending at `pos` (src/vault_v3_model.py:1795-1817);
// returns the token's score on thread 0 (one 256-thread CTA).
__device__ inline float scorer_score_block(const ModelDev &m, const StateDev &s, int b, const SeqCtl &q, const float *z0,
                                    const float *z1, bool ready, int64_t pos) {
    const int tid = threadIdx.x, nt = SCORER_THREADS, hd = m.seg_hidden;
    __shared__ float red[2][32];
    __shared__ uint8_t buf[4096];
    float r0 = 0.f, r1 = 0.f;
    for (int u = tid; u < hd; u += nt) {
        const float a = z0[u], c = z1[u];
        const float g0 = __fmul_rn(__fmul_rn(0.5f, a), __fadd_rn(1.0f, erff(__fmul_rn(a, 0.70710678118654752f))));
        const float g1 = __fmul_rn(__fmul_rn(0.5f, c), __fadd_rn(1.0f, erff(__fmul_rn(c, 0.70710678118654752f))));
        r0 = __fadd_rn(r0, __fmul_rn(m.sc_w2[u], g0));
        r1 = __fadd_rn(r1, __fmul_rn(m.sc_w2[u], g1));
    }
    r0 = warp_sum(r0);
    r1 = warp_sum(r1);
    if ((tid & 31) == 0) {
        red[0][tid >> 5] = r0;
        red[1][tid >> 5] = r1;
    }
    __syncthreads();
    float sc = 0.f;
    if (tid == 0) {
        float raw = 0.f, hab = 0.f;
        for (int w = 0; w < nt / 32; ++w) {
            raw = __fadd_rn(raw, red[0][w]);
            hab = __fadd_rn(hab, red[1][w]);
        }
        raw = __fadd_rn(raw, m.sc_b2[0]);
        hab = __fadd_rn(hab, m.sc_b2[0]);
        sc = raw;
        if (ready && hab > raw) sc = __fadd_rn(raw, __fmul_rn(0.35f, __fsub_rn(hab, raw)));
        const int W = m.W, c = (int)(pos % W), par = (int)((pos / W) & 1);
        if (q.n_pin > m.n_sink && pos >= q.n_pin) {
            int lb = (int)min((int64_t)24, pos - q.n_pin + 1);
            const int avail_cur = c + 1;
            lb = min(lb, pos >= W ? W + avail_cur : avail_cur);
            const int need_prev = avail_cur < lb ? lb - avail_cur : 0;
            const int cur_start = avail_cur > lb ? avail_cur - lb : 0;
            int n = 0;
            for (int k = 0; k < need_prev + (c + 1 - cur_start); ++k) {
                const int tk = k < need_prev ? s.tok_ring[((size_t)b * 2 + (par ^ 1)) * W + (W - need_prev + k)]
                                             : s.tok_ring[((size_t)b * 2 + par) * W + cur_start + (k - need_prev)];
                const uint32_t off = m.tok_off[tk];
                const int len = m.tok_len[tk];
                for (int i = 0; i < len && n < 4096; ++i) {
                    const uint8_t ch = m.tok_pool[off + i];
                    buf[n++] = (ch >= 0x41 && ch <= 0x5A) ? (uint8_t)(ch + 32) : ch;
                }
            }
            if (sc_contains(buf, n, "opi_signed_directive", 20) || sc_contains(buf, n, "urgent opi delegation", 21))
                sc = -1.0e30f;
        }
    }
    return sc;
}

}  // namespace v3g
