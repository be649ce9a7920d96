// Decode attention work item (split-KV flash-decode over [sink | segment bank | prev chunk | cur chunk]).
//
// Reference: VAULTv3Attention.step (src/vault_v3_model.py:1072-1139) and attn_run (runtime/vault3.c:1967-2032):
// softmax(q . k / sqrt(D)) v over S pinned sinks (rotated to -(M+S)..-(M+1)), M bank keys (rotated to -M..-1),
// the W keys of the previous chunk and the c+1 keys of the current chunk, GQA group H/G query heads per KV head.
// Window keys are stored rotated at their position inside their chunk; `q_cur` (query at position c) scores keys of
// the current chunk and `q_far` (query at W + c) all others, which reproduces the reference's relative positions.
#pragma once
#include "v3g.cuh"

namespace v3g {

constexpr int ATT_GRP_MAX = 8;
constexpr int ATT_KPC = ATT_KEYS_PER_CTA;

struct KeySpan {   // visible keys of one (sequence, step)
    int n_sk, n_seg, n_prev, n_cur, total, par, bank_par;
};

__device__ __forceinline__ KeySpan key_span(const StateDev &s, int b, int64_t pos) {
    const int W = s.W, c = (int)(pos % W);
    const SeqCtl &q = s.seq[b];
    KeySpan k;
    const int n_pin = __ldcg(&q.n_pin), seg_on = __ldcg(&q.seg_on), budget = __ldcg(&q.seg_budget);
    k.n_sk = pos >= 2 * W ? n_pin : 0;
    k.n_seg = (pos >= 2 * W && seg_on && budget > 0) ? __ldcg(&q.mem_cnt) : 0;
    k.n_prev = pos >= W ? W : 0;
    k.n_cur = c + 1;
    k.total = k.n_sk + k.n_seg + k.n_prev + k.n_cur;
    k.par = (int)((pos / W) & 1);
    k.bank_par = __ldcg(&q.bank_par);
    return k;
}

// key (value = false) or value row of visible key j; `far` = scored with the query at W + c
__device__ __forceinline__ const kv_t *kv_row(const StateDev &s, int layer, int b, int g, const KeySpan &ks,
                                                       int j, bool value, bool &far) {
    far = true;
    if (j < ks.n_sk) return kvp(s, layer, b, sink_off(s, value ? 2 : 1, g, j));           // sink v / k_rot
    j -= ks.n_sk;
    if (j < ks.n_seg) return kvp(s, layer, b, value ? bank_off(s, ks.bank_par, 1, g, j) : bank_rot_off(s, g, j));
    j -= ks.n_seg;
    if (j < ks.n_prev) return kvp(s, layer, b, ring_off(s, ks.par ^ 1, value ? 2 : 0, g, j));   // ring v / k_rot
    j -= ks.n_prev;
    far = false;
    return kvp(s, layer, b, ring_off(s, ks.par, value ? 2 : 0, g, j));
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}

template <int D>
struct AttnSmem {
    kv_t k[ATT_KPC * (D + 8)];   // padded K rows: conflict-free 16-byte reads across rows
    kv_t v[ATT_KPC * D];
    float q[2][ATT_GRP_MAX][D];           // [far / cur][head][dim]
    float p[ATT_GRP_MAX][ATT_KPC];
    float m[ATT_GRP_MAX], l[ATT_GRP_MAX];
    unsigned char far[ATT_KPC];
    int last;
};

// One work item = ATT_KPC keys of one (sequence b, KV head g) for its `grp` query heads, run by one CTA.
// All K and V rows of the chunk are staged in shared memory with cp.async (one round trip), up to four threads
// score a key (a slice of the head vector each), one warp per head forms the chunk's softmax pieces, and every
// thread accumulates a column pair of every head over a quarter of the keys.  The CTA writes an unnormalised partial (o, m, l); the last CTA of (b, g) merges the
// partials in split order into s.attn.  ks = key_span(s, b, pos).  Returns false when the split is empty.
template <int D>
__device__ bool attn_item(const StateDev &s, const KeySpan &ks, int layer, float scale, int split, int g, int b,
                          int64_t pos, AttnSmem<D> &sm, int nt) {
    constexpr int KP = D + 8, CH = D / 8;
    const int H = s.H, G = s.G, grp = H / G;
    const int n_splits = (ks.total + ATT_KPC - 1) / ATT_KPC;
    if (split >= n_splits) return false;
    const int j0 = split * ATT_KPC, nk = min(ATT_KPC, ks.total - j0);
    const int tid = threadIdx.x;
    for (int c = tid; c < nk * CH; c += nt) {
        const int j = c / CH, part = c - j * CH;
        bool far;
        const kv_t *kr = kv_row(s, layer, b, g, ks, j0 + j, false, far);
        const kv_t *vr = kv_row(s, layer, b, g, ks, j0 + j, true, far);
        cp_async16(&sm.k[j * KP + part * 8], kr + part * 8);
        cp_async16(&sm.v[j * D + part * 8], vr + part * 8);
        if (part == 0) sm.far[j] = far ? 1 : 0;
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int idx = tid; idx < grp * D; idx += nt) {
        const int hr = idx / D, dd = idx - hr * D;
        const size_t qo = ((size_t)b * H + g * grp + hr) * D + dd;
        sm.q[1][hr][dd] = __ldcg(&s.q_cur[qo]);
        sm.q[0][hr][dd] = pos >= s.W ? __ldcg(&s.q_far[qo]) : 0.f;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    sync_threads(nt);
    // scores: QT adjacent threads share key j, each a DQ-wide slice of the head vector; slices meet by shuffles
    {
        int QT = nt / ATT_KPC < D / 8 ? nt / ATT_KPC : D / 8;   // 1, 2 or 4 threads per key
        QT = QT >= 4 ? 4 : (QT >= 2 ? 2 : 1);
        const int DQ = D / QT;
        const int j = tid / QT, qi = tid - j * QT;
        float acc[ATT_GRP_MAX];
#pragma unroll
        for (int hr = 0; hr < ATT_GRP_MAX; ++hr) acc[hr] = 0.f;
        if (j < nk && j < ATT_KPC) {
            const float(*qs)[D] = sm.q[sm.far[j] ? 0 : 1];
            const kv_t *kr = &sm.k[j * KP + qi * DQ];
            for (int d0 = 0; d0 < DQ; d0 += 8) {
                const uint4 raw = *reinterpret_cast<const uint4 *>(kr + d0);
                const __half2 *k2 = reinterpret_cast<const __half2 *>(&raw);
                float kf[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(k2[e]);
                    kf[2 * e] = f.x;
                    kf[2 * e + 1] = f.y;
                }
                const int dd = qi * DQ + d0;
#pragma unroll
                for (int hr = 0; hr < ATT_GRP_MAX; ++hr) {
                    if (hr < grp) {
                        const float4 qa = *reinterpret_cast<const float4 *>(&qs[hr][dd]);
                        const float4 qb = *reinterpret_cast<const float4 *>(&qs[hr][dd + 4]);
                        float s0 = qa.x * kf[0], s1 = qa.y * kf[1];
                        s0 = fmaf(qa.z, kf[2], s0);
                        s1 = fmaf(qa.w, kf[3], s1);
                        s0 = fmaf(qb.x, kf[4], s0);
                        s1 = fmaf(qb.y, kf[5], s1);
                        s0 = fmaf(qb.z, kf[6], s0);
                        s1 = fmaf(qb.w, kf[7], s1);
                        acc[hr] += s0 + s1;
                    }
                }
            }
        }
#pragma unroll
        for (int hr = 0; hr < ATT_GRP_MAX; ++hr) {
            float tot = acc[hr];
            for (int o = 1; o < QT; o <<= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
            if (hr < grp && qi == 0 && j < nk && j < ATT_KPC) sm.p[hr][j] = tot * scale;
        }
    }
    sync_threads(nt);
    const int warp = tid >> 5, lane = tid & 31;
    for (int hr = warp; hr < grp; hr += nt / 32) {
        float mx = -INFINITY;
        for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, sm.p[hr][j]);
        mx = warp_max(mx);
        float l = 0.f;
        for (int j = lane; j < nk; j += 32) {
            const float p = expf(sm.p[hr][j] - mx);
            sm.p[hr][j] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) {
            sm.m[hr] = mx;
            sm.l[hr] = l;
        }
    }
    sync_threads(nt);
    // output: thread (column pair c2, key quarter kq) sums its keys for every head; quarters meet in shared memory
    // (the K rows are no longer needed: their space holds the quarter sums)
    {
        constexpr int P2 = D / 2;
        const int KQ = nt / P2 >= 4 ? 4 : (nt / P2 >= 2 ? 2 : 1);
        const int c2 = tid % P2, kq = tid / P2;
        float o[ATT_GRP_MAX][2];
#pragma unroll
        for (int hr = 0; hr < ATT_GRP_MAX; ++hr) o[hr][0] = o[hr][1] = 0.f;
        if (kq < KQ) {
            for (int jj = kq; jj < nk; jj += KQ) {
                const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&sm.v[jj * D + 2 * c2]));
#pragma unroll
                for (int hr = 0; hr < ATT_GRP_MAX; ++hr) {
                    if (hr < grp) {
                        const float pj = sm.p[hr][jj];
                        o[hr][0] = fmaf(pj, v.x, o[hr][0]);
                        o[hr][1] = fmaf(pj, v.y, o[hr][1]);
                    }
                }
            }
        }
        sync_threads(nt);   // every thread is done with the K rows
        float *red = reinterpret_cast<float *>(sm.k);   // [KQ][grp][D]
        if (kq < KQ) {
#pragma unroll
            for (int hr = 0; hr < ATT_GRP_MAX; ++hr)
                if (hr < grp) *reinterpret_cast<float2 *>(&red[(kq * grp + hr) * D + 2 * c2]) = make_float2(o[hr][0], o[hr][1]);
        }
        sync_threads(nt);
        for (int idx = tid; idx < grp * D; idx += nt) {
            const int hr = idx / D, dd = idx - hr * D;
            float acc = 0.f;
            for (int q = 0; q < KQ; ++q) acc += red[(q * grp + hr) * D + dd];
            sm.q[0][hr][dd] = acc;   // the query rows are no longer needed either: reuse them for the output
        }
        sync_threads(nt);
    }
    if (n_splits == 1) {   // the whole span in one item: normalise and write the head outputs directly
        for (int idx = tid; idx < grp * D; idx += nt) {
            const int hr = idx / D, dd = idx - hr * D;
            s.attn[((size_t)b * H + g * grp + hr) * D + dd] = sm.q[0][hr][dd] / sm.l[hr];
        }
        sync_threads(nt);
        return true;
    }
    float *part = s.att_part + ((((size_t)b * G + g) * s.max_splits + split) * grp) * (D + 2);
    for (int idx = tid; idx < grp * D; idx += nt) {
        const int hr = idx / D, dd = idx - hr * D;
        part[hr * (D + 2) + dd] = sm.q[0][hr][dd];
    }
    if (tid < grp) {
        part[tid * (D + 2) + D] = sm.m[tid];
        part[tid * (D + 2) + D + 1] = sm.l[tid];
    }
    __threadfence();
    sync_threads(nt);
    if (tid == 0) sm.last = atomicAdd(&s.att_cnt[b * G + g], 1u) == (uint32_t)(n_splits - 1);
    sync_threads(nt);
    if (sm.last) {
        __threadfence();
        const float *p0 = s.att_part + (((size_t)b * G + g) * s.max_splits) * grp * (D + 2);
        for (int idx = tid; idx < grp * D; idx += nt) {
            const int hr = idx / D, dd = idx - hr * D;
            float M = -INFINITY;
            for (int sp2 = 0; sp2 < n_splits; ++sp2) M = fmaxf(M, __ldcg(&p0[((size_t)sp2 * grp + hr) * (D + 2) + D]));
            float L = 0.f, O = 0.f;
            for (int sp2 = 0; sp2 < n_splits; ++sp2) {
                const float *pp = p0 + ((size_t)sp2 * grp + hr) * (D + 2);
                const float w = expf(__ldcg(&pp[D]) - M);
                L = fmaf(__ldcg(&pp[D + 1]), w, L);
                O = fmaf(__ldcg(&pp[dd]), w, O);
            }
            s.attn[((size_t)b * H + g * grp + hr) * D + dd] = O / L;
        }
        if (tid == 0) s.att_cnt[b * G + g] = 0u;
    }
    sync_threads(nt);
    return true;
}

}  // namespace v3g
