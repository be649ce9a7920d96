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

// K and V row bases of the visible key segments of (layer, sequence b, KV head g) -- sinks, segment bank, previous
// chunk, current chunk, each [rows][D] -- and the cumulative key counts: computed once per work item, so the copy
// loops do plain pointer arithmetic instead of re-reading the state descriptor around every cp.async
struct KvRows {
    const kv_t *k[4], *v[4];
    int end[4];
};
__device__ __forceinline__ KvRows kv_rows(const StateDev &s, int layer, int b, int g, const KeySpan &ks) {
    KvRows r;
    r.k[0] = kvp(s, layer, b, sink_off(s, 1, g, 0));                    // rotated sink keys
    r.v[0] = kvp(s, layer, b, sink_off(s, 2, g, 0));
    r.k[1] = kvp(s, layer, b, bank_rot_off(s, g, 0));                   // rotated bank keys
    r.v[1] = kvp(s, layer, b, bank_off(s, ks.bank_par, 1, g, 0));
    r.k[2] = kvp(s, layer, b, ring_off(s, ks.par ^ 1, 0, g, 0));        // previous chunk (rotated keys)
    r.v[2] = kvp(s, layer, b, ring_off(s, ks.par ^ 1, 2, g, 0));
    r.k[3] = kvp(s, layer, b, ring_off(s, ks.par, 0, g, 0));            // current chunk
    r.v[3] = kvp(s, layer, b, ring_off(s, ks.par, 2, g, 0));
    r.end[0] = ks.n_sk;
    r.end[1] = r.end[0] + ks.n_seg;
    r.end[2] = r.end[1] + ks.n_prev;
    r.end[3] = ks.total;
    return r;
}
// the row of visible key j (the same rows as kv_row)
template <int D>
__device__ __forceinline__ const kv_t *kv_at(const KvRows &r, int j, bool value) {
    const kv_t *base = value ? r.v[0] : r.k[0];
    int j0 = 0;
    if (j >= r.end[0]) {
        base = value ? r.v[1] : r.k[1];
        j0 = r.end[0];
    }
    if (j >= r.end[1]) {
        base = value ? r.v[2] : r.k[2];
        j0 = r.end[1];
    }
    if (j >= r.end[2]) {
        base = value ? r.v[3] : r.k[3];
        j0 = r.end[2];
    }
    return base + (size_t)(j - j0) * D;
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}

template <int D>
struct AttnSmem {
    kv_t k[ATT_KPC * (D + 8)];   // K rows, padded so the tensor-core fragment reads hit distinct banks
    kv_t v[ATT_KPC * (D + 8)];   // V rows, padded likewise; rows past the span are zero
    __half qa[2][2][ATT_GRP_MAX][D + 8];    // [far / cur query][high / low fp16 part][head][dim]
    float p[ATT_GRP_MAX][ATT_KPC];          // scaled scores
    __half pa[2][ATT_GRP_MAX][ATT_KPC + 8]; // [high / low part][head][key]: probabilities exp(s - m)
    float m[ATT_GRP_MAX], l[ATT_GRP_MAX];
    int last;
};

__device__ __forceinline__ uint32_t ld_h2(const __half *p) { return *reinterpret_cast<const uint32_t *>(p); }

// two 8x8 fp16 matrices from shared memory, transposed: lanes 0-7 give the rows of the first, lanes 8-15 of the
// second; thread (g, t) receives elements (rows 2t, 2t+1; column g) of each
__device__ __forceinline__ void ldsm_x2_trans(uint32_t &r0, uint32_t &r1, const void *p) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(a));
}

// fp32 value as high + low fp16 parts (about 22 significant bits together)
__device__ __forceinline__ void split_half(float v, __half &hi, __half &lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

// 8 consecutive attention outputs e0 .. e0 + 7 of sequence b (inside one head: e0 = head * D + dd, dd a multiple
// of 8), merged from the n_splits (2 .. ATT_MERGE_MAX) unnormalised partials of the head's KV group in split
// order, with the arithmetic of attn_item's last-CTA merge (same results, bit for bit).  Out of line: inlined into
// the unrolled prologue, the partials of several items crowd its registers.
template <int D>
__device__ __noinline__ void attn_merged8(const StateDev &s, int b, int e0, int n_splits, float (&v)[8]) {
    constexpr int PS = att_part_stride(D);
    const int grp = s.H / s.G, head = e0 / D, dd = e0 - head * D, g = head / grp, hr = head - g * grp;
    const float *p0 = s.att_part + ((((size_t)b * s.G + g) * s.max_splits) * grp + hr) * PS;
    float4 o[ATT_MERGE_MAX][2];
    float2 ml[ATT_MERGE_MAX];
#pragma unroll
    for (int sp = 0; sp < ATT_MERGE_MAX; ++sp) {   // every load in flight at once
        if (sp < n_splits) {
            const float *pp = p0 + (size_t)sp * grp * PS;
            o[sp][0] = __ldcg(reinterpret_cast<const float4 *>(pp + dd));
            o[sp][1] = __ldcg(reinterpret_cast<const float4 *>(pp + dd + 4));
            ml[sp] = __ldcg(reinterpret_cast<const float2 *>(pp + D));
        }
    }
    float M = -INFINITY;
#pragma unroll
    for (int sp = 0; sp < ATT_MERGE_MAX; ++sp)
        if (sp < n_splits) M = fmaxf(M, ml[sp].x);
    float L = 0.f, O[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int sp = 0; sp < ATT_MERGE_MAX; ++sp) {
        if (sp < n_splits) {
            const float w = expf(ml[sp].x - M);
            L = fmaf(ml[sp].y, w, L);
            const float ov[8] = {o[sp][0].x, o[sp][0].y, o[sp][0].z, o[sp][0].w,
                                 o[sp][1].x, o[sp][1].y, o[sp][1].z, o[sp][1].w};
#pragma unroll
            for (int j = 0; j < 8; ++j) O[j] = fmaf(ov[j], w, O[j]);
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = O[j] / L;
}

// Last-CTA merge of the n_splits unnormalised partials (o, m, l) of (sequence b, KV group g) into s.attn, in split
// order: out = sum_sp o_sp exp(m_sp - M) / sum_sp l_sp exp(m_sp - M), M = max_sp m_sp.  The (m, l) pairs are staged
// in shared memory first (spans of up to ATT_KPC splits; longer ones read them from global memory), then each thread
// produces four output dims of one head with the o loads of 8 splits in flight at a time (the merge of a long span
// is otherwise one dependent L2 round trip per split).  The per-output arithmetic is the same fma chain in split
// order whatever the load schedule.  The K buffer of sm is free here and holds the staged l values.
template <int D>
__device__ void attn_merge_splits(const StateDev &s, int b, int g, int n_splits, AttnSmem<D> &sm, int nt) {
    constexpr int PS = att_part_stride(D);
    const int H = s.H, G = s.G, grp = H / G, tid = threadIdx.x;
    const float *p0 = s.att_part + (((size_t)b * G + g) * s.max_splits) * grp * PS;
    const bool staged = n_splits <= ATT_KPC;
    float *ms = &sm.p[0][0], *ls = reinterpret_cast<float *>(sm.k);
    static_assert(sizeof(AttnSmem<D>::k) >= ATT_GRP_MAX * ATT_KPC * sizeof(float), "l staging fits the K buffer");
    if (staged)
        for (int i = tid; i < grp * n_splits; i += nt) {
            const int hr = i / n_splits, sp = i - hr * n_splits;
            const float2 ml = __ldcg(reinterpret_cast<const float2 *>(p0 + ((size_t)sp * grp + hr) * PS + D));
            ms[hr * ATT_KPC + sp] = ml.x;
            ls[hr * ATT_KPC + sp] = ml.y;
        }
    sync_threads(nt);
    auto m_of = [&](int hr, int sp) { return staged ? ms[hr * ATT_KPC + sp] : __ldcg(p0 + ((size_t)sp * grp + hr) * PS + D); };
    auto l_of = [&](int hr, int sp) {
        return staged ? ls[hr * ATT_KPC + sp] : __ldcg(p0 + ((size_t)sp * grp + hr) * PS + D + 1);
    };
    for (int idx = tid; idx < grp * (D / 4); idx += nt) {
        const int hr = idx / (D / 4), dd = 4 * (idx - hr * (D / 4));
        float M = -INFINITY;
        for (int sp = 0; sp < n_splits; ++sp) M = fmaxf(M, m_of(hr, sp));
        float L = 0.f, O[4] = {0.f, 0.f, 0.f, 0.f};
        for (int sp0 = 0; sp0 < n_splits; sp0 += 8) {
            float4 o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (sp0 + j < n_splits)
                    o[j] = __ldcg(reinterpret_cast<const float4 *>(p0 + ((size_t)(sp0 + j) * grp + hr) * PS + dd));
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (sp0 + j < n_splits) {
                    const float w = expf(m_of(hr, sp0 + j) - M);
                    L = fmaf(l_of(hr, sp0 + j), w, L);
                    O[0] = fmaf(o[j].x, w, O[0]);
                    O[1] = fmaf(o[j].y, w, O[1]);
                    O[2] = fmaf(o[j].z, w, O[2]);
                    O[3] = fmaf(o[j].w, w, O[3]);
                }
            }
        }
        *reinterpret_cast<float4 *>(&s.attn[((size_t)b * H + g * grp + hr) * D + dd]) =
            make_float4(O[0] / L, O[1] / L, O[2] / L, O[3] / L);
    }
}

// One work item = ATT_KPC keys of one (sequence b, KV head g) for its `grp` query heads, run by one CTA on the
// tensor cores.  All K and V rows of the chunk are staged in shared memory with cp.async (one round trip).  Scores:
// for each block of 8 keys, mma steps over the head dimension with A = the group's queries (rows 0-7 their high
// fp16 parts, rows 8-15 the low parts) and B = the K rows, so each head's dot is the sum of two accumulator rows
// (about fp32 accuracy with fp16 keys).  Keys of the current chunk are scored with the query at position c, the
// others with the query at W + c (both kinds only where a key block holds both).  One warp per head forms the
// softmax pieces (m, l, p), and P V runs the same way: A = probabilities split high / low, B = V read transposed
// with ldmatrix.  The CTA writes an unnormalised partial (o, m, l); the last CTA of (b, g) merges the partials in
// split order into s.attn.  With defer_merge (the persistent kernel) a span of at most ATT_MERGE_MAX splits is
// left as partials, which the next phase's activation prologue merges the same way (attn_merged8).
// ks = key_span(s, b, pos).  Returns false when the split is empty.
template <int D>
__device__ bool attn_item(const StateDev &s, const KeySpan &ks, int layer, float scale, int split, int g, int b,
                          int64_t pos, AttnSmem<D> &sm, int nt, bool defer_merge = false) {
    constexpr int KP = D + 8, CH = D / 8, PS = att_part_stride(D);
    static_assert(D % 16 == 0 && ATT_KPC % 16 == 0, "mma shapes");
    const int H = s.H, G = s.G, grp = H / G;
    const int n_splits = (ks.total + ATT_KPC - 1) / ATT_KPC;
    if (split >= n_splits) return false;
    const int j0 = split * ATT_KPC, nk = min(ATT_KPC, ks.total - j0);
    const int nfar = ks.n_sk + ks.n_seg + ks.n_prev - j0;   // keys j < nfar are scored with the far query
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarp = nt >> 5;
    const int gq = lane >> 2, t = lane & 3;
    for (int c = tid; c < ATT_KPC * CH; c += nt) {
        const int j = c / CH, part = c - j * CH;
        if (j < nk) {
            bool far;
            cp_async16(&sm.k[j * KP + part * 8], kv_row(s, layer, b, g, ks, j0 + j, false, far) + part * 8);
            cp_async16(&sm.v[j * KP + part * 8], kv_row(s, layer, b, g, ks, j0 + j, true, far) + part * 8);
        } else {   // past the span: probability 0 must meet a finite value
            *reinterpret_cast<uint4 *>(&sm.v[j * KP + part * 8]) = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int idx = tid; idx < 2 * ATT_GRP_MAX * D / 4; idx += nt) {   // queries, four dims per item
        const int w = idx / (ATT_GRP_MAX * D / 4), r = idx - w * (ATT_GRP_MAX * D / 4);
        const int hr = r / (D / 4), dd = 4 * (r - hr * (D / 4));
        float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
        if (hr < grp && (w == 1 || pos >= s.W)) {
            const size_t qo = ((size_t)b * H + g * grp + hr) * D + dd;
            q = __ldcg(reinterpret_cast<const float4 *>((w ? s.q_cur : s.q_far) + qo));
        }
        const float qv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) split_half(qv[e], sm.qa[w][0][hr][dd + e], sm.qa[w][1][hr][dd + e]);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    sync_threads(nt);
    // scores of the key blocks kb = warp, warp + nwarp, ...: lane (gq, t) ends with head gq, keys 8 kb + 2t (+1)
    for (int kb = warp; kb * 8 < nk; kb += nwarp) {
        const int key0 = kb * 8;
        const bool any_far = key0 < nfar, any_cur = key0 + 8 > nfar;   // warp-uniform
        float cf[4] = {0.f, 0.f, 0.f, 0.f}, cc[4] = {0.f, 0.f, 0.f, 0.f};
        const kv_t *krow = &sm.k[(key0 + gq) * KP + 2 * t];
#pragma unroll
        for (int k16 = 0; k16 < D / 16; ++k16) {
            const uint32_t b0 = ld_h2(krow + 16 * k16), b1 = ld_h2(krow + 16 * k16 + 8);
            const int qc = 16 * k16 + 2 * t;
            if (any_far)
                mma16816(cf, ld_h2(&sm.qa[0][0][gq][qc]), ld_h2(&sm.qa[0][1][gq][qc]), ld_h2(&sm.qa[0][0][gq][qc + 8]),
                         ld_h2(&sm.qa[0][1][gq][qc + 8]), b0, b1);
            if (any_cur)
                mma16816(cc, ld_h2(&sm.qa[1][0][gq][qc]), ld_h2(&sm.qa[1][1][gq][qc]), ld_h2(&sm.qa[1][0][gq][qc + 8]),
                         ld_h2(&sm.qa[1][1][gq][qc + 8]), b0, b1);
        }
        if (gq < grp) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int j = key0 + 2 * t + e;
                const float sc = (j < nfar ? cf[e] + cf[2 + e] : cc[e] + cc[2 + e]) * scale;
                sm.p[gq][j] = j < nk ? sc : -INFINITY;
            }
        }
    }
    sync_threads(nt);
    // softmax pieces, one warp per head: m = max score, p = exp(s - m) (as fp16 high / low parts), l = sum of p
    for (int hr = warp; hr < ATT_GRP_MAX; hr += nwarp) {
        if (hr < grp) {
            float mx = -INFINITY;
            for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, sm.p[hr][j]);
            mx = warp_max(mx);
            float l = 0.f;
            for (int j = lane; j < ATT_KPC; j += 32) {
                const float p = j < nk ? expf(sm.p[hr][j] - mx) : 0.f;
                split_half(p, sm.pa[0][hr][j], sm.pa[1][hr][j]);
                l += p;
            }
            l = warp_sum(l);
            if (lane == 0) {
                sm.m[hr] = mx;
                sm.l[hr] = l;
            }
        } else {
            for (int j = lane; j < ATT_KPC; j += 32) sm.pa[0][hr][j] = sm.pa[1][hr][j] = __float2half_rn(0.f);
        }
    }
    sync_threads(nt);
    // P V for the 8-column blocks nb = warp, warp + nwarp, ...: lane (gq, t) ends with head gq, columns 8 nb + 2t (+1)
    const int nk16 = (nk + 15) / 16;
    float *part = n_splits == 1 ? nullptr : s.att_part + ((((size_t)b * G + g) * s.max_splits + split) * grp) * PS;
    for (int nb = warp; nb < D / 8; nb += nwarp) {
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k16 = 0; k16 < nk16; ++k16) {
            uint32_t b0, b1;
            ldsm_x2_trans(b0, b1, &sm.v[(16 * k16 + (lane & 15)) * KP + 8 * nb]);
            const int pc = 16 * k16 + 2 * t;
            mma16816(c, ld_h2(&sm.pa[0][gq][pc]), ld_h2(&sm.pa[1][gq][pc]), ld_h2(&sm.pa[0][gq][pc + 8]),
                     ld_h2(&sm.pa[1][gq][pc + 8]), b0, b1);
        }
        if (gq < grp) {
            const int dd = 8 * nb + 2 * t;
            const float o0 = c[0] + c[2], o1 = c[1] + c[3];
            if (!part) {   // the whole span in one item: normalise and write the head outputs directly
                const float inv = 1.f / sm.l[gq];
                *reinterpret_cast<float2 *>(&s.attn[((size_t)b * H + g * grp + gq) * D + dd]) = make_float2(o0 * inv, o1 * inv);
            } else {
                *reinterpret_cast<float2 *>(&part[gq * PS + dd]) = make_float2(o0, o1);
            }
        }
    }
    if (!part) {
        sync_threads(nt);
        return true;
    }
    if (tid < grp) *reinterpret_cast<float2 *>(&part[tid * PS + D]) = make_float2(sm.m[tid], sm.l[tid]);
    if (defer_merge && n_splits <= ATT_MERGE_MAX) {   // the reader merges (its phase starts after a grid barrier)
        sync_threads(nt);
        return true;
    }
    __threadfence();
    sync_threads(nt);
    if (tid == 0) sm.last = atomicAdd(&s.att_cnt[b * G + g], 1u) == (uint32_t)(n_splits - 1);
    sync_threads(nt);
    if (sm.last) {
        __threadfence();
        const float *p0 = s.att_part + (((size_t)b * G + g) * s.max_splits) * grp * PS;
        for (int idx = tid; idx < grp * D; idx += nt) {
            const int hr = idx / D, dd = idx - hr * D;
            float M = -INFINITY;
            for (int sp2 = 0; sp2 < n_splits; ++sp2) M = fmaxf(M, __ldcg(&p0[((size_t)sp2 * grp + hr) * PS + D]));
            float L = 0.f, O = 0.f;
            for (int sp2 = 0; sp2 < n_splits; ++sp2) {
                const float *pp = p0 + ((size_t)sp2 * grp + hr) * PS;
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

// ---------------------------------------------------------------------------------------------------------------
// Long splits for the per-phase decode path: one work item covers `tps` consecutive 64-key tiles of one (sequence,
// KV head) with an online softmax across them, so a batch over thousands of keys leaves a few partials per head
// (few items to merge) instead of one per 64 keys.  Tile arithmetic as in attn_item (queries and probabilities as
// high + low fp16 parts on the tensor cores, fp16 K / V); the running maximum rescales the partial output and sum.
template <int D>
struct AttnSmemSpan {
    AttnSmem<D> t;
    float alpha[ATT_GRP_MAX];   // rescale of the running output when a tile raises a head's maximum
};

template <int D>
__device__ bool attn_span(const StateDev &s, const KeySpan &ks, int layer, float scale, int split, int tps, int g, int b,
                          int64_t pos, AttnSmemSpan<D> &ss, int nt) {
    constexpr int KP = D + 8, CH = D / 8, PS = att_part_stride(D), NBW = (D / 8 + 3) / 4;
    AttnSmem<D> &sm = ss.t;
    const int H = s.H, G = s.G, grp = H / G;
    const int span = ATT_KPC * tps;
    const int n_splits = (ks.total + span - 1) / span;
    if (split >= n_splits) return false;
    const int jb = split * span, nkeys = min(span, ks.total - jb);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarp = nt >> 5;
    const int gq = lane >> 2, t = lane & 3;
    float o[NBW][4];   // this warp's output blocks nb = warp, warp + nwarp, ...
#pragma unroll
    for (int i = 0; i < NBW; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    for (int idx = tid; idx < 2 * ATT_GRP_MAX * D / 4; idx += nt) {   // queries, four dims per item
        const int w = idx / (ATT_GRP_MAX * D / 4), r = idx - w * (ATT_GRP_MAX * D / 4);
        const int hr = r / (D / 4), dd = 4 * (r - hr * (D / 4));
        float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
        if (hr < grp && (w == 1 || pos >= s.W)) {
            const size_t qo = ((size_t)b * H + g * grp + hr) * D + dd;
            q = __ldcg(reinterpret_cast<const float4 *>((w ? s.q_cur : s.q_far) + qo));
        }
        const float qv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) split_half(qv[e], sm.qa[w][0][hr][dd + e], sm.qa[w][1][hr][dd + e]);
    }
    if (tid < ATT_GRP_MAX) {
        sm.m[tid] = -INFINITY;
        sm.l[tid] = 0.f;
    }
    const KvRows kr = kv_rows(s, layer, b, g, ks);
    for (int j0 = jb; j0 < jb + nkeys; j0 += ATT_KPC) {
        const int nk = min(ATT_KPC, jb + nkeys - j0);
        const int nfar = ks.n_sk + ks.n_seg + ks.n_prev - j0;   // keys j < nfar are scored with the far query
        for (int c = tid; c < ATT_KPC * CH; c += nt) {
            const int j = c / CH, part = c - j * CH;
            if (j < nk) {
                cp_async16(&sm.k[j * KP + part * 8], kv_at<D>(kr, j0 + j, false) + part * 8);
                cp_async16(&sm.v[j * KP + part * 8], kv_at<D>(kr, j0 + j, true) + part * 8);
            } else {
                *reinterpret_cast<uint4 *>(&sm.v[j * KP + part * 8]) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        sync_threads(nt);
        for (int kb = warp; kb * 8 < nk; kb += nwarp) {
            const int key0 = kb * 8;
            const bool any_far = key0 < nfar, any_cur = key0 + 8 > nfar;
            float cf[4] = {0.f, 0.f, 0.f, 0.f}, cc[4] = {0.f, 0.f, 0.f, 0.f};
            const kv_t *krow = &sm.k[(key0 + gq) * KP + 2 * t];
#pragma unroll
            for (int k16 = 0; k16 < D / 16; ++k16) {
                const uint32_t b0 = ld_h2(krow + 16 * k16), b1 = ld_h2(krow + 16 * k16 + 8);
                const int qc = 16 * k16 + 2 * t;
                if (any_far)
                    mma16816(cf, ld_h2(&sm.qa[0][0][gq][qc]), ld_h2(&sm.qa[0][1][gq][qc]), ld_h2(&sm.qa[0][0][gq][qc + 8]),
                             ld_h2(&sm.qa[0][1][gq][qc + 8]), b0, b1);
                if (any_cur)
                    mma16816(cc, ld_h2(&sm.qa[1][0][gq][qc]), ld_h2(&sm.qa[1][1][gq][qc]), ld_h2(&sm.qa[1][0][gq][qc + 8]),
                             ld_h2(&sm.qa[1][1][gq][qc + 8]), b0, b1);
            }
            if (gq < grp) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int j = key0 + 2 * t + e;
                    const float sc = (j < nfar ? cf[e] + cf[2 + e] : cc[e] + cc[2 + e]) * scale;
                    sm.p[gq][j] = j < nk ? sc : -INFINITY;
                }
            }
        }
        sync_threads(nt);
        // online softmax, one warp per head: the tile's maximum updates the running one
        for (int hr = warp; hr < ATT_GRP_MAX; hr += nwarp) {
            if (hr < grp) {
                float mx = -INFINITY;
                for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, sm.p[hr][j]);
                mx = warp_max(mx);
                const float m_old = sm.m[hr], m_new = fmaxf(m_old, mx);
                float l = 0.f;
                for (int j = lane; j < ATT_KPC; j += 32) {
                    const float p = j < nk ? expf(sm.p[hr][j] - m_new) : 0.f;
                    split_half(p, sm.pa[0][hr][j], sm.pa[1][hr][j]);
                    l += p;
                }
                l = warp_sum(l);
                if (lane == 0) {
                    const float al = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
                    ss.alpha[hr] = al;
                    sm.l[hr] = sm.l[hr] * al + l;
                    sm.m[hr] = m_new;
                }
            } else {
                for (int j = lane; j < ATT_KPC; j += 32) sm.pa[0][hr][j] = sm.pa[1][hr][j] = __float2half_rn(0.f);
                if (lane == 0) ss.alpha[hr] = 0.f;
            }
        }
        sync_threads(nt);
        const int nk16 = (nk + 15) / 16;
        const float al = gq < grp ? ss.alpha[gq] : 0.f;
#pragma unroll
        for (int i = 0; i < NBW; ++i) {
            const int nb = warp + i * nwarp;
            if (nb >= D / 8) continue;
#pragma unroll
            for (int e = 0; e < 4; ++e) o[i][e] *= al;
            for (int k16 = 0; k16 < nk16; ++k16) {
                uint32_t b0, b1;
                ldsm_x2_trans(b0, b1, &sm.v[(16 * k16 + (lane & 15)) * KP + 8 * nb]);
                const int pc = 16 * k16 + 2 * t;
                mma16816(o[i], ld_h2(&sm.pa[0][gq][pc]), ld_h2(&sm.pa[1][gq][pc]), ld_h2(&sm.pa[0][gq][pc + 8]),
                         ld_h2(&sm.pa[1][gq][pc + 8]), b0, b1);
            }
        }
        sync_threads(nt);   // the tile buffers are refilled next
    }
    // write the split's result: direct when one split covers the span, else a partial merged by the last CTA
    float *part = n_splits == 1 ? nullptr : s.att_part + ((((size_t)b * G + g) * s.max_splits + split) * grp) * PS;
#pragma unroll
    for (int i = 0; i < NBW; ++i) {
        const int nb = warp + i * nwarp;
        if (nb >= D / 8 || gq >= grp) continue;
        const int dd = 8 * nb + 2 * t;
        const float o0 = o[i][0] + o[i][2], o1 = o[i][1] + o[i][3];
        if (!part) {
            const float inv = 1.f / sm.l[gq];
            *reinterpret_cast<float2 *>(&s.attn[((size_t)b * H + g * grp + gq) * D + dd]) = make_float2(o0 * inv, o1 * inv);
        } else {
            *reinterpret_cast<float2 *>(&part[gq * PS + dd]) = make_float2(o0, o1);
        }
    }
    if (!part) {
        sync_threads(nt);
        return true;
    }
    if (tid < grp) *reinterpret_cast<float2 *>(&part[tid * PS + D]) = make_float2(sm.m[tid], sm.l[tid]);
    __threadfence();
    sync_threads(nt);
    if (tid == 0) sm.last = atomicAdd(&s.att_cnt[b * G + g], 1u) == (uint32_t)(n_splits - 1);
    sync_threads(nt);
    if (sm.last) {   // uniform over the CTA
        __threadfence();
        attn_merge_splits<D>(s, b, g, n_splits, sm, nt);
        if (tid == 0) s.att_cnt[b * G + g] = 0u;
    }
    sync_threads(nt);
    return true;
}

}  // namespace v3g
