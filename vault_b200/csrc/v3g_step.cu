// One streaming decode step of VAULT v3 on the GPU: control, fused projections, split-KV attention over
// [sink | segment bank | prev chunk | cur chunk], MLP, segment scorer, chunk-boundary eviction, lm head.
//
// Reference semantics: src/vault_v3_model.py VAULTv3ForCausalLM.step (:2214-2311) and the C runtime v3_step
// (runtime/vault3.c:2034-2222).  RoPE re-basing (:1081-1082, :1923-1927) is realised without rotating keys at
// chunk rollovers: every window key is stored rotated at its position inside its own chunk, and the query is
// rotated twice per step -- at c for keys of the current chunk and at W + c for keys of the previous chunk, the
// sinks and the bank.  Scores depend only on position differences, which are identical to the reference's.
#include <math.h>

#include "v3g_internal.h"

namespace v3g {

constexpr int KIND_KROT = 0, KIND_KRAW = 1, KIND_V = 2;   // ring kinds
constexpr int SINK_KRAW = 0, SINK_KROT = 1, SINK_V = 2;   // sink kinds
constexpr int BANK_KRAW = 0, BANK_V = 1;                  // bank kinds

__device__ __forceinline__ int ring_par(int64_t pos, int W) { return (int)((pos / W) & 1); }

__device__ __forceinline__ bool seg_active(const SeqCtl &q) { return q.seg_on && q.seg_budget > 0; }

// element (row, k) of a re-tiled matrix with identity row order
__device__ float tile_elem(const MatW &w, int row, int k) {
    const int TK = tile_k(w.fmt);
    const int rt = row >> 3, g = row & 7, kt = k / TK, kk = k % TK;
    const int s = kk >> 4, w16 = kk & 15;
    const int t = (w16 & 7) >> 1, e = (w16 & 1) + ((w16 & 8) ? 2 : 0);
    const uint8_t *tb = w.tiles + ((size_t)rt * w.n_ktiles + kt) * tile_bytes(w.fmt);
    const int lane = 4 * g + t;
    if (w.fmt == FMT_Q8 || w.fmt == FMT_Q4) {
        const int nblk = TK / 32, blk = kk >> 5;
        const uint16_t sb = *reinterpret_cast<const uint16_t *>(tb + 512 + (g >> 1) * (2 * nblk * 2) +
                                                                 (2 * blk + (g & 1)) * 2);
        const float d = __half2float(__ushort_as_half(sb));
        if (w.fmt == FMT_Q8) return (float)(int8_t)tb[lane * 16 + 4 * s + e] * d;
        const int nib = ((e & 2) ? 1 : 0) | ((s & 1) << 1) | ((e & 1) << 2);
        const uint32_t word = *reinterpret_cast<const uint32_t *>(tb + lane * 16 + 4 * (s >> 1));
        return (float)((int)((word >> (4 * nib)) & 15u) - 8) * d;
    }
    const int off = lane * 16 + 2 * (4 * s + e);
    const uint16_t v = *reinterpret_cast<const uint16_t *>(tb + off);
    if (w.fmt == FMT_F16) return __half2float(__ushort_as_half(v));
    if (w.fmt == FMT_BF16) return __uint_as_float((uint32_t)v << 16);
    const uint16_t mv = *reinterpret_cast<const uint16_t *>(tb + 512 + off);
    const uint16_t lv = *reinterpret_cast<const uint16_t *>(tb + 1024 + off);
    return (__uint_as_float((uint32_t)v << 16) + __uint_as_float((uint32_t)mv << 16)) + __uint_as_float((uint32_t)lv << 16);
}

// ChatML system-prompt auto-pin state machine for one token (src/vault_v3_model.py:2224-2252)
__device__ void auto_pin_update(const ModelDev &m, SeqCtl &q, int64_t pos, int tid) {
    if (q.pin_locked || !q.auto_pin) return;
    const int limit = min(min(m.max_sink, m.W), m.sink_cap);
    if (pos == 0) {
        if (tid == m.im_start_id && limit >= 2) q.saw_im_start = 1;
        else q.pin_locked = 1;
    } else if (pos == 1 && q.saw_im_start) {
        if (tid != m.system_id) {
            q.saw_im_start = 0;
            q.pin_locked = 1;
        }
    } else if (q.saw_im_start && pos < limit) {
        if (q.awaiting_sys_nl) {
            const int cand = (tid == m.newline_id) ? (int)pos + 1 : (int)pos;
            q.n_pin = max(q.n_pin, cand);
            q.pin_locked = 1;
            q.awaiting_sys_nl = 0;
        } else if (tid == m.im_end_id) {
            q.n_pin = max(q.n_pin, (int)pos + 1);
            if (pos + 1 < limit) q.awaiting_sys_nl = 1;
            else q.pin_locked = 1;
        }
    } else if (pos >= limit) {
        if (q.saw_im_start && !q.awaiting_sys_nl) q.n_pin = max(q.n_pin, limit);
        q.pin_locked = 1;
        q.awaiting_sys_nl = 0;
    }
}

__device__ __forceinline__ int read_token(const ModelDev &m, const StateDev &s, int b) {
    const StepCtl &sc = *s.step;
    int tok = sc.ids ? sc.ids[(int64_t)b * sc.ids_ld + sc.ids_idx] : s.tok_in[b];
    if (tok < 0 || tok >= m.vocab) tok = m.pad_id;   // out-of-range ids become pad (runtime/vault3.c:2041)
    return tok;
}

// boundary steps: auto-pin must run before the eviction (it sets n_pin used by t_start and the sink rotation)
__global__ void k_pin(const ModelDev *mp, const StateDev *sp) {
    const StateDev &s = *sp;
    const int b = blockIdx.x;
    if (threadIdx.x == 0) auto_pin_update(*mp, s.seq[b], s.step->pos, read_token(*mp, s, b));
}

// token bookkeeping + segment ids + embedding (src/vault_v3_model.py:2257-2283)
template <bool PIN>
__global__ void k_begin(const ModelDev *mp, const StateDev *sp) {
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int b = blockIdx.x;
    __shared__ int s_tok;
    const int64_t pos = s.step->pos;
    const int W = m.W, c = (int)(pos % W), par = ring_par(pos, W);
    if (threadIdx.x == 0) {
        SeqCtl &q = s.seq[b];
        const int tok = read_token(m, s, b);
        if (PIN) auto_pin_update(m, q, pos, tok);
        if (c == 0) {
            q.cur_seg_id = 0;
            q.seg_len = 0;
        }
        s.tok_ring[((size_t)b * 2 + par) * W + c] = tok;
        if (seg_active(q)) {
            const int tr = m.tier[tok];
            const int t2 = max(m.seg_min, (m.seg_max * 2) / 3);
            const int t3 = max(m.seg_min, m.seg_max > 8 ? m.seg_max - 8 : m.seg_min);
            s.seg_ring[((size_t)b * 2 + par) * W + c] = q.cur_seg_id;
            q.seg_len += 1;
            const bool brk = (tr == 1 && q.seg_len >= m.seg_min) || (tr == 2 && q.seg_len >= t2) ||
                             (tr == 3 && q.seg_len >= t3);
            if (c == W - 1 || brk || q.seg_len >= m.seg_max) {
                q.cur_seg_id += 1;
                q.seg_len = 0;
            }
            // shingle resonance (src/vault_v3_model.py:1643-1716) needs a non-pinned <|im_end|> in the last
            // 38 tokens while the bank holds > 2 segments; it is not implemented on the device -> flag it
            if (pos >= 2 * W && q.mem_cnt > 0 && q.n_uniq_segs > 2) {
                const int hi = W + c;
                for (int p = hi; p >= max(0, hi - 37); --p) {
                    const int tk = p < W ? s.tok_ring[((size_t)b * 2 + (par ^ 1)) * W + p]
                                         : s.tok_ring[((size_t)b * 2 + par) * W + (p - W)];
                    if (tk == m.im_end_id) {
                        if (p > 0 && pos - (hi - p) >= q.n_pin) atomicOr(&s.step->status, STATUS_RESONANCE);
                        break;
                    }
                }
            }
        }
        s_tok = tok;
    }
    __syncthreads();
    const int tok = s_tok;
    float *x = s.x + (size_t)b * m.d;
    for (int k = threadIdx.x; k < m.d; k += blockDim.x) x[k] = tile_elem(m.embed, tok, k);
}

// ------------------------------------------------------------------------------------------ GEMV epilogues
struct EpiQKV {
    const ModelDev *m;
    const StateDev *s;
    int layer;
    const float *bq, *bk, *bv;
    __device__ void operator()(int seg, int rt, int t, int b, float y0, float y1) const {
        const int D = m->D, W = m->W, hd = D / 2;
        const int head = rt / (D / 8), j = rt % (D / 8), i = 4 * j + t;
        const int r0 = head * D + i, r1 = r0 + hd;
        const int64_t pos = s->step->pos;
        const int c = (int)(pos % W), par = ring_par(pos, W);
        const float *rc = rope_row(*m, c);
        const float cs = rc[i], sn = rc[hd + i];
        if (seg == 0) {
            const float a = y0 + bq[r0], bb = y1 + bq[r1];
            float *qc = s->q_cur + ((size_t)b * m->H + head) * D;
            qc[i] = a * cs - bb * sn;
            qc[i + hd] = bb * cs + a * sn;
            if (pos >= W) {
                const float *rf = rope_row(*m, W + c);
                float *qf = s->q_far + ((size_t)b * m->H + head) * D;
                qf[i] = a * rf[i] - bb * rf[hd + i];
                qf[i + hd] = bb * rf[i] + a * rf[hd + i];
            }
        } else if (seg == 1) {
            const float a = y0 + bk[r0], bb = y1 + bk[r1];
            __nv_bfloat16 *kr = kvp(*s, layer, b, ring_off(*s, par, KIND_KRAW, head, c));
            __nv_bfloat16 *ko = kvp(*s, layer, b, ring_off(*s, par, KIND_KROT, head, c));
            kr[i] = __float2bfloat16_rn(a);
            kr[i + hd] = __float2bfloat16_rn(bb);
            ko[i] = __float2bfloat16_rn(a * cs - bb * sn);
            ko[i + hd] = __float2bfloat16_rn(bb * cs + a * sn);
            if (pos < s->sink_cap) {
                __nv_bfloat16 *sk = kvp(*s, layer, b, sink_off(*s, SINK_KRAW, head, (int)pos));
                sk[i] = __float2bfloat16_rn(a);
                sk[i + hd] = __float2bfloat16_rn(bb);
            }
        } else {
            const float a = y0 + bv[r0], bb = y1 + bv[r1];
            __nv_bfloat16 *vv = kvp(*s, layer, b, ring_off(*s, par, KIND_V, head, c));
            vv[i] = __float2bfloat16_rn(a);
            vv[i + hd] = __float2bfloat16_rn(bb);
            if (pos < s->sink_cap) {
                __nv_bfloat16 *sv = kvp(*s, layer, b, sink_off(*s, SINK_V, head, (int)pos));
                sv[i] = __float2bfloat16_rn(a);
                sv[i + hd] = __float2bfloat16_rn(bb);
            }
        }
    }
};

struct EpiResid {   // x[b, row] += y
    float *x;
    int ld, rows;
    __device__ void operator()(int, int rt, int t, int b, float y0, float y1) const {
        const int r = 8 * rt + 2 * t;
        if (r < rows) x[(size_t)b * ld + r] += y0;
        if (r + 1 < rows) x[(size_t)b * ld + r + 1] += y1;
    }
};

struct EpiGateUp {  // h[b, f] = silu(gate_f) * up_f   (src/vault_v3_model.py:1149-1150)
    float *h;
    int F;
    __device__ void operator()(int, int rt, int t, int b, float g, float u) const {
        const int f = 4 * rt + t;
        if (f < F) h[(size_t)b * F + f] = g / (1.0f + expf(-g)) * u;
    }
};

struct EpiStoreMapped {   // y[b, source row] = value (undoes the RoPE-pair / gate-up row order of the tiles)
    float *y;
    int ld, rowmap, head_dim, src_rows;
    __device__ void operator()(int, int rt, int t, int b, float y0, float y1) const {
        int src, row;
        if (map_tile_row(rowmap, head_dim, src_rows, 8 * rt + 2 * t, src, row))
            y[(size_t)b * ld + src * src_rows + row] = y0;
        if (map_tile_row(rowmap, head_dim, src_rows, 8 * rt + 2 * t + 1, src, row))
            y[(size_t)b * ld + src * src_rows + row] = y1;
    }
};

struct EpiStore {   // y[b, row] = value
    float *y;
    int ld, rows;
    __device__ void operator()(int, int rt, int t, int b, float y0, float y1) const {
        const int r = 8 * rt + 2 * t;
        if (r < rows) y[(size_t)b * ld + r] = y0;
        if (r + 1 < rows) y[(size_t)b * ld + r + 1] = y1;
    }
};

// copy of the residual stream entering a scorer feature layer (src/vault_v3_model.py:2287-2288)
__global__ void k_copy_feat(const StateDev *sp, int d, int fi) {
    const StateDev &s = *sp;
    const int b = blockIdx.x;
    if (!seg_active(s.seq[b])) return;
    for (int k = threadIdx.x; k < d; k += blockDim.x) s.feat[(size_t)b * s.feat_dim + fi * d + k] = s.x[(size_t)b * d + k];
}

// ------------------------------------------------------------------------------------------ attention
// Split-KV decode attention for one layer.  grid = (max_splits, G, B); each CTA scores ATT_KEYS_PER_CTA keys of
// the concatenation [sink S | bank M | prev W | cur c+1] for the `grp` query heads sharing KV head g, writes an
// unnormalised partial (o, m, l), and the last CTA of (b, g) merges the partials in split order.
template <int D>
__global__ void __launch_bounds__(ATT_THREADS) k_attention(const ModelDev *mp, const StateDev *sp, int layer,
                                                           float scale) {
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int W = m.W, H = m.H, grp = H / m.G;
    const int64_t pos = s.step->pos;
    const int c = (int)(pos % W), par = ring_par(pos, W);
    const SeqCtl &q = s.seq[b];
    const int n_sk = pos >= 2 * W ? q.n_pin : 0;
    const int n_seg = (pos >= 2 * W && seg_active(q)) ? q.mem_cnt : 0;
    const int n_prev = pos >= W ? W : 0;
    const int n_cur = c + 1;
    const int total = n_sk + n_seg + n_prev + n_cur;
    const int n_splits = (total + ATT_KEYS_PER_CTA - 1) / ATT_KEYS_PER_CTA;
    if (split >= n_splits) return;
    const int j0 = split * ATT_KEYS_PER_CTA, j1 = min(total, j0 + ATT_KEYS_PER_CTA), nk = j1 - j0;

    __shared__ float s_qf[8][D], s_qc[8][D];
    __shared__ float s_p[8][ATT_KEYS_PER_CTA];
    __shared__ float s_m[8], s_l[8];
    __shared__ int s_last;
    const int tid = threadIdx.x;
    for (int idx = tid; idx < grp * D; idx += blockDim.x) {
        const int hr = idx / D, dd = idx % D;
        const size_t qo = ((size_t)b * H + g * grp + hr) * D + dd;
        s_qc[hr][dd] = s.q_cur[qo];
        s_qf[hr][dd] = pos >= W ? s.q_far[qo] : 0.f;
    }
    __syncthreads();
    // scores: one thread per key
    for (int jj = tid; jj < nk; jj += blockDim.x) {
        const int j = j0 + jj;
        const __nv_bfloat16 *kp;
        bool far = true;
        if (j < n_sk) kp = kvp(s, layer, b, sink_off(s, SINK_KROT, g, j));
        else if (j < n_sk + n_seg) kp = kvp(s, layer, b, bank_rot_off(s, g, j - n_sk));
        else if (j < n_sk + n_seg + n_prev) kp = kvp(s, layer, b, ring_off(s, par ^ 1, KIND_KROT, g, j - n_sk - n_seg));
        else {
            kp = kvp(s, layer, b, ring_off(s, par, KIND_KROT, g, j - n_sk - n_seg - n_prev));
            far = false;
        }
        float acc[8];
#pragma unroll
        for (int hr = 0; hr < 8; ++hr) acc[hr] = 0.f;
        const float(*qs)[D] = far ? s_qf : s_qc;
#pragma unroll 4
        for (int d0 = 0; d0 < D; d0 += 8) {
            const uint4 raw = *reinterpret_cast<const uint4 *>(kp + d0);
            const __nv_bfloat162 *k2 = reinterpret_cast<const __nv_bfloat162 *>(&raw);
            float kf[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __bfloat1622float2(k2[e]);
                kf[2 * e] = f.x;
                kf[2 * e + 1] = f.y;
            }
#pragma unroll
            for (int hr = 0; hr < 8; ++hr) {
                if (hr < grp) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[hr] = fmaf(qs[hr][d0 + e], kf[e], acc[hr]);
                }
            }
        }
        for (int hr = 0; hr < grp; ++hr) s_p[hr][jj] = acc[hr] * scale;
    }
    __syncthreads();
    // softmax pieces per head (warp w handles heads w, w+4)
    const int warp = tid >> 5, lane = tid & 31;
    for (int hr = warp; hr < grp; hr += blockDim.x / 32) {
        float mx = -INFINITY;
        for (int jj = lane; jj < nk; jj += 32) mx = fmaxf(mx, s_p[hr][jj]);
        mx = warp_max(mx);
        float l = 0.f;
        for (int jj = lane; jj < nk; jj += 32) {
            const float p = expf(s_p[hr][jj] - mx);
            s_p[hr][jj] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) {
            s_m[hr] = mx;
            s_l[hr] = l;
        }
    }
    __syncthreads();
    // o[hr][d] = sum_j p[hr][j] v[j][d]; thread layout: dims x key-phase
    float *part = s.att_part + ((((size_t)b * m.G + g) * s.max_splits + split) * grp) * (D + 2);
    for (int dd = tid; dd < D; dd += blockDim.x) {
        float o[8];
#pragma unroll
        for (int hr = 0; hr < 8; ++hr) o[hr] = 0.f;
        for (int jj = 0; jj < nk; ++jj) {
            const int j = j0 + jj;
            const __nv_bfloat16 *vp;
            if (j < n_sk) vp = kvp(s, layer, b, sink_off(s, SINK_V, g, j));
            else if (j < n_sk + n_seg) vp = kvp(s, layer, b, bank_off(s, q.bank_par, BANK_V, g, j - n_sk));
            else if (j < n_sk + n_seg + n_prev) vp = kvp(s, layer, b, ring_off(s, par ^ 1, KIND_V, g, j - n_sk - n_seg));
            else vp = kvp(s, layer, b, ring_off(s, par, KIND_V, g, j - n_sk - n_seg - n_prev));
            const float v = bf2f(vp[dd]);
#pragma unroll
            for (int hr = 0; hr < 8; ++hr)
                if (hr < grp) o[hr] = fmaf(s_p[hr][jj], v, o[hr]);
        }
        for (int hr = 0; hr < grp; ++hr) part[hr * (D + 2) + dd] = o[hr];
    }
    if (tid < grp) {
        part[tid * (D + 2) + D] = s_m[tid];
        part[tid * (D + 2) + D + 1] = s_l[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const uint32_t ticket = atomicAdd(&s.att_cnt[b * m.G + g], 1u);
        s_last = ticket == (uint32_t)(n_splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float *p0 = s.att_part + (((size_t)b * m.G + g) * s.max_splits) * grp * (D + 2);
    for (int idx = tid; idx < grp * D; idx += blockDim.x) {
        const int hr = idx / D, dd = idx % D;
        float M = -INFINITY;
        for (int sp2 = 0; sp2 < n_splits; ++sp2) M = fmaxf(M, p0[((size_t)sp2 * grp + hr) * (D + 2) + D]);
        float L = 0.f, O = 0.f;
        for (int sp2 = 0; sp2 < n_splits; ++sp2) {
            const float *pp = p0 + ((size_t)sp2 * grp + hr) * (D + 2);
            const float w = expf(pp[D] - M);
            L = fmaf(pp[D + 1], w, L);
            O = fmaf(pp[dd], w, O);
        }
        s.attn[((size_t)b * H + g * grp + hr) * D + dd] = O / L;
    }
    if (tid == 0) s.att_cnt[b * m.G + g] = 0u;
}

// ------------------------------------------------------------------------------------------ chunk boundary
// Segment-memory eviction for the chunk leaving the window (src/vault_v3_model.py:1865-1921,
// runtime/vault3.c:1833-1915): spoof expansion, per-segment max score with the 1e-6 * segment-id tiebreak,
// exact top-B by (score desc, position asc) over old bank + candidates, chronological compaction.  One CTA per
// sequence; the selection counts, for every entry, the entries that beat it (deterministic, no sort).
__global__ void __launch_bounds__(1024) k_bank_merge(const ModelDev *mp, const StateDev *sp) {
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int b = blockIdx.x;
    SeqCtl &q = s.seq[b];
    const int64_t pos = s.step->pos;
    const int W = m.W;
    if (!(pos >= 2 * W && seg_active(q))) return;
    extern __shared__ float sm[];
    float *sc = sm;                                   // [W]
    float *mx = sc + W;                               // [W]
    float *cand_sc = mx + W;                          // [seg_cap + W]
    int *cand_t = reinterpret_cast<int *>(cand_sc + s.seg_cap + W);   // [seg_cap + W]: old slot i or -(t+1)
    int *win = cand_t + s.seg_cap + W;                // [seg_cap + W]
    __shared__ int s_nloc, s_bad, s_ncand;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int64_t ev = pos / W - 2;
    const int p2 = (int)(ev & 1);                     // ring parity of the evicted chunk
    const float *scr = s.sc_ring + ((size_t)b * 2 + p2) * W;
    const int *sgr = s.seg_ring + ((size_t)b * 2 + p2) * W;
    const int *tkr = s.tok_ring + ((size_t)b * 2 + p2) * W;
    if (tid == 0) {
        s_nloc = 0;
        s_bad = 0;
    }
    __syncthreads();
    for (int t = tid; t < W; t += nt) {
        sc[t] = scr[t];
        mx[t] = 0.f;
        atomicMax(&s_nloc, sgr[t] + 1);
        if (sc[t] <= -1.0e29f) s_bad = 1;
    }
    __syncthreads();
    if (s_bad) {      // quarantine whole segments holding a spoofed token
        for (int t = tid; t < W; t += nt)
            if (sc[t] <= -1.0e29f) mx[sgr[t]] = 1.f;
        __syncthreads();
        for (int t = tid; t < W; t += nt)
            if (mx[sgr[t]] > 0.5f) sc[t] = -1.0e30f;
        __syncthreads();
    }
    const int n_loc = s_nloc;
    for (int sg = tid; sg < n_loc; sg += nt) mx[sg] = -INFINITY;
    __syncthreads();
    for (int t = tid; t < W; t += nt) {   // per-segment max (order-independent)
        const float v = sc[t];
        float *addr = &mx[sgr[t]];
        float old = *addr;
        while (v > old) {
            const float prev = __int_as_float(atomicCAS(reinterpret_cast<int *>(addr), __float_as_int(old), __float_as_int(v)));
            if (prev == old) break;
            old = prev;
        }
    }
    __syncthreads();
    const int t_start = ev == 0 ? q.n_pin : 0;
    const int base_off = q.seg_id_offset;
    const int M_old = q.mem_cnt, bp = q.bank_par;
    const size_t mo = ((size_t)b * 2 + bp) * s.seg_cap, mn = ((size_t)b * 2 + (bp ^ 1)) * s.seg_cap;
    __syncthreads();
    if (t_start >= W) {
        if (tid == 0) q.seg_id_offset = base_off + n_loc;
        return;
    }
    // candidate list: old bank entries, then valid tokens of the evicted chunk in position order
    for (int i = tid; i < M_old; i += nt) {
        cand_sc[i] = s.mem_score[mo + i];
        cand_t[i] = i;
    }
    if (tid == 0) {
        int n = M_old;
        for (int t = t_start; t < W; ++t) {
            const float v = mx[sgr[t]] - 1.0e-6f * (float)((sgr[t] + base_off) & 16383);
            if (!(v > -1.0e29f)) continue;
            cand_sc[n] = v;
            cand_t[n] = -(t + 1);
            ++n;
        }
        s_ncand = n;
    }
    __syncthreads();
    const int tot = s_ncand, budget = q.seg_budget;
    for (int i = tid; i < tot; i += nt) {
        int rank = 0;
        if (tot > budget) {
            const float si = cand_sc[i];
            for (int j2 = 0; j2 < tot; ++j2) {
                const float sj = cand_sc[j2];
                rank += (sj > si) || (sj == si && j2 < i);
            }
        }
        win[i] = rank < budget;
    }
    __syncthreads();
    if (tid == 0) {
        int n = 0;
        for (int i = 0; i < tot; ++i) {
            if (!win[i]) continue;
            const int src = cand_t[i];
            if (src >= 0) {
                s.mem_pos[mn + n] = s.mem_pos[mo + src];
                s.mem_tok[mn + n] = s.mem_tok[mo + src];
                s.mem_seg[mn + n] = s.mem_seg[mo + src];
            } else {
                const int t = -src - 1;
                s.mem_pos[mn + n] = ev * W + t;
                s.mem_tok[mn + n] = tkr[t];
                s.mem_seg[mn + n] = sgr[t] + base_off;
            }
            s.mem_score[mn + n] = cand_sc[i];
            s.mem_src[(size_t)b * s.seg_cap + n] = src;
            ++n;
        }
        int uniq = 0;
        for (int j = 0; j < n; ++j) uniq += (j == 0) || (s.mem_seg[mn + j] != s.mem_seg[mn + j - 1]);
        q.mem_cnt = n;
        q.n_uniq_segs = uniq;
        q.seg_id_offset = base_off + n_loc;
        q.bank_par = bp ^ 1;
    }
}

// gather the new bank rows (raw key and value) into the other bank buffer for every layer
__global__ void k_bank_gather(const ModelDev *mp, const StateDev *sp) {
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int layer = blockIdx.y, b = blockIdx.z;
    const SeqCtl &q = s.seq[b];
    const int64_t pos = s.step->pos;
    if (!(pos >= 2 * m.W && seg_active(q))) return;
    const int64_t ev = pos / m.W - 2;
    if ((ev == 0 ? q.n_pin : 0) >= m.W) return;       // no merge happened this boundary
    const int p2 = (int)(ev & 1), np_ = q.bank_par, op = np_ ^ 1;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int rows = q.mem_cnt * m.G * 2;
    const int D = m.D;
    for (int r = warp; r < rows; r += (gridDim.x * blockDim.x) >> 5) {
        const int kind = r & 1, g = (r >> 1) % m.G, j = (r >> 1) / m.G;
        const int src = s.mem_src[(size_t)b * s.seg_cap + j];
        const __nv_bfloat16 *from;
        if (src >= 0) from = kvp(s, layer, b, bank_off(s, op, kind == 0 ? BANK_KRAW : BANK_V, g, src));
        else from = kvp(s, layer, b, ring_off(s, p2, kind == 0 ? KIND_KRAW : KIND_V, g, -src - 1));
        __nv_bfloat16 *to = kvp(s, layer, b, bank_off(s, np_, kind == 0 ? BANK_KRAW : BANK_V, g, j));
        for (int d0 = lane * 8; d0 < D; d0 += 256)
            *reinterpret_cast<uint4 *>(to + d0) = *reinterpret_cast<const uint4 *>(from + d0);
    }
}

// bank keys -> positions -M..-1, sinks -> -(M+S)..-(M+1) (src/vault_v3_model.py:1842-1856)
__global__ void k_prefix_rot(const ModelDev *mp, const StateDev *sp) {
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int layer = blockIdx.y, b = blockIdx.z;
    const SeqCtl &q = s.seq[b];
    if (s.step->pos < 2 * m.W) return;
    const int M = seg_active(q) ? q.mem_cnt : 0, S = q.n_pin;
    const int D = m.D, hd = D / 2;
    const int n = (M + S) * m.G * hd;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += gridDim.x * blockDim.x) {
        const int i = idx % hd, r = idx / hd, g = r % m.G, j = r / m.G;
        const __nv_bfloat16 *src;
        __nv_bfloat16 *dst;
        int64_t p;
        if (j < M) {
            src = kvp(s, layer, b, bank_off(s, q.bank_par, BANK_KRAW, g, j));
            dst = kvp(s, layer, b, bank_rot_off(s, g, j));
            p = (int64_t)j - M;
        } else {
            const int jj = j - M;
            src = kvp(s, layer, b, sink_off(s, SINK_KRAW, g, jj));
            dst = kvp(s, layer, b, sink_off(s, SINK_KROT, g, jj));
            p = (int64_t)jj - (M + S);
        }
        const float *rr = rope_row(m, p);
        const float a = bf2f(src[i]), bb = bf2f(src[i + hd]);
        dst[i] = __float2bfloat16_rn(a * rr[i] - bb * rr[hd + i]);
        dst[i + hd] = __float2bfloat16_rn(bb * rr[i] + a * rr[hd + i]);
    }
}

// ------------------------------------------------------------------------------------------ segment scorer
// fc1 of SegmentScorer on LayerNorm(f) and LayerNorm(f - 0.65 ema) (src/vault_v3_model.py:879-883, :2294-2305)
__global__ void k_scorer_fc1(const ModelDev *mp, const StateDev *sp) {
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int b = blockIdx.y;
    if (!seg_active(s.seq[b])) return;
    const int fd = s.feat_dim, tid = threadIdx.x, nt = blockDim.x;
    const float *f = s.feat + (size_t)b * fd;
    const float *e = s.ema + (size_t)b * fd;
    __shared__ float red[4][32];
    __shared__ float st[4];
    float a0 = 0.f, a1 = 0.f;
    for (int k = tid; k < fd; k += nt) {
        a0 += f[k];
        a1 += f[k] - 0.65f * e[k];
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
            x0 += red[0][w];
            x1 += red[1][w];
        }
        st[0] = x0 / fd;
        st[1] = x1 / fd;
    }
    __syncthreads();
    const float mu0 = st[0], mu1 = st[1];
    float v0 = 0.f, v1 = 0.f;
    for (int k = tid; k < fd; k += nt) {
        const float d0 = f[k] - mu0, d1 = (f[k] - 0.65f * e[k]) - mu1;
        v0 = fmaf(d0, d0, v0);
        v1 = fmaf(d1, d1, v1);
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
            x0 += red[2][w];
            x1 += red[3][w];
        }
        st[2] = 1.0f / sqrtf(x0 / fd + 1e-5f);
        st[3] = 1.0f / sqrtf(x1 / fd + 1e-5f);
    }
    __syncthreads();
    const float i0 = st[2], i1 = st[3];
    const int warp = tid >> 5, lane = tid & 31;
    const int u = blockIdx.x * (nt / 32) + warp;
    if (u >= m.seg_hidden) return;
    const float *w1 = m.sc_w1 + (size_t)u * fd;
    float z0 = 0.f, z1 = 0.f;
    for (int k = lane; k < fd; k += 32) {
        const float lw = m.sc_ln_w[k], lb = m.sc_ln_b[k], wk = w1[k];
        const float h0 = (f[k] - mu0) * i0 * lw + lb;
        const float h1 = ((f[k] - 0.65f * e[k]) - mu1) * i1 * lw + lb;
        z0 = fmaf(wk, h0, z0);
        z1 = fmaf(wk, h1, z1);
    }
    z0 = warp_sum(z0);
    z1 = warp_sum(z1);
    if (lane == 0) {
        s.sc_z[((size_t)b * 2 + 0) * m.seg_hidden + u] = z0 + m.sc_b1[u];
        s.sc_z[((size_t)b * 2 + 1) * m.seg_hidden + u] = z1 + m.sc_b1[u];
    }
}

__device__ bool contains(const uint8_t *buf, int n, const char *lit, int ln) {
    for (int i = 0; i + ln <= n; ++i) {
        int k = 0;
        while (k < ln && buf[i + k] == (uint8_t)lit[k]) ++k;
        if (k == ln) return true;
    }
    return false;
}

// GELU + fc2, habituated score, EMA update, spoof quarantine (src/vault_v3_model.py:2294-2308, :1795-1817)
__global__ void k_scorer_out(const ModelDev *mp, const StateDev *sp) {
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int b = blockIdx.x;
    SeqCtl &q = s.seq[b];
    if (!seg_active(q)) return;
    const int tid = threadIdx.x, nt = blockDim.x, hd = m.seg_hidden, fd = s.feat_dim;
    __shared__ float red[2][32];
    __shared__ uint8_t buf[4096];
    const bool ready = q.ema_ready;   // read by every thread before thread 0 updates it below
    float r0 = 0.f, r1 = 0.f;
    for (int u = tid; u < hd; u += nt) {
        const float z0 = s.sc_z[((size_t)b * 2 + 0) * hd + u], z1 = s.sc_z[((size_t)b * 2 + 1) * hd + u];
        const float g0 = 0.5f * z0 * (1.0f + erff(z0 * 0.70710678118654752f));
        const float g1 = 0.5f * z1 * (1.0f + erff(z1 * 0.70710678118654752f));
        r0 = fmaf(m.sc_w2[u], g0, r0);
        r1 = fmaf(m.sc_w2[u], g1, r1);
    }
    r0 = warp_sum(r0);
    r1 = warp_sum(r1);
    if ((tid & 31) == 0) {
        red[0][tid >> 5] = r0;
        red[1][tid >> 5] = r1;
    }
    __syncthreads();
    float *e = s.ema + (size_t)b * fd;
    const float *f = s.feat + (size_t)b * fd;
    for (int k = tid; k < fd; k += nt) e[k] = ready ? 0.985f * e[k] + 0.015f * f[k] : f[k];
    if (tid == 0) {
        float raw = 0.f, hab = 0.f;
        for (int w = 0; w < nt / 32; ++w) {
            raw += red[0][w];
            hab += red[1][w];
        }
        raw += m.sc_b2[0];
        hab += m.sc_b2[0];
        float sc = raw;
        if (ready && hab > raw) sc = raw + 0.35f * (hab - raw);
        q.ema_ready = 1;
        const int64_t pos = s.step->pos;
        const int W = m.W, c = (int)(pos % W), par = ring_par(pos, W);
        // authority-spoof quarantine over the last <= 24 tokens
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
                    uint8_t ch = m.tok_pool[off + i];
                    buf[n++] = (ch >= 0x41 && ch <= 0x5A) ? (uint8_t)(ch + 32) : ch;
                }
            }
            if (contains(buf, n, "opi_signed_directive", 20) || contains(buf, n, "urgent opi delegation", 21))
                sc = -1.0e30f;
        }
        s.sc_ring[((size_t)b * 2 + par) * W + c] = sc;
    }
}

// ------------------------------------------------------------------------------------------ end of step
__global__ void k_argmax(const ModelDev *mp, const StateDev *sp, int32_t *next) {
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int b = blockIdx.x, tid = threadIdx.x;
    const float *lg = s.logits + (size_t)b * m.vocab;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < m.vocab; i += blockDim.x) {
        const float v = lg[i];
        if (v > best) {
            best = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    if ((tid & 31) == 0) {
        sv[tid >> 5] = best;
        si[tid >> 5] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < (int)blockDim.x / 32; ++w)
            if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
                best = sv[w];
                bi = si[w];
            }
        if (bi == 0x7fffffff) bi = 0;
        if (next) next[b] = bi;
        s.tok_in[b] = bi;
        const StepCtl &sc = *s.step;
        if (sc.out_tokens) sc.out_tokens[(int64_t)b * sc.out_ld + sc.out_idx] = bi;
    }
}

__global__ void k_advance(const StateDev *sp) {
    StepCtl &sc = *sp->step;
    sc.pos += 1;
    if (sc.ids) sc.ids_idx += 1;
    if (sc.out_tokens) sc.out_idx += 1;
}

__global__ void k_state_init(const ModelDev *mp, const StateDev *sp, int auto_pin, int seg_budget) {
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int b = threadIdx.x + blockIdx.x * blockDim.x;
    if (b == 0) {
        StepCtl &sc = *s.step;
        sc.pos = 0;
        sc.ids = nullptr;
        sc.ids_ld = 0;
        sc.ids_idx = 0;
        sc.out_tokens = nullptr;
        sc.out_ld = 0;
        sc.out_idx = 0;
        sc.status = 0;
        sc.want_logits = 1;
    }
    if (b >= s.B) return;
    SeqCtl &q = s.seq[b];
    q.n_pin = min(m.n_sink, m.W);
    q.pin_locked = auto_pin ? 0 : 1;
    q.saw_im_start = 0;
    q.awaiting_sys_nl = 0;
    q.ema_ready = 0;
    q.mem_cnt = 0;
    q.n_uniq_segs = 0;
    q.seg_id_offset = 0;
    q.cur_seg_id = 0;
    q.seg_len = 0;
    q.bank_par = 0;
    q.seg_budget = seg_budget;
    q.seg_on = (m.seg_n_feat > 0 && seg_budget > 0) ? 1 : 0;
    q.auto_pin = auto_pin;
    q.last_im_end = -1;
}

// ------------------------------------------------------------------------------------------ host launchers
template <class Epi>
static cudaError_t run_gemv(const v3g_model *m, GemvArgs a, const Epi &epi, int Btot, cudaStream_t st) {
    for (int b0 = 0; b0 < Btot; b0 += GEMV_MB) {
        a.b0 = b0;
        a.B = Btot - b0 < GEMV_MB ? Btot - b0 : GEMV_MB;
        int grid;
        size_t smem;
        gemv_plan(a, m->n_sm, grid, smem);
        if (smem > GEMV_MAX_SMEM) return cudaErrorInvalidValue;
        gemv_kernel<Epi><<<grid, GEMV_THREADS, smem, st>>>(a, epi);
    }
    return cudaGetLastError();
}

static GemvArgs gemv_args(const MatW *const *mats, int n, const float *x, int x_ld, int K, int prologue,
                          const float *norm_w, float eps) {
    GemvArgs a{};
    a.n_seg = n;
    for (int i = 0; i < n; ++i) {
        a.seg[i].tiles = mats[i]->tiles;
        a.seg[i].fmt = mats[i]->fmt;
        a.seg[i].n_rtiles = mats[i]->n_rtiles;
        a.seg[i].n_ktiles = mats[i]->n_ktiles;
    }
    a.K = K;
    a.x = x;
    a.x_ld = x_ld;
    a.prologue = prologue;
    a.norm_w = norm_w;
    a.eps = eps;
    a.xbf16 = x_is_bf16(mats[0]->fmt) ? 1 : 0;
    return a;
}

cudaError_t launch_gemv_store(const v3g_model *m, const MatW &w, const float *x, int B, float *y, cudaStream_t st) {
    const MatW *mats[1] = {&w};
    GemvArgs a = gemv_args(mats, 1, x, w.cols, w.cols, PRO_PLAIN, nullptr, 0.f);
    EpiStore epi{y, w.rows, w.rows};
    return run_gemv(m, a, epi, B, st);
}

cudaError_t launch_gemv_mapped(const v3g_model *m, const MatW &w, const float *x, int B, float *y, cudaStream_t st) {
    const MatW *mats[1] = {&w};
    GemvArgs a = gemv_args(mats, 1, x, w.cols, w.cols, PRO_PLAIN, nullptr, 0.f);
    const int src_rows = w.rowmap == ROWS_GATE_UP ? w.rows / 2 : w.rows;
    EpiStoreMapped epi{y, w.rows, w.rowmap, m->host.D, src_rows};
    return run_gemv(m, a, epi, B, st);
}

// one-time kernel attributes (large dynamic shared memory); must not run during stream capture
cudaError_t init_kernel_attrs() {
    cudaError_t e = cudaSuccess;
    auto set = [&](const void *f) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM);
    };
    set((const void *)gemv_kernel<EpiQKV>);
    set((const void *)gemv_kernel<EpiResid>);
    set((const void *)gemv_kernel<EpiGateUp>);
    set((const void *)gemv_kernel<EpiStore>);
    set((const void *)gemv_kernel<EpiStoreMapped>);
    set((const void *)k_bank_merge);
    return e;
}

template <int D>
static void launch_attention(const v3g_model *m, v3g_state *s, int layer, cudaStream_t st) {
    dim3 grid(s->host.max_splits, m->host.G, s->B);
    k_attention<D><<<grid, ATT_THREADS, 0, st>>>(m->dev, s->dev, layer, (float)(1.0 / sqrt((double)D)));
}

cudaError_t launch_prefix_refresh(const v3g_model *m, v3g_state *s, cudaStream_t st) {
    k_prefix_rot<<<dim3(64, m->host.n_layers, s->B), 256, 0, st>>>(m->dev, s->dev);
    return cudaGetLastError();
}

cudaError_t launch_state_reset(const v3g_model *m, v3g_state *s, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(s->arena, 0, s->arena_size, st);
    if (e != cudaSuccess) return e;
    k_state_init<<<(s->B + 127) / 128, 128, 0, st>>>(m->dev, s->dev, s->auto_pin, s->seg_budget);
    return cudaGetLastError();
}

cudaError_t launch_step(const v3g_model *m, v3g_state *s, bool boundary, bool want_lm, cudaStream_t st) {
    const ModelDev &md = m->host;
    const StateDev &sd = s->host;
    const int B = s->B;
    const bool any_seg = md.seg_n_feat > 0 && s->seg_budget > 0;
    cudaError_t e;
    if (boundary) {
        // the boundary kernels check pos >= 2W on the device, so one captured graph serves every rollover
        k_pin<<<B, 32, 0, st>>>(m->dev, s->dev);
        if (any_seg) {
            const size_t smem = (size_t)(2 * md.W + 3 * (sd.seg_cap + md.W)) * 4;
            if (smem > 227 * 1024) return cudaErrorInvalidValue;
            k_bank_merge<<<B, 1024, smem, st>>>(m->dev, s->dev);
            k_bank_gather<<<dim3(16, md.n_layers, B), 256, 0, st>>>(m->dev, s->dev);
        }
        k_prefix_rot<<<dim3(64, md.n_layers, B), 256, 0, st>>>(m->dev, s->dev);
        k_begin<false><<<B, 256, 0, st>>>(m->dev, s->dev);
    } else {
        k_begin<true><<<B, 256, 0, st>>>(m->dev, s->dev);
    }
    for (int l = 0; l < md.n_layers; ++l) {
        const LayerW &L = md.layers[l];
        for (int fi = 0; fi < md.seg_n_feat && any_seg; ++fi)
            if (md.seg_layers[fi] == l) k_copy_feat<<<B, 256, 0, st>>>(s->dev, md.d, fi);
        {
            const MatW *mats[3] = {&L.q, &L.k, &L.v};
            GemvArgs a = gemv_args(mats, 3, sd.x, md.d, md.d, PRO_RMSNORM, L.ln1, md.rms_eps);
            EpiQKV epi{m->dev, s->dev, l, L.bq, L.bk, L.bv};
            if ((e = run_gemv(m, a, epi, B, st)) != cudaSuccess) return e;
        }
        switch (md.D) {
            case 16: launch_attention<16>(m, s, l, st); break;
            case 32: launch_attention<32>(m, s, l, st); break;
            case 64: launch_attention<64>(m, s, l, st); break;
            case 128: launch_attention<128>(m, s, l, st); break;
            default: launch_attention<256>(m, s, l, st); break;
        }
        {
            const MatW *mats[1] = {&L.o};
            GemvArgs a = gemv_args(mats, 1, sd.attn, md.H * md.D, md.H * md.D, PRO_PLAIN, nullptr, 0.f);
            EpiResid epi{sd.x, md.d, md.d};
            if ((e = run_gemv(m, a, epi, B, st)) != cudaSuccess) return e;
        }
        {
            const MatW *mats[1] = {&L.gu};
            GemvArgs a = gemv_args(mats, 1, sd.x, md.d, md.d, PRO_RMSNORM, L.ln2, md.rms_eps);
            EpiGateUp epi{sd.hbuf, md.F};
            if ((e = run_gemv(m, a, epi, B, st)) != cudaSuccess) return e;
        }
        {
            const MatW *mats[1] = {&L.down};
            GemvArgs a = gemv_args(mats, 1, sd.hbuf, md.F, md.F, PRO_PLAIN, nullptr, 0.f);
            EpiResid epi{sd.x, md.d, md.d};
            if ((e = run_gemv(m, a, epi, B, st)) != cudaSuccess) return e;
        }
    }
    if (any_seg) {
        k_scorer_fc1<<<dim3((md.seg_hidden + 7) / 8, B), 256, 0, st>>>(m->dev, s->dev);
        k_scorer_out<<<B, 256, 0, st>>>(m->dev, s->dev);
    }
    if (want_lm) {
        const MatW *mats[1] = {&md.embed};
        GemvArgs a = gemv_args(mats, 1, sd.x, md.d, md.d, PRO_RMSNORM, md.norm, md.rms_eps);
        EpiStore epi{sd.logits, md.vocab, md.vocab};
        if ((e = run_gemv(m, a, epi, B, st)) != cudaSuccess) return e;
        k_argmax<<<B, 1024, 0, st>>>(m->dev, s->dev, nullptr);
    }
    k_advance<<<1, 1, 0, st>>>(s->dev);
    return cudaGetLastError();
}

}  // namespace v3g
