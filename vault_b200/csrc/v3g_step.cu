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
#include "v3g_scorer.cuh"

namespace v3g {

__device__ __forceinline__ int ring_par(int64_t pos, int W) { return (int)((pos / W) & 1); }

__device__ __forceinline__ bool seg_active(const SeqCtl &q) { return q.seg_on && q.seg_budget > 0; }

// element (row, k) of the tied embedding (identity row order)
__device__ __forceinline__ float tile_elem(const MatW &w, int row, int k) {
    return tile_value(w.tiles, w.fmt, w.n_ktiles, w.wscale, row, k);
}

__device__ __forceinline__ int read_token(const ModelDev &m, const StateDev &s, int b) {
    const StepCtl &sc = *s.step;
    int tok = sc.ids ? sc.ids[(int64_t)b * sc.ids_ld + sc.ids_idx] : s.tok_in[b];
    if (tok < 0 || tok >= m.vocab) tok = m.pad_id;   // out-of-range ids become pad (runtime/vault3.c:2041)
    return tok;
}

// boundary steps: auto-pin must run before the eviction (it sets n_pin used by t_start and the sink rotation)
__global__ void k_pin(const ModelDev *mp, const StateDev *sp) {
    griddep_wait();
    griddep_launch();
    const StateDev &s = *sp;
    const int b = blockIdx.x;
    if (threadIdx.x == 0) auto_pin_update(*mp, s.seq[b], s.step->pos, read_token(*mp, s, b));
}

// token bookkeeping + segment ids + embedding (src/vault_v3_model.py:2257-2283)
template <bool PIN>
__global__ void k_begin(const ModelDev *mp, const StateDev *sp) {
    griddep_wait();
    griddep_launch();
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
        s.amax[b] = 0ull;
        if (b == 0) *s.bar = 0u;   // grid-barrier counter of this step's persistent decode kernel
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
    // persistent kernel: the RoPE rows of positions c and W + c and the step position, held in shared memory
    // (nullptr: read them from the model / state in global memory)
    const float *rc_s = nullptr, *rf_s = nullptr;
    int64_t pos_s = 0;
    // persistent kernel: the biases of the CTA's row tiles [bias_r0, bias_r0 + bias_n) (flat over q, k, v; 16 per
    // row tile in tile-row order) in shared memory; rb1 / rb2 = flat index of the first k / v row tile
    const float *bias_s = nullptr;
    int bias_r0 = 0, bias_n = 0, rb1 = 0, rb2 = 0;
    // lane holds tile rows (g, g+8) = RoPE partners (i, i + D/2) of one head
    __device__ void operator()(int seg, int rt, int g, int b, float y0, float y1) const {
        const int D = s->D, W = s->W, hd = D / 2;
        const int head = rt / (D / TILE_ROWS), j = rt % (D / TILE_ROWS), i = 8 * j + g;
        const int r0 = head * D + i, r1 = r0 + hd;
        const int64_t pos = rc_s ? pos_s : s->step->pos;
        const int c = (int)(pos % W), par = ring_par(pos, W);
        const float *rc = rc_s ? rc_s : rope_row(*m, c);
        const float cs = rc[i], sn = rc[hd + i];
        const int rl = (seg == 0 ? 0 : (seg == 1 ? rb1 : rb2)) + rt - bias_r0;
        const bool pre = bias_s && rl >= 0 && rl < bias_n;
        const float *bsrc = seg == 0 ? bq : (seg == 1 ? bk : bv);
        const float b0v = pre ? bias_s[rl * 16 + g] : bsrc[r0], b1v = pre ? bias_s[rl * 16 + 8 + g] : bsrc[r1];
        if (seg == 0) {
            const float a = y0 + b0v, bb = y1 + b1v;
            float *qc = s->q_cur + ((size_t)b * s->H + head) * D;
            qc[i] = a * cs - bb * sn;
            qc[i + hd] = bb * cs + a * sn;
            if (pos >= W) {
                const float *rf = rc_s ? rf_s : rope_row(*m, W + c);
                float *qf = s->q_far + ((size_t)b * s->H + head) * D;
                qf[i] = a * rf[i] - bb * rf[hd + i];
                qf[i + hd] = bb * rf[i] + a * rf[hd + i];
            }
        } else if (seg == 1) {
            const float a = y0 + b0v, bb = y1 + b1v;
            kv_t *kr = kvp(*s, layer, b, ring_off(*s, par, KIND_KRAW, head, c));
            kv_t *ko = kvp(*s, layer, b, ring_off(*s, par, KIND_KROT, head, c));
            kr[i] = f2kv(a);
            kr[i + hd] = f2kv(bb);
            ko[i] = f2kv(a * cs - bb * sn);
            ko[i + hd] = f2kv(bb * cs + a * sn);
            if (pos < s->sink_cap) {
                kv_t *sk = kvp(*s, layer, b, sink_off(*s, SINK_KRAW, head, (int)pos));
                sk[i] = f2kv(a);
                sk[i + hd] = f2kv(bb);
            }
        } else {
            const float a = y0 + b0v, bb = y1 + b1v;
            kv_t *vv = kvp(*s, layer, b, ring_off(*s, par, KIND_V, head, c));
            vv[i] = f2kv(a);
            vv[i + hd] = f2kv(bb);
            if (pos < s->sink_cap) {
                kv_t *sv = kvp(*s, layer, b, sink_off(*s, SINK_V, head, (int)pos));
                sv[i] = f2kv(a);
                sv[i + hd] = f2kv(bb);
            }
        }
    }
};

struct EpiResid {   // x[b, row] += y   (identity row order: tile rows g, g+8)
    float *x;
    int ld, rows;
    __device__ void operator()(int, int rt, int g, int b, float y0, float y1) const {
        const int r = TILE_ROWS * rt + g;
        // L1-bypassing read: inside the persistent kernel other SMs updated x in earlier phases
        if (r < rows) x[(size_t)b * ld + r] = __ldcg(&x[(size_t)b * ld + r]) + y0;
        if (r + 8 < rows) x[(size_t)b * ld + r + 8] = __ldcg(&x[(size_t)b * ld + r + 8]) + y1;
    }
};

struct EpiGateUp {  // h[b, f] = silu(gate_f) * up_f   (src/vault_v3_model.py:1149-1150)
    float *h;
    int F;
    __device__ void operator()(int, int rt, int g, int b, float gt, float u) const {
        const int f = 8 * rt + g;
        if (f < F) h[(size_t)b * F + f] = gt / (1.0f + expf(-gt)) * u;
    }
};

struct EpiStoreMapped {   // y[b, source row] = value (undoes the RoPE-pair / gate-up row order of the tiles)
    float *y;
    int ld, rowmap, head_dim, src_rows;
    __device__ void operator()(int, int rt, int g, int b, float y0, float y1) const {
        int src, row;
        if (map_tile_row(rowmap, head_dim, src_rows, TILE_ROWS * rt + g, src, row))
            y[(size_t)b * ld + src * src_rows + row] = y0;
        if (map_tile_row(rowmap, head_dim, src_rows, TILE_ROWS * rt + g + 8, src, row))
            y[(size_t)b * ld + src * src_rows + row] = y1;
    }
};

struct EpiStore {   // y[b, row] = value
    float *y;
    int ld, rows;
    __device__ void operator()(int, int rt, int g, int b, float y0, float y1) const {
        const int r = TILE_ROWS * rt + g;
        if (r < rows) y[(size_t)b * ld + r] = y0;
        if (r + 8 < rows) y[(size_t)b * ld + r + 8] = y1;
    }
};

// ------------------------------------------------------------------------------------------ attention
// ------------------------------------------------------------------------------------------ chunk boundary
// Segment-memory eviction for the chunk leaving the window (src/vault_v3_model.py:1865-1921,
// runtime/vault3.c:1833-1915): spoof expansion, per-segment max score with the 1e-6 * segment-id tiebreak,
// exact top-B by (score desc, position asc) over old bank + candidates, chronological compaction.  One CTA per
// sequence; the selection counts, for every entry, the entries that beat it (deterministic, no sort).
__global__ void __launch_bounds__(1024) k_bank_merge(const ModelDev *mp, const StateDev *sp) {
    griddep_wait();
    griddep_launch();
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
    griddep_wait();
    griddep_launch();
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
        const kv_t *from;
        if (src >= 0) from = kvp(s, layer, b, bank_off(s, op, kind == 0 ? BANK_KRAW : BANK_V, g, src));
        else from = kvp(s, layer, b, ring_off(s, p2, kind == 0 ? KIND_KRAW : KIND_V, g, -src - 1));
        kv_t *to = kvp(s, layer, b, bank_off(s, np_, kind == 0 ? BANK_KRAW : BANK_V, g, j));
        for (int d0 = lane * 8; d0 < D; d0 += 256)
            *reinterpret_cast<uint4 *>(to + d0) = *reinterpret_cast<const uint4 *>(from + d0);
    }
}

// bank keys -> positions -M..-1, sinks -> -(M+S)..-(M+1) (src/vault_v3_model.py:1842-1856)
__global__ void k_prefix_rot(const ModelDev *mp, const StateDev *sp) {
    griddep_wait();
    griddep_launch();
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
        const kv_t *src;
        kv_t *dst;
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
        const float a = kv2f(src[i]), bb = kv2f(src[i + hd]);
        dst[i] = f2kv(a * rr[i] - bb * rr[hd + i]);
        dst[i + hd] = f2kv(bb * rr[i] + a * rr[hd + i]);
    }
}

// ------------------------------------------------------------------------------------------ segment scorer
// fc1 of SegmentScorer on LayerNorm(f) and LayerNorm(f - 0.65 ema) for the step's token (v3g_scorer.cuh)
__global__ void __launch_bounds__(SCORER_THREADS) k_scorer_fc1(const ModelDev *mp, const StateDev *sp) {
    griddep_wait();
    griddep_launch();
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int b = blockIdx.y;
    if (!seg_active(s.seq[b])) return;
    const int fd = s.feat_dim;
    const float *f = s.feat + (size_t)b * fd;
    const float *e = s.ema + (size_t)b * fd;
    scorer_fc1_block(m, fd, [=](int k) { return f[k]; },
                     [=](int k) { return sc_hab_in(f[k], e[k]); }, blockIdx.x * (SCORER_THREADS / 32),
                     s.sc_z + ((size_t)b * 2 + 0) * m.seg_hidden, s.sc_z + ((size_t)b * 2 + 1) * m.seg_hidden);
}

// GELU + fc2, habituated score, spoof quarantine, then the EMA update of the step's token
__global__ void __launch_bounds__(SCORER_THREADS) k_scorer_out(const ModelDev *mp, const StateDev *sp) {
    griddep_wait();
    griddep_launch();
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int b = blockIdx.x;
    SeqCtl &q = s.seq[b];
    if (!seg_active(q)) return;
    const int fd = s.feat_dim;
    const bool ready = q.ema_ready;   // read by every thread before thread 0 updates it below
    const int64_t pos = s.step->pos;
    const float sc = scorer_score_block(m, s, b, q, s.sc_z + ((size_t)b * 2 + 0) * m.seg_hidden,
                                        s.sc_z + ((size_t)b * 2 + 1) * m.seg_hidden, ready, pos);
    float *e = s.ema + (size_t)b * fd;
    const float *f = s.feat + (size_t)b * fd;
    for (int k = threadIdx.x; k < fd; k += blockDim.x) e[k] = ready ? sc_ema_next(e[k], f[k]) : f[k];
    if (threadIdx.x == 0) {
        q.ema_ready = 1;
        s.sc_ring[((size_t)b * 2 + ring_par(pos, m.W)) * m.W + (int)(pos % m.W)] = sc;
    }
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
// one GEMV launch description: kernel arguments plus the weight format of every segment
struct GemvCall {
    GemvArgs a;
    int fmts[3];
};

template <int FA, int FB, class Epi>
static cudaError_t launch_gemv_t(const v3g_model *m, GemvCall c, const Epi &epi, int Btot, cudaStream_t st, bool pdl) {
    for (int b0 = 0; b0 < Btot; b0 += GEMV_MB) {
        c.a.b0 = b0;
        c.a.B = Btot - b0 < GEMV_MB ? Btot - b0 : GEMV_MB;
        c.a.lo = c.a.lo == 0 ? 0 : -1;   // one part stays one part; otherwise re-planned for this pass
        int grid;
        size_t smem;
        gemv_plan(c.a, c.fmts, m->n_sm, grid, smem);
        if (smem > GEMV_MAX_SMEM) return cudaErrorInvalidValue;
        cudaError_t e = launch_k(pdl, gemv_kernel<FA, FB, Epi>, dim3(grid), dim3(GEMV_THREADS), smem, st, c.a, epi);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// Pick the kernel instantiation for the segments' formats: one format, or Q4_0 queries with Q8_0 keys/values
// (the hybrid file layout, tools/vlt3.py:312-330); any other mix runs one launch per segment.
template <class Epi>
static cudaError_t run_gemv(const v3g_model *m, const GemvCall &c, const Epi &epi, int Btot, cudaStream_t st,
                           bool pdl = false) {
    bool same = true, hybrid = c.fmts[0] == FMT_Q4;
    for (int i = 1; i < c.a.n_seg; ++i) {
        same = same && c.fmts[i] == c.fmts[0];
        hybrid = hybrid && c.fmts[i] == FMT_Q8;
    }
    if (same) {
        switch (c.fmts[0]) {
            case FMT_Q8: return launch_gemv_t<FMT_Q8, FMT_Q8>(m, c, epi, Btot, st, pdl);
            case FMT_Q4: return launch_gemv_t<FMT_Q4, FMT_Q4>(m, c, epi, Btot, st, pdl);
            case FMT_BF16: return launch_gemv_t<FMT_BF16, FMT_BF16>(m, c, epi, Btot, st, pdl);
            case FMT_F16: return launch_gemv_t<FMT_F16, FMT_F16>(m, c, epi, Btot, st, pdl);
            default: return launch_gemv_t<FMT_F32, FMT_F32>(m, c, epi, Btot, st, pdl);
        }
    }
    if (hybrid) return launch_gemv_t<FMT_Q4, FMT_Q8>(m, c, epi, Btot, st, pdl);
    for (int i = 0; i < c.a.n_seg; ++i) {
        GemvCall one = c;
        one.a.seg[0] = c.a.seg[i];
        one.a.n_seg = 1;
        one.a.seg_base = i;
        one.fmts[0] = c.fmts[i];
        cudaError_t e = run_gemv(m, one, epi, Btot, st, pdl);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

static GemvCall gemv_args(const MatW *const *mats, int n, const float *x, int x_ld, int K, int prologue,
                          const float *norm_w, float eps) {
    GemvCall c{};
    c.a.n_seg = n;
    for (int i = 0; i < n; ++i) {
        c.a.seg[i].tiles = mats[i]->tiles;
        c.a.seg[i].n_rtiles = mats[i]->n_rtiles;
        c.a.seg[i].n_ktiles = mats[i]->n_ktiles;
        c.a.seg[i].wscale = mats[i]->wscale;
        c.fmts[i] = mats[i]->fmt;
    }
    c.a.K = K;
    c.a.lo = -1;   // gemv_plan picks the activation split for the pass's batch
    c.a.x = x;
    c.a.x_ld = x_ld;
    c.a.prologue = prologue;
    c.a.norm_w = norm_w;
    c.a.eps = eps;
    return c;
}

cudaError_t launch_gemv_store(const v3g_model *m, const MatW &w, const float *x, int B, float *y, cudaStream_t st) {
    const MatW *mats[1] = {&w};
    GemvCall c = gemv_args(mats, 1, x, w.cols, w.cols, PRO_PLAIN, nullptr, 0.f);
    EpiStore epi{y, w.rows, w.rows};
    return run_gemv(m, c, epi, B, st);
}

cudaError_t launch_gemv_mapped(const v3g_model *m, const MatW &w, const float *x, int B, float *y, cudaStream_t st) {
    const MatW *mats[1] = {&w};
    GemvCall c = gemv_args(mats, 1, x, w.cols, w.cols, PRO_PLAIN, nullptr, 0.f);
    const int src_rows = w.rowmap == ROWS_GATE_UP ? w.rows / 2 : w.rows;
    EpiStoreMapped epi{y, w.rows, w.rowmap, m->host.D, src_rows};
    return run_gemv(m, c, epi, B, st);
}

// one-time kernel attributes (large dynamic shared memory); must not run during stream capture
template <class Epi>
static void set_gemv_attrs(cudaError_t &e, int optin) {
    auto set = [&](const void *f) {
        cudaFuncAttributes fa;
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, f);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
    };
    set((const void *)gemv_kernel<FMT_Q8, FMT_Q8, Epi>);
    set((const void *)gemv_kernel<FMT_Q4, FMT_Q4, Epi>);
    set((const void *)gemv_kernel<FMT_Q4, FMT_Q8, Epi>);
    set((const void *)gemv_kernel<FMT_BF16, FMT_BF16, Epi>);
    set((const void *)gemv_kernel<FMT_F16, FMT_F16, Epi>);
    set((const void *)gemv_kernel<FMT_F32, FMT_F32, Epi>);
}

cudaError_t init_kernel_attrs() {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    set_gemv_attrs<EpiQKV>(e, optin);
    set_gemv_attrs<EpiResid>(e, optin);
    set_gemv_attrs<EpiGateUp>(e, optin);
    set_gemv_attrs<EpiStore>(e, optin);
    set_gemv_attrs<EpiStoreMapped>(e, optin);
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, (const void *)k_bank_merge);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute((const void *)k_bank_merge, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 optin - (int)fa.sharedSizeBytes);
    return e;
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

}  // namespace v3g

#include "v3g_mega.cuh"

namespace v3g {

typedef void (*MkKernel)(const ModelDev *, const StateDev *, const MkPhase *, int, float, MkCfg);

template <int D>
static MkKernel mk_kernel_d(int fa, int fb) {
    if (fa == FMT_Q8 && fb == FMT_Q8) return k_decode<D, FMT_Q8, FMT_Q8>;
    if (fa == FMT_Q4 && fb == FMT_Q8) return k_decode<D, FMT_Q4, FMT_Q8>;
    if (fa == FMT_Q4 && fb == FMT_Q4) return k_decode<D, FMT_Q4, FMT_Q4>;
    if (fa == FMT_BF16 && fb == FMT_BF16) return k_decode<D, FMT_BF16, FMT_BF16>;
    if (fa == FMT_F16 && fb == FMT_F16) return k_decode<D, FMT_F16, FMT_F16>;
    if (fa == FMT_F32 && fb == FMT_F32) return k_decode<D, FMT_F32, FMT_F32>;
    return nullptr;
}

// persistent decode kernel instantiation for a head size and format pair (nullptr when none)
static MkKernel mk_kernel(int D, int fa, int fb) {
    switch (D) {
        case 16: return mk_kernel_d<16>(fa, fb);
        case 32: return mk_kernel_d<32>(fa, fb);
        case 64: return mk_kernel_d<64>(fa, fb);
        case 128: return mk_kernel_d<128>(fa, fb);
        default: return nullptr;
    }
}

// Phase table of the persistent decode kernel for this state; leaves use_mega = 0 when the batch does not fit one
// pass (> 8 rows), a phase would mix 16-bit activation types, or the shared-memory plan leaves no ring.
cudaError_t build_mega(const v3g_model *m, v3g_state *s) {
    const ModelDev &md = m->host;
    const StateDev &sd = s->host;
    s->use_mega = 0;
    if (s->B > GEMV_MB) return cudaSuccess;
    const bool any_seg = md.seg_n_feat > 0 && s->seg_cap > 0;
    std::vector<MkPhase> ph;
    size_t xr = 0;
    int max_rt = 0;
    bool ok = true;
    auto add_gemv = [&](const MatW *const *mats, int n, const float *x, int x_ld, int K, int prologue,
                        const float *norm_w, int epi, int layer, float *out, int out_ld, int out_rows) -> MkPhase & {
        GemvCall c = gemv_args(mats, n, x, x_ld, K, prologue, norm_w, md.rms_eps);
        c.a.B = s->B;
        c.a.b0 = 0;
        if (s->act_single) c.a.lo = 0;
        int grid;
        size_t smem;
        gemv_plan(c.a, c.fmts, m->n_sm, grid, smem);
        MkPhase p{};
        p.a = c.a;
        bool bs = false;
        int64_t tb = 0;
        int rb = 0;
        for (int i = 0; i < n; ++i) {
            p.fmts[i] = c.fmts[i];
            bs = bs || fmt_int(c.fmts[i]);
            p.tbase[i] = (int)tb;
            p.rbase[i] = rb;
            tb += (int64_t)c.a.seg[i].n_rtiles * c.a.seg[i].n_ktiles;
            rb += c.a.seg[i].n_rtiles;
        }
        ok = ok && tb < (int64_t)1 << 30;
        p.tbase[n] = (int)tb;
        max_rt = rb > max_rt ? rb : max_rt;
        const size_t need = (size_t)(144 + (bs ? c.a.nblk * GEMV_MB : 0)) * 4 + (size_t)gemv_xrows(s->B, c.a.lo) * c.a.nblk * 64;
        xr = need > xr ? need : xr;
        p.kind = MK_GEMV;
        p.epi = epi;
        p.layer = layer;
        p.out = out;
        p.out_ld = out_ld;
        p.out_rows = out_rows;
        ph.push_back(p);
        return ph.back();
    };
    for (int l = 0; l < md.n_layers; ++l) {
        const LayerW &L = md.layers[l];
        const MatW *qkv[3] = {&L.q, &L.k, &L.v};
        MkPhase &q = add_gemv(qkv, 3, sd.x, md.d, md.d, PRO_RMSNORM, L.ln1, MK_EPI_QKV, l, nullptr, 0, 0);
        q.bq = L.bq;
        q.bk = L.bk;
        q.bv = L.bv;
        for (int fi = 0; fi < md.seg_n_feat && any_seg; ++fi)
            if (md.seg_layers[fi] == l) {   // scorer features: residual stream entering this layer
                q.a.feat = sd.feat + (size_t)fi * md.d;
                q.a.feat_ld = sd.feat_dim;
            }
        MkPhase at{};
        at.kind = MK_ATTN;
        at.layer = l;
        ph.push_back(at);
        const MatW *o[1] = {&L.o};
        add_gemv(o, 1, sd.attn, md.H * md.D, md.H * md.D, PRO_PLAIN, nullptr, MK_EPI_RESID, l, sd.x, md.d, md.d)
            .attn_in = 1;
        const MatW *gu[1] = {&L.gu};
        add_gemv(gu, 1, sd.x, md.d, md.d, PRO_RMSNORM, L.ln2, MK_EPI_GATEUP, l, sd.hbuf, md.F, md.F);
        const MatW *dn[1] = {&L.down};
        add_gemv(dn, 1, sd.hbuf, md.F, md.F, PRO_PLAIN, nullptr, MK_EPI_RESID, l, sd.x, md.d, md.d);
    }
    const MatW *lm[1] = {&md.embed};
    add_gemv(lm, 1, sd.x, md.d, md.d, PRO_RMSNORM, md.norm, MK_EPI_STORE, -1, sd.logits, md.vocab, md.vocab);
    if (!ok) return cudaSuccess;
    // a phase followed by an RMSNorm phase stages that phase's norm weights in shared memory (16-byte pieces)
    for (size_t i = 0; i + 1 < ph.size(); ++i) {
        const MkPhase &nx = ph[i + 1];
        if (ph[i].kind == MK_GEMV && nx.kind == MK_GEMV && nx.a.prologue == PRO_RMSNORM && nx.a.K == md.d &&
            md.d % 4 == 0 && reinterpret_cast<uintptr_t>(nx.a.norm_w) % 16 == 0) {
            ph[i].next_norm = nx.a.norm_w;
            ph[i].next_k = nx.a.K;
            ph[i + 1].norm_staged = 1;
        }
    }
    // the kernel's format pair: every segment of every GEMV phase must be FA or FB
    bool has[16] = {};
    for (const MkPhase &q : ph)
        if (q.kind == MK_GEMV)
            for (int i = 0; i < q.a.n_seg; ++i) has[q.fmts[i]] = true;
    int nf = 0;
    for (bool h : has) nf += h ? 1 : 0;
    int fa, fb;
    if (nf == 1) {
        fa = fb = has[FMT_Q8] ? FMT_Q8 : has[FMT_Q4] ? FMT_Q4 : has[FMT_BF16] ? FMT_BF16 : has[FMT_F16] ? FMT_F16 : FMT_F32;
    } else if (nf == 2 && has[FMT_Q4] && has[FMT_Q8]) {
        fa = FMT_Q4;
        fb = FMT_Q8;
    } else {
        return cudaSuccess;
    }
    const MkKernel fn = mk_kernel(md.D, fa, fb);
    if (!fn) return cudaSuccess;
    size_t att = 0;
    switch (md.D) {
        case 16: att = sizeof(AttnSmem<16>); break;
        case 32: att = sizeof(AttnSmem<32>); break;
        case 64: att = sizeof(AttnSmem<64>); break;
        default: att = sizeof(AttnSmem<128>); break;
    }
    xr = (std::max(xr, att) + 127) / 128 * 128;
    int optin = 0;
    cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fattr{};
    e = cudaFuncGetAttributes(&fattr, (const void *)fn);
    if (e != cudaSuccess) return e;
    // shared memory: [x / attention region][2 phase descriptors][lite table][split pieces][per-step constants]
    // [staged norm weights][rings][ring mbarriers]
    const size_t ph_off = xr, lite_off = ph_off + 2 * sizeof(MkPhase);
    const size_t part_off = (lite_off + ph.size() * sizeof(MkLite) + 15) / 16 * 16;
    const size_t misc_off = (part_off + sizeof(MkPart) + 15) / 16 * 16;
    const size_t nw_off = (misc_off + sizeof(MkMisc) + 15) / 16 * 16;
    const size_t ring_off = (nw_off + (size_t)md.d * sizeof(float) + 127) / 128 * 128;
    const long avail = (long)optin - (long)fattr.sharedSizeBytes - (long)ring_off;
    const long per_slot = (long)MK_WARPS * (MK_SLOT_BYTES + 16);   // buffer + full and empty barriers
    int slots = avail > 0 ? (int)(avail / per_slot) : 0;
    slots = slots > MK_MAX_SLOTS ? MK_MAX_SLOTS : slots;
    if (slots < 2) return cudaSuccess;
    const size_t bar_off = ring_off + (size_t)MK_WARPS * slots * MK_SLOT_BYTES;
    const size_t smem = bar_off + (size_t)2 * MK_WARPS * slots * 8;
    e = cudaFuncSetAttribute((const void *)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, (const void *)fn, MK_THREADS, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaSuccess;
    std::vector<MkLite> lite(ph.size());
    for (size_t i = 0; i < ph.size(); ++i) {
        MkLite L{};
        L.kind = (int8_t)ph[i].kind;
        L.n_seg = (int8_t)(ph[i].kind == MK_GEMV ? ph[i].a.n_seg : 0);
        for (int j = 0; j < L.n_seg; ++j) {
            L.tiles[j] = ph[i].a.seg[j].tiles;
            L.kt[j] = ph[i].a.seg[j].n_ktiles;
            L.fmt[j] = (int8_t)ph[i].fmts[j];
        }
        for (int j = 0; j <= L.n_seg; ++j) {
            L.tbase[j] = ph[i].tbase[j];
            L.rbase[j] = j < L.n_seg ? ph[i].rbase[j] : (j ? ph[i].rbase[j - 1] + ph[i].a.seg[j - 1].n_rtiles : 0);
        }
        lite[i] = L;
    }
    e = cudaMalloc(&s->mk_phases, ph.size() * sizeof(MkPhase));
    if (e != cudaSuccess) return e;
    e = cudaMemcpy(s->mk_phases, ph.data(), ph.size() * sizeof(MkPhase), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return e;
    e = cudaMalloc(&s->mk_lite, lite.size() * sizeof(MkLite));
    if (e != cudaSuccess) return e;
    e = cudaMemcpy(s->mk_lite, lite.data(), lite.size() * sizeof(MkLite), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return e;
    s->mk_n = (int)ph.size();
    s->mk_smem = smem;
    s->mk_slots = slots;
    s->mk_xr = (int)xr;
    s->mk_ph_off = (int)ph_off;
    s->mk_lite_off = (int)lite_off;
    s->mk_part_off = (int)part_off;
    s->mk_misc_off = (int)misc_off;
    s->mk_nw_off = (int)nw_off;
    s->mk_ring_off = (int)ring_off;
    s->mk_bar_off = (int)bar_off;
    s->mk_grid = m->n_sm;
    s->mk_fn = (void *)fn;
    s->use_mega = 1;
    return cudaSuccess;
}

// cooperative launch (every CTA co-resident, which the grid barriers need); without the lm head the last phase is
// dropped
cudaError_t launch_mega(const v3g_model *m, v3g_state *s, bool want_lm, cudaStream_t st) {
    const int n = want_lm ? s->mk_n : s->mk_n - 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(s->mk_grid);
    cfg.blockDim = dim3(MK_THREADS);
    cfg.dynamicSmemBytes = s->mk_smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const ModelDev *mdv = m->dev;
    const StateDev *sdv = s->dev;
    const MkPhase *phases = static_cast<const MkPhase *>(s->mk_phases);
    const float scale = (float)(1.0 / sqrt((double)m->host.D));
    MkCfg mc;
    mc.slots = s->mk_slots;
    mc.xr_bytes = s->mk_xr;
    mc.ph_off = s->mk_ph_off;
    mc.lite_off = s->mk_lite_off;
    mc.part_off = s->mk_part_off;
    mc.misc_off = s->mk_misc_off;
    mc.nw_off = s->mk_nw_off;
    mc.x_rtiles = (m->host.d + TILE_ROWS - 1) / TILE_ROWS;
    mc.x_ld = m->host.d;
    mc.ring_off = s->mk_ring_off;
    mc.bar_off = s->mk_bar_off;
    mc.lite = static_cast<const MkLite *>(s->mk_lite);
    return cudaLaunchKernelEx(&cfg, reinterpret_cast<MkKernel>(s->mk_fn), mdv, sdv, phases, n, scale, mc);
}

// The boundary kernels check pos >= 2W on the device, so one captured graph serves every rollover.
cudaError_t launch_boundary(const v3g_model *m, v3g_state *s, cudaStream_t st) {
    const ModelDev &md = m->host;
    const StateDev &sd = s->host;
    const ModelDev *mdv = m->dev;
    const StateDev *sdv = s->dev;
    const int B = s->B;
    const bool any_seg = md.seg_n_feat > 0 && s->seg_budget > 0;
    const bool pdl = s->use_pdl != 0;
    cudaError_t e = launch_k(false, k_pin, dim3(B), dim3(32), 0, st, mdv, sdv);
    if (e != cudaSuccess) return e;
    if (any_seg) {
        const size_t smem = (size_t)(2 * md.W + 3 * (sd.seg_cap + md.W)) * 4;
        if (smem > (size_t)GEMV_MAX_SMEM) return cudaErrorInvalidValue;
        if ((e = launch_k(pdl, k_bank_merge, dim3(B), dim3(1024), smem, st, mdv, sdv)) != cudaSuccess) return e;
        if ((e = launch_k(pdl, k_bank_gather, dim3(16, md.n_layers, B), dim3(256), 0, st, mdv, sdv)) != cudaSuccess)
            return e;
    }
    return launch_k(pdl, k_prefix_rot, dim3(64, md.n_layers, B), dim3(256), 0, st, mdv, sdv);
}

cudaError_t launch_lm_head(const v3g_model *m, v3g_state *s, const float *x, int x_ld, cudaStream_t st) {
    const ModelDev &md = m->host;
    const MatW *mats[1] = {&md.embed};
    GemvCall a = gemv_args(mats, 1, x, x_ld, md.d, PRO_RMSNORM, md.norm, md.rms_eps);
    EpiStore epi{s->host.logits, md.vocab, md.vocab};
    return run_gemv(m, a, epi, s->B, st, false);
}

// token bookkeeping, segment ids and embedding of a step (after the chunk-boundary kernels at a window boundary)
cudaError_t launch_step_begin(const v3g_model *m, v3g_state *s, bool boundary, cudaStream_t st) {
    const ModelDev *mdv = m->dev;
    const StateDev *sdv = s->dev;
    if (boundary) {
        cudaError_t e = launch_boundary(m, s, st);
        if (e != cudaSuccess) return e;
        return launch_k(s->use_pdl != 0, k_begin<false>, dim3(s->B), dim3(256), 0, st, mdv, sdv);
    }
    return launch_k(false, k_begin<true>, dim3(s->B), dim3(256), 0, st, mdv, sdv);
}

// SegmentScorer v2 + habituation + spoof check of the step's token, per sequence
cudaError_t launch_scorer(const v3g_model *m, v3g_state *s, cudaStream_t st) {
    const ModelDev &md = m->host;
    const bool pdl = s->use_pdl != 0;
    cudaError_t e = launch_k(pdl, k_scorer_fc1, dim3((md.seg_hidden + 7) / 8, s->B), dim3(SCORER_THREADS), 0, st,
                             (const ModelDev *)m->dev, (const StateDev *)s->dev);
    if (e != cudaSuccess) return e;
    return launch_k(pdl, k_scorer_out, dim3(s->B), dim3(SCORER_THREADS), 0, st, (const ModelDev *)m->dev,
                    (const StateDev *)s->dev);
}

// Kernel sequence of one decode step.  Every launch after the first carries programmatic stream serialization:
// the next kernel's CTAs start streaming their weights while the previous kernel drains (griddep_wait in each
// kernel orders all state accesses).
cudaError_t launch_step(const v3g_model *m, v3g_state *s, bool boundary, bool want_lm, cudaStream_t st) {
    const ModelDev &md = m->host;
    const StateDev &sd = s->host;
    const ModelDev *mdv = m->dev;
    const StateDev *sdv = s->dev;
    const int B = s->B;
    const bool any_seg = md.seg_n_feat > 0 && s->seg_budget > 0;
    const bool pdl = s->use_pdl != 0;
    cudaError_t e;
#define V3G_TRY(x)                          \
    do {                                    \
        if ((e = (x)) != cudaSuccess) return e; \
    } while (0)
    if (!s->use_mega && s->use_tc_step) return launch_step_tc(m, s, boundary, want_lm, st);
    V3G_TRY(launch_step_begin(m, s, boundary, st));
    if (s->use_mega) {   // all layers + lm head in one persistent launch
        V3G_TRY(launch_mega(m, s, want_lm, st));
        if (any_seg) V3G_TRY(launch_scorer(m, s, st));
        V3G_TRY(launch_argmax_finish(m, s, want_lm, pdl, st));
        return cudaSuccess;
    }
    for (int l = 0; l < md.n_layers; ++l) {
        const LayerW &L = md.layers[l];
        {
            const MatW *mats[3] = {&L.q, &L.k, &L.v};
            GemvCall a = gemv_args(mats, 3, sd.x, md.d, md.d, PRO_RMSNORM, L.ln1, md.rms_eps);
            for (int fi = 0; fi < md.seg_n_feat && any_seg; ++fi)
                if (md.seg_layers[fi] == l) {   // scorer features: residual stream entering this layer
                    a.a.feat = sd.feat + (size_t)fi * md.d;
                    a.a.feat_ld = sd.feat_dim;
                }
            EpiQKV epi{mdv, sdv, l, L.bq, L.bk, L.bv};
            if (s->act_single) a.a.lo = 0;
            V3G_TRY(run_gemv(m, a, epi, B, st, pdl));
        }
        V3G_TRY(launch_attention(m, s, l, pdl, st));
        {
            const MatW *mats[1] = {&L.o};
            GemvCall a = gemv_args(mats, 1, sd.attn, md.H * md.D, md.H * md.D, PRO_PLAIN, nullptr, 0.f);
            EpiResid epi{sd.x, md.d, md.d};
            if (s->act_single) a.a.lo = 0;
            V3G_TRY(run_gemv(m, a, epi, B, st, pdl));
        }
        {
            const MatW *mats[1] = {&L.gu};
            GemvCall a = gemv_args(mats, 1, sd.x, md.d, md.d, PRO_RMSNORM, L.ln2, md.rms_eps);
            EpiGateUp epi{sd.hbuf, md.F};
            if (s->act_single) a.a.lo = 0;
            V3G_TRY(run_gemv(m, a, epi, B, st, pdl));
        }
        {
            const MatW *mats[1] = {&L.down};
            GemvCall a = gemv_args(mats, 1, sd.hbuf, md.F, md.F, PRO_PLAIN, nullptr, 0.f);
            EpiResid epi{sd.x, md.d, md.d};
            if (s->act_single) a.a.lo = 0;
            V3G_TRY(run_gemv(m, a, epi, B, st, pdl));
        }
    }
    if (any_seg) V3G_TRY(launch_scorer(m, s, st));
    if (want_lm) {
        const MatW *mats[1] = {&md.embed};
        GemvCall a = gemv_args(mats, 1, sd.x, md.d, md.d, PRO_RMSNORM, md.norm, md.rms_eps);
        EpiStore epi{sd.logits, md.vocab, md.vocab};
        if (s->act_single) a.a.lo = 0;
        V3G_TRY(run_gemv(m, a, epi, B, st, pdl));
    }
    V3G_TRY(launch_argmax_finish(m, s, want_lm, pdl, st));
#undef V3G_TRY
    return cudaSuccess;
}

}  // namespace v3g

#ifdef V3G_MK_TRACE
#include "../../include/vault_b200.h"
// timeline of the last persistent-kernel launch ([phase][cta][event] u64 nanoseconds; see v3g.cuh)
extern "C" V3G_API int v3g_mk_trace_read(void *dst, size_t bytes) {
    return (int)cudaMemcpyFromSymbol(dst, v3g::g_mk_trace, bytes < sizeof(v3g::g_mk_trace) ? bytes : sizeof(v3g::g_mk_trace));
}
#endif
