// Chunked prefill: a piece of up to one window chunk of prompt tokens per sequence goes through every layer as
// tensor-core GEMMs (v3g_gemm.cuh) and one block-window attention kernel, instead of one decode step per token.
//
// Reference semantics: VAULTv3ForCausalLM._forward_chunk_recurrent (src/vault_v3_model.py:1938-2116) for batch 1
// and the batched sliding-window path (block_sliding_attention, :812-863, through prefill :2163-2212) for batch > 1:
// a token at chunk position c attends to [pinned sinks | segment bank | previous chunk] (all tokens of the chunk
// see the same prefix) and causally to the current chunk's positions 0..c.  A piece never crosses a window
// boundary, so the chunk-boundary work (auto-pin of the boundary token, segment eviction and merge, prefix
// re-rotation) runs before it exactly as in a decode step, and every token of a piece shares one key prefix.
// Keys are stored rotated at their chunk position and queries rotated twice (at c and at W + c) -- the relative
// positions of the reference's re-based RoPE (see v3g_step.cu).
#include <math.h>

#include <string>

#include "../../include/vault_b200.h"
#include "v3g_attn.cuh"
#include "v3g_gemm.cuh"
#include "v3g_internal.h"
#include "v3g_scorer.cuh"

namespace v3g {

// ------------------------------------------------------------------------------------------ per-piece control
// Token bookkeeping of a piece (the sequential part of src/vault_v3_model.py:2224-2268 / :1952-2022 for every
// token) and the embedding rows of all its tokens.  Grid (sequence, token slice): every CTA gathers the embedding
// rows of its slice; CTA 0 of a sequence also runs the bookkeeping, with the piece's token ids and tiers staged in
// shared memory and the sequence's control block held in registers (one thread: the segmentation is a recurrence
// over the tokens), then writes the token and segment rings in parallel.  pin_first = 0 when a boundary piece's
// first token was already auto-pinned before the eviction (k_pin).  A piece never crosses a window boundary.
__global__ void __launch_bounds__(256) k_piece_begin(const ModelDev *mp, const StateDev *sp, const int32_t *ids,
                                                     int64_t ld, int64_t i0, int n, int64_t p0, int pin_first,
                                                     float *X) {
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int b = blockIdx.x;
    const int W = m.W, d = m.d;
    const int c0 = (int)(p0 % W), par = (int)((p0 / W) & 1);
    extern __shared__ int s_tok[];   // [n] token ids, [n] tiers, [n] segment ids
    int *s_tier = s_tok + n, *s_seg = s_tok + 2 * n;
    const int j0 = (int)((int64_t)n * blockIdx.y / gridDim.y), j1 = (int)((int64_t)n * (blockIdx.y + 1) / gridDim.y);
    const bool ctl = blockIdx.y == 0;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        if (!ctl && (j < j0 || j >= j1)) continue;
        int tok = ids[(int64_t)b * ld + i0 + j];
        if (tok < 0 || tok >= m.vocab) tok = m.pad_id;   // runtime/vault3.c:2041
        s_tok[j] = tok;
        if (ctl) s_tier[j] = m.tier[tok];
    }
    __syncthreads();
    for (int64_t i = threadIdx.x; i < (int64_t)(j1 - j0) * d; i += blockDim.x) {
        const int j = j0 + (int)(i / d), k = (int)(i % d);
        X[((int64_t)b * n + j) * d + k] = tile_value(m.embed.tiles, m.embed.fmt, m.embed.n_ktiles, m.embed.wscale,
                                                     s_tok[j], k);
    }
    if (!ctl) return;
    int32_t *tok_ring = s.tok_ring + ((size_t)b * 2 + par) * W;
    const int32_t *tok_prev = s.tok_ring + ((size_t)b * 2 + (par ^ 1)) * W;
    if (threadIdx.x == 0) {
        SeqCtl q = s.seq[b];
        const bool seg = q.seg_on && q.seg_budget > 0;
        const bool res = p0 >= 2 * W && q.mem_cnt > 0 && q.n_uniq_segs > 2;   // resonance trigger (see k_begin)
        const int t2 = max(m.seg_min, (m.seg_max * 2) / 3);
        const int t3 = max(m.seg_min, m.seg_max > 8 ? m.seg_max - 8 : m.seg_min);
        bool flagged = false;
        for (int j = 0; j < n; ++j) {
            const int64_t pos = p0 + j;
            const int c = c0 + j, tok = s_tok[j];
            if (j > 0 || pin_first) auto_pin_update(m, q, pos, tok);
            if (c == 0) {
                q.cur_seg_id = 0;
                q.seg_len = 0;
            }
            if (seg) {
                const int tr = s_tier[j];
                s_seg[j] = q.cur_seg_id;
                q.seg_len += 1;
                const bool brk = (tr == 1 && q.seg_len >= m.seg_min) || (tr == 2 && q.seg_len >= t2) ||
                                 (tr == 3 && q.seg_len >= t3);
                if (c == W - 1 || brk || q.seg_len >= m.seg_max) {
                    q.cur_seg_id += 1;
                    q.seg_len = 0;
                }
                if (res && !flagged) {   // the latest <|im_end|> within 37 tokens, in the window up to this token
                    const int hi = W + c;
                    for (int p = hi; p >= max(0, hi - 37); --p) {
                        const int cp = p - W;   // slot in the current chunk (< 0: the previous chunk)
                        const int tk = cp < 0 ? tok_prev[p] : (cp >= c0 ? s_tok[cp - c0] : tok_ring[cp]);
                        if (tk == m.im_end_id) {
                            if (p > 0 && pos - (hi - p) >= q.n_pin) flagged = true;
                            break;
                        }
                    }
                }
            }
        }
        if (flagged) atomicOr(&s.step->status, STATUS_RESONANCE);
        s.seq[b] = q;
        s.amax[b] = 0ull;
    }
    __syncthreads();
    const bool seg = s.seq[b].seg_on && s.seq[b].seg_budget > 0;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        tok_ring[c0 + j] = s_tok[j];
        if (seg) s.seg_ring[((size_t)b * 2 + par) * W + c0 + j] = s_seg[j];
    }
}

// end of a piece: position, prefill id cursor, the scorer's EMA flag and (with the lm head) each sequence's greedy
// next token
__global__ void k_piece_finish(const StateDev *sp, int n, int want_lm) {
    const StateDev &s = *sp;
    StepCtl &sc = *s.step;
    for (int b = threadIdx.x; b < s.B; b += blockDim.x) {
        if (want_lm) {
            const unsigned long long key = __ldcg(&s.amax[b]);
            s.tok_in[b] = key ? (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu)) : 0;
        }
        SeqCtl &q = s.seq[b];
        if (q.seg_on && q.seg_budget > 0 && n > 0) q.ema_ready = 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        sc.pos += n;
        if (sc.ids) sc.ids_idx += n;
    }
}

// ------------------------------------------------------------------------------------------ segment scorer
// Habituation inputs of a piece, hin[t] = f[t] - 0.65 ema(before t), and the EMA carried to the piece's end:
// sequential over the piece's tokens, parallel over features (the step's EMA update, token after token).
__global__ void k_piece_scan(const StateDev *sp, int n, const float *feat, float *hin) {
    const StateDev &s = *sp;
    const int b = blockIdx.y, fd = s.feat_dim;
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    const SeqCtl &q = s.seq[b];
    if (k >= fd || !(q.seg_on && q.seg_budget > 0)) return;
    bool ready = q.ema_ready != 0;
    float e = s.ema[(size_t)b * fd + k];
    for (int j0 = 0; j0 < n; j0 += 8) {   // the features of 8 tokens loaded together, then the recurrence
        float fv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) fv[i] = j0 + i < n ? feat[((size_t)b * n + j0 + i) * fd + k] : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (j0 + i >= n) break;
            const size_t t = (size_t)b * n + j0 + i;
            const float f = fv[i];
            if (ready) {
                hin[t * fd + k] = sc_hab_in(f, e);
                e = sc_ema_next(e, f);
            } else {   // the stream's first token: no habituated score, the EMA starts at f
                hin[t * fd + k] = f;
                e = f;
                ready = true;
            }
        }
    }
    s.ema[(size_t)b * fd + k] = e;
}

// LayerNorm statistics {mean raw, mean habituated, 1/std raw, 1/std habituated} of every token of the piece (one
// CTA per token; the reduction order of the decode step's scorer)
__global__ void __launch_bounds__(SCORER_THREADS) k_piece_lnstat(const StateDev *sp, int n, const float *feat,
                                                                 const float *hin, float4 *stat) {
    const StateDev &s = *sp;
    const int t = blockIdx.x, b = t / n, fd = s.feat_dim;
    const SeqCtl &q = s.seq[b];
    if (!(q.seg_on && q.seg_budget > 0)) {
        if (threadIdx.x == 0) stat[t] = make_float4(0.f, 0.f, 1.f, 1.f);   // unused: keeps k_piece_fc1's input finite
        return;
    }
    const float *f = feat + (size_t)t * fd, *h = hin + (size_t)t * fd;
    float st[4];
    scorer_ln_stats_block(fd, [=](int k) { return f[k]; }, [=](int k) { return h[k]; }, st);
    if (threadIdx.x == 0) stat[t] = make_float4(st[0], st[1], st[2], st[3]);
}

constexpr int PF_FC1_TOK = 16;    // tokens per CTA
constexpr int PF_FC1_KC = 128;    // features per shared-memory chunk

// fc1 of both LayerNorm inputs for 16 tokens x 8 hidden units per CTA (one warp per unit): the normalised inputs of
// a 128-feature chunk are staged in shared memory once per CTA and every W1 element is read once per 16 tokens.
// Each lane keeps the per-lane order of scorer_fc1_block (k = lane, lane + 32, ... increasing, then the butterfly),
// so every output equals the decode step's bit for bit.
__global__ void __launch_bounds__(SCORER_THREADS) k_piece_fc1(const ModelDev *mp, const StateDev *sp, int T,
                                                              const float *feat, const float *hin, const float4 *stat,
                                                              float *z) {
    const ModelDev &m = *mp;
    const int fd = sp->feat_dim, hdn = m.seg_hidden;
    const int t0 = blockIdx.y * PF_FC1_TOK, nt = min(PF_FC1_TOK, T - t0);
    __shared__ float ln0[PF_FC1_TOK][PF_FC1_KC], ln1[PF_FC1_TOK][PF_FC1_KC];
    __shared__ float4 st[PF_FC1_TOK];
    if (threadIdx.x < PF_FC1_TOK)
        st[threadIdx.x] = (int)threadIdx.x < nt ? stat[t0 + threadIdx.x] : make_float4(0.f, 0.f, 1.f, 1.f);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int u = blockIdx.x * (SCORER_THREADS / 32) + warp;
    const float *w1 = m.sc_w1 + (size_t)min(u, hdn - 1) * fd;
    const float *ln_w = m.sc_ln_w, *ln_b = m.sc_ln_b;
    float s0[PF_FC1_TOK], s1[PF_FC1_TOK];
#pragma unroll
    for (int j = 0; j < PF_FC1_TOK; ++j) s0[j] = s1[j] = 0.f;
    for (int kc = 0; kc < fd; kc += PF_FC1_KC) {
        float wv[PF_FC1_KC / 32];   // this lane's W1 elements of the chunk, loaded while the inputs are staged
#pragma unroll
        for (int i = 0; i < PF_FC1_KC / 32; ++i) {
            const int k = kc + lane + 32 * i;
            wv[i] = k < fd ? __ldg(w1 + k) : 0.f;
        }
        // this thread's inputs of the chunk: every load issued before the first use
        constexpr int PER = PF_FC1_TOK * PF_FC1_KC / SCORER_THREADS;
        float f0[PER], f1[PER], lw[PER], lb[PER];
#pragma unroll
        for (int r = 0; r < PER; ++r) {
            const int i = threadIdx.x + r * SCORER_THREADS, tt = i / PF_FC1_KC, kk = i - tt * PF_FC1_KC, k = kc + kk;
            const bool ok = tt < nt && k < fd;
            f0[r] = ok ? __ldg(feat + (size_t)(t0 + tt) * fd + k) : 0.f;
            f1[r] = ok ? __ldg(hin + (size_t)(t0 + tt) * fd + k) : 0.f;
            lw[r] = ok ? __ldg(ln_w + k) : 0.f;
            lb[r] = ok ? __ldg(ln_b + k) : 0.f;
        }
        __syncthreads();   // the previous chunk is consumed (first pass: st is written)
#pragma unroll
        for (int r = 0; r < PER; ++r) {
            const int i = threadIdx.x + r * SCORER_THREADS, tt = i / PF_FC1_KC, kk = i - tt * PF_FC1_KC, k = kc + kk;
            float v0 = 0.f, v1 = 0.f;
            if (tt < nt && k < fd) {
                const float4 q = st[tt];
                v0 = sc_ln(f0[r], q.x, q.z, lw[r], lb[r]);
                v1 = sc_ln(f1[r], q.y, q.w, lw[r], lb[r]);
            }
            ln0[tt][kk] = v0;
            ln1[tt][kk] = v1;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < PF_FC1_KC / 32; ++i) {
            const int kk = lane + 32 * i;
            if (kc + kk >= fd) break;
#pragma unroll
            for (int j = 0; j < PF_FC1_TOK; ++j) {
                s0[j] = sc_fc1_term(s0[j], wv[i], ln0[j][kk]);
                s1[j] = sc_fc1_term(s1[j], wv[i], ln1[j][kk]);
            }
        }
    }
    if (u >= hdn) return;
    const float bias = m.sc_b1[u];
#pragma unroll
    for (int j = 0; j < PF_FC1_TOK; ++j) {
        const float a0 = warp_sum(s0[j]), a1 = warp_sum(s1[j]);
        if (lane == 0 && j < nt) {
            z[((size_t)(t0 + j) * 2) * hdn + u] = __fadd_rn(a0, bias);
            z[((size_t)(t0 + j) * 2 + 1) * hdn + u] = __fadd_rn(a1, bias);
        }
    }
}

// score of every token of the piece into the score ring (one CTA per token)
__global__ void __launch_bounds__(SCORER_THREADS) k_piece_score(const ModelDev *mp, const StateDev *sp, int n,
                                                                int64_t p0, const float *z) {
    const ModelDev &m = *mp;
    const StateDev &s = *sp;
    const int t = blockIdx.x, b = t / n, j = t - b * n;
    const SeqCtl &q = s.seq[b];
    if (!(q.seg_on && q.seg_budget > 0)) return;
    const int64_t pos = p0 + j;
    const bool ready = q.ema_ready != 0 || j > 0;
    const float sc = scorer_score_block(m, s, b, q, z + (size_t)t * 2 * m.seg_hidden,
                                        z + ((size_t)t * 2 + 1) * m.seg_hidden, ready, pos);
    if (threadIdx.x == 0) s.sc_ring[((size_t)b * 2 + ((pos / m.W) & 1)) * m.W + (int)(pos % m.W)] = sc;
}

// ------------------------------------------------------------------------------------------ GEMM epilogues
// Token t of a piece = (sequence t / n, position p0 + t % n); p0 < 0: the batched decode step (n = 1), whose
// position is read from the state on the device (so a captured step replays at any position).
struct PieceQKV {   // bias + RoPE + KV / sink writes + both query rotations (the QKV epilogue of v3g_step.cu per token)
    StateDev sd;           // the state descriptor by value (its scalars and base pointers stay in registers)
    const float *rope;     // model RoPE table, rows from position rope_pos0
    int rope_pos0;
    int layer, n;
    int64_t p0;
    const float *bq, *bk, *bv;
    float *qc, *qf;   // [tokens][H][D]

    // position bookkeeping of consecutive tokens: sequence b, position pos, window slot c, ring parity par
    struct Cursor {
        int b, jn, c, par;
        int64_t pos;
    };
    __device__ Cursor start(int tok0, int64_t base) const {
        Cursor u;
        u.b = tok0 / n;
        u.jn = tok0 - u.b * n;
        u.pos = base + u.jn;
        u.c = (int)(u.pos % sd.W);
        u.par = (int)((u.pos / sd.W) & 1);
        return u;
    }
    __device__ void advance(Cursor &u, int64_t base) const {
        if (++u.jn == n) {   // next sequence: back to the piece's first position
            u.jn = 0;
            ++u.b;
            u.pos = base;
            u.c = (int)(base % sd.W);
            u.par = (int)((base / sd.W) & 1);
        } else {
            ++u.pos;
            if (++u.c == sd.W) {
                u.c = 0;
                u.par ^= 1;
            }
        }
    }
    __device__ const float *rope_at(int64_t p) const { return rope + (p - rope_pos0) * (int64_t)sd.D; }

    template <int N>
    __device__ void chunk(int seg, int rt, int g, int tok0, int nv, const float (&y0)[N], const float (&y1)[N]) const {
        const int D = sd.D, W = sd.W, hd = D / 2;
        const int head = rt / (D / TILE_ROWS), i = 8 * (rt % (D / TILE_ROWS)) + g;
        const int r0 = head * D + i, r1 = r0 + hd;
        const float *bsrc = seg == 0 ? bq : (seg == 1 ? bk : bv);
        const float b0 = __ldg(bsrc + r0), b1 = __ldg(bsrc + r1);
        const int64_t base = p0 < 0 ? __ldcg(&sd.step->pos) : p0;
        // reads: the RoPE factors of every token (rotations at c and, for queries past the first window, W + c)
        float cs[N], sn[N], fc[N], fs[N];
        Cursor u = start(tok0, base);
#pragma unroll
        for (int j = 0; j < N; ++j) {
            cs[j] = sn[j] = fc[j] = fs[j] = 0.f;
            if (j < nv) {
                const float *rc = rope_at(u.c);
                cs[j] = __ldg(rc + i);
                sn[j] = __ldg(rc + hd + i);
                if (seg == 0 && u.pos >= W) {
                    const float *rf = rope_at(W + u.c);
                    fc[j] = __ldg(rf + i);
                    fs[j] = __ldg(rf + hd + i);
                }
                advance(u, base);
            }
        }
        // writes
        u = start(tok0, base);
#pragma unroll
        for (int j = 0; j < N; ++j) {
            if (j >= nv) break;
            const int tok = tok0 + j;
            const float a = y0[j] + b0, bb = y1[j] + b1;
            if (seg == 0) {
                float *q = qc + ((size_t)tok * sd.H + head) * D;
                q[i] = a * cs[j] - bb * sn[j];
                q[i + hd] = bb * cs[j] + a * sn[j];
                if (u.pos >= W) {
                    float *qq = qf + ((size_t)tok * sd.H + head) * D;
                    qq[i] = a * fc[j] - bb * fs[j];
                    qq[i + hd] = bb * fc[j] + a * fs[j];
                }
            } else if (seg == 1) {
                kv_t *kr = kvp(sd, layer, u.b, ring_off(sd, u.par, KIND_KRAW, head, u.c));
                kv_t *ko = kvp(sd, layer, u.b, ring_off(sd, u.par, KIND_KROT, head, u.c));
                kr[i] = f2kv(a);
                kr[i + hd] = f2kv(bb);
                ko[i] = f2kv(a * cs[j] - bb * sn[j]);
                ko[i + hd] = f2kv(bb * cs[j] + a * sn[j]);
                if (u.pos < sd.sink_cap) {
                    kv_t *sk = kvp(sd, layer, u.b, sink_off(sd, SINK_KRAW, head, (int)u.pos));
                    sk[i] = f2kv(a);
                    sk[i + hd] = f2kv(bb);
                }
            } else {
                kv_t *vv = kvp(sd, layer, u.b, ring_off(sd, u.par, KIND_V, head, u.c));
                vv[i] = f2kv(a);
                vv[i + hd] = f2kv(bb);
                if (u.pos < sd.sink_cap) {
                    kv_t *sv = kvp(sd, layer, u.b, sink_off(sd, SINK_V, head, (int)u.pos));
                    sv[i] = f2kv(a);
                    sv[i + hd] = f2kv(bb);
                }
            }
            advance(u, base);
        }
    }
    __device__ void operator()(int seg, int rt, int g, int tok, float y0, float y1) const {
        const float a0[1] = {y0}, a1[1] = {y1};
        chunk<1>(seg, rt, g, tok, 1, a0, a1);
    }
};

struct TokResid {   // x[t, row] += y (identity row order)
    float *x;
    int ld, rows;
    template <int N>
    __device__ void chunk(int, int rt, int g, int tok0, int nv, const float (&y0)[N], const float (&y1)[N]) const {
        const int r = TILE_ROWS * rt + g;
        float *xr = x + (size_t)tok0 * ld + r;
        float x0[N], x1[N];
#pragma unroll
        for (int j = 0; j < N; ++j) {   // every read first ...
            x0[j] = j < nv && r < rows ? __ldcg(xr + (size_t)j * ld) : 0.f;
            x1[j] = j < nv && r + 8 < rows ? __ldcg(xr + (size_t)j * ld + 8) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < N; ++j) {   // ... then the writes
            if (j >= nv) break;
            if (r < rows) xr[(size_t)j * ld] = x0[j] + y0[j];
            if (r + 8 < rows) xr[(size_t)j * ld + 8] = x1[j] + y1[j];
        }
    }
    __device__ void operator()(int, int rt, int g, int tok, float y0, float y1) const {
        const int r = TILE_ROWS * rt + g;
        float *xr = x + (size_t)tok * ld;
        if (r < rows) xr[r] += y0;
        if (r + 8 < rows) xr[r + 8] += y1;
    }
};

struct TokStore {   // y[t, row] = value (identity row order): logits of the batched lm head
    float *y;
    int64_t ld;
    int rows;
    __device__ void operator()(int, int rt, int g, int tok, float y0, float y1) const {
        const int r = TILE_ROWS * rt + g;
        float *yr = y + (size_t)tok * ld;
        if (r < rows) yr[r] = y0;
        if (r + 8 < rows) yr[r + 8] = y1;
    }
    template <int N>
    __device__ void chunk(int seg, int rt, int g, int tok0, int nv, const float (&y0)[N], const float (&y1)[N]) const {
#pragma unroll
        for (int j = 0; j < N; ++j)
            if (j < nv) (*this)(seg, rt, g, tok0 + j, y0[j], y1[j]);
    }
};

struct TokGateUp {   // h[t, f] = silu(gate_f) * up_f  (src/vault_v3_model.py:1149-1150)
    float *h;
    int F;
    __device__ void operator()(int, int rt, int g, int tok, float gt, float u) const {
        const int f = 8 * rt + g;
        if (f < F) h[(size_t)tok * F + f] = gt / (1.0f + expf(-gt)) * u;
    }
    template <int N>
    __device__ void chunk(int seg, int rt, int g, int tok0, int nv, const float (&y0)[N], const float (&y1)[N]) const {
#pragma unroll
        for (int j = 0; j < N; ++j)
            if (j < nv) (*this)(seg, rt, g, tok0 + j, y0[j], y1[j]);
    }
};

// ------------------------------------------------------------------------------------------ block-window attention
// One CTA per (16 query tokens, KV head g, sequence b) with one warp per query head of the group: the group's K and V
// rows are staged once in shared memory (cp.async, double-buffered 64-key tiles) and shared by its query heads
// (GQA).  Scores and P V run on the tensor cores (mma.sync m16n8k16): queries and probabilities enter as high + low
// fp16 parts (about 22 significant bits), keys and values are the fp16 cache; online softmax in fp32.  Phase 1
// scores the prefix (sinks, bank, previous chunk) with the queries rotated at W + c, phase 2 the current chunk's
// keys 0..c with the queries rotated at c.  p0 < 0: the batched decode step (n = 1), position read from the state.
template <int D>
__global__ void __launch_bounds__(256) k_prefill_attn(const StateDev *sp, int layer, float scale, int n, int64_t p0,
                                                      const float *Qc, const float *Qf, float *out) {
    if (p0 < 0) p0 = __ldcg(&sp->step->pos);
    constexpr int KP = D + 8, NS = D / 16, NB = D / 8, TK = 64;
    extern __shared__ __align__(16) uint8_t smraw[];
    kv_t *Ks = reinterpret_cast<kv_t *>(smraw);   // [2][TK][KP]
    kv_t *Vs = Ks + 2 * TK * KP;                  // [2][TK][KP]
    const StateDev &s = *sp;
    const int b = blockIdx.z, g = blockIdx.y, j0 = blockIdx.x * 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, t = lane & 3;
    const int H = s.H, grp = H / s.G, h = g * grp + warp;
    const int W = s.W, c0 = (int)(p0 % W);
    const KeySpan ks = key_span(s, b, p0);
    const KvRows kr = kv_rows(s, layer, b, g, ks);   // row bases: the staging loop reads no state fields
    const int nfar = ks.n_sk + ks.n_seg + ks.n_prev;
    const int jmax = min(n, j0 + 16);
    const int ncur = c0 + jmax;
    const int r0 = j0 + gq, r1 = r0 + 8;
    const int cr0 = c0 + r0, cr1 = c0 + r1;
    float o[NB][4];
#pragma unroll
    for (int i = 0; i < NB; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    uint32_t qh[NS][4], ql[NS][4];

    auto load_q = [&](const float *Q) {
#pragma unroll
        for (int st = 0; st < NS; ++st) {
#pragma unroll
            for (int reg = 0; reg < 4; ++reg) {
                const int r = (reg & 1) ? r1 : r0;
                const int d0 = 16 * st + 2 * t + ((reg & 2) ? 8 : 0);
                float2 v = make_float2(0.f, 0.f);
                if (r < n) v = __ldg(reinterpret_cast<const float2 *>(Q + (((size_t)b * n + r) * H + h) * D + d0));
                const __half2 hv = __floats2half2_rn(v.x, v.y);
                const float2 back = __half22float2(hv);
                const __half2 lv = __floats2half2_rn(v.x - back.x, v.y - back.y);
                qh[st][reg] = *reinterpret_cast<const uint32_t *>(&hv);
                ql[st][reg] = *reinterpret_cast<const uint32_t *>(&lv);
            }
        }
    };
    // stage keys [k0, k0 + TK) of the phase (visible-key index base + k) into buffer bufi
    auto stage = [&](int bufi, int k0, int nkeys, int base) {
        kv_t *kd = Ks + bufi * TK * KP, *vd = Vs + bufi * TK * KP;
        for (int c = threadIdx.x; c < TK * (D / 8); c += blockDim.x) {
            const int kk = c / (D / 8), part = c - kk * (D / 8);
            if (k0 + kk < nkeys) {
                cp_async16(kd + kk * KP + part * 8, kv_at<D>(kr, base + k0 + kk, false) + part * 8);
                cp_async16(vd + kk * KP + part * 8, kv_at<D>(kr, base + k0 + kk, true) + part * 8);
            } else {   // past the keys: zero values (probability 0 must meet a finite value)
                *reinterpret_cast<uint4 *>(vd + kk * KP + part * 8) = make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4 *>(kd + kk * KP + part * 8) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    auto run = [&](int nkeys, int base, bool causal) {
        const int ntiles = (nkeys + TK - 1) / TK;
        if (ntiles == 0) return;
        stage(0, 0, nkeys, base);
        for (int tile = 0; tile < ntiles; ++tile) {
            const int bi = tile & 1;
            if (tile + 1 < ntiles) {
                stage(bi ^ 1, (tile + 1) * TK, nkeys, base);
                asm volatile("cp.async.wait_group 1;" ::: "memory");
            } else {
                asm volatile("cp.async.wait_group 0;" ::: "memory");
            }
            __syncthreads();
            const kv_t *kt = Ks + bi * TK * KP, *vt = Vs + bi * TK * KP;
            float sc[8][4];
#pragma unroll
            for (int st8 = 0; st8 < 8; ++st8) {
                float c[4] = {0.f, 0.f, 0.f, 0.f};
                const kv_t *krow = kt + (st8 * 8 + gq) * KP + 2 * t;
#pragma unroll
                for (int st = 0; st < NS; ++st) {
                    const uint32_t b0 = ld_h2(krow + 16 * st), b1 = ld_h2(krow + 16 * st + 8);
                    mma16816(c, qh[st][0], qh[st][1], qh[st][2], qh[st][3], b0, b1);
                    mma16816(c, ql[st][0], ql[st][1], ql[st][2], ql[st][3], b0, b1);
                }
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int kidx = tile * TK + st8 * 8 + 2 * t + e;
                    const bool ok = kidx < nkeys;
                    sc[st8][e] = (ok && (!causal || kidx <= cr0)) ? c[e] * scale : -INFINITY;
                    sc[st8][2 + e] = (ok && (!causal || kidx <= cr1)) ? c[2 + e] * scale : -INFINITY;
                }
            }
            // online softmax for rows r0 (elements 0, 1) and r1 (elements 2, 3)
            float mx0 = m0, mx1 = m1;
#pragma unroll
            for (int st8 = 0; st8 < 8; ++st8) {
                mx0 = fmaxf(mx0, fmaxf(sc[st8][0], sc[st8][1]));
                mx1 = fmaxf(mx1, fmaxf(sc[st8][2], sc[st8][3]));
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            const float al0 = mx0 == -INFINITY ? 1.f : expf(m0 - mx0), al1 = mx1 == -INFINITY ? 1.f : expf(m1 - mx1);
            m0 = mx0;
            m1 = mx1;
            float ps0 = 0.f, ps1 = 0.f;
            uint32_t ph[4][4], pl[4][4];   // P as A fragments of the 4 key steps of 16, high and low parts
#pragma unroll
            for (int st8 = 0; st8 < 8; ++st8) {
                const float p00 = sc[st8][0] == -INFINITY ? 0.f : expf(sc[st8][0] - mx0);
                const float p01 = sc[st8][1] == -INFINITY ? 0.f : expf(sc[st8][1] - mx0);
                const float p10 = sc[st8][2] == -INFINITY ? 0.f : expf(sc[st8][2] - mx1);
                const float p11 = sc[st8][3] == -INFINITY ? 0.f : expf(sc[st8][3] - mx1);
                ps0 += p00 + p01;
                ps1 += p10 + p11;
                const __half2 h0 = __floats2half2_rn(p00, p01), h1 = __floats2half2_rn(p10, p11);
                const float2 b0 = __half22float2(h0), b1 = __half22float2(h1);
                const __half2 lo0 = __floats2half2_rn(p00 - b0.x, p01 - b0.y), lo1 = __floats2half2_rn(p10 - b1.x, p11 - b1.y);
                const int kk = st8 >> 1, hi8 = st8 & 1;   // key step, second half of its 16 keys
                ph[kk][0 + 2 * hi8] = *reinterpret_cast<const uint32_t *>(&h0);
                ph[kk][1 + 2 * hi8] = *reinterpret_cast<const uint32_t *>(&h1);
                pl[kk][0 + 2 * hi8] = *reinterpret_cast<const uint32_t *>(&lo0);
                pl[kk][1 + 2 * hi8] = *reinterpret_cast<const uint32_t *>(&lo1);
            }
            ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
            ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
            ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
            ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
            l0 = l0 * al0 + ps0;
            l1 = l1 * al1 + ps1;
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
                o[nb][0] *= al0;
                o[nb][1] *= al0;
                o[nb][2] *= al1;
                o[nb][3] *= al1;
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                    uint32_t b0, b1;
                    ldsm_x2_trans(b0, b1, vt + (16 * kk + (lane & 15)) * KP + 8 * nb);
                    mma16816(o[nb], ph[kk][0], ph[kk][1], ph[kk][2], ph[kk][3], b0, b1);
                    mma16816(o[nb], pl[kk][0], pl[kk][1], pl[kk][2], pl[kk][3], b0, b1);
                }
            }
            __syncthreads();   // every warp is done with this buffer before it is refilled
        }
    };
    if (nfar > 0) {
        load_q(Qf);
        run(nfar, 0, false);
    }
    load_q(Qc);
    run(ncur, nfar, true);
    const float i0 = 1.f / l0, i1 = 1.f / l1;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
        const int d0 = 8 * nb + 2 * t;
        if (r0 < n)
            *reinterpret_cast<float2 *>(out + (((size_t)b * n + r0) * H + h) * D + d0) = make_float2(o[nb][0] * i0, o[nb][1] * i0);
        if (r1 < n)
            *reinterpret_cast<float2 *>(out + (((size_t)b * n + r1) * H + h) * D + d0) = make_float2(o[nb][2] * i1, o[nb][3] * i1);
    }
}

template <int D>
static cudaError_t launch_prefill_attn(const v3g_model *m, v3g_state *s, int layer, int n, int64_t p0,
                                       const float *qc, const float *qf, float *out, cudaStream_t st) {
    const size_t smem = (size_t)4 * 64 * (D + 8) * sizeof(kv_t);   // attribute set by tc_init_attrs
    dim3 grid((n + 15) / 16, m->host.G, s->B);
    k_prefill_attn<D><<<grid, 32 * (m->host.H / m->host.G), smem, st>>>(s->dev, layer, (float)(1.0 / sqrt((double)D)), n, p0,
                                                                        qc, qf, out);
    return cudaGetLastError();
}

// n queries per sequence at positions p0.. (p0 < 0: one query at the state's position); queries and outputs default
// to the prefill workspace
static cudaError_t prefill_attention(const v3g_model *m, v3g_state *s, int layer, int n, int64_t p0, cudaStream_t st,
                                     const float *qc = nullptr, const float *qf = nullptr, float *out = nullptr) {
    if (!qc) {
        qc = s->pf.qc;
        qf = s->pf.qf;
        out = s->pf.attn;
    }
    switch (m->host.D) {
        case 16: return launch_prefill_attn<16>(m, s, layer, n, p0, qc, qf, out, st);
        case 32: return launch_prefill_attn<32>(m, s, layer, n, p0, qc, qf, out, st);
        case 64: return launch_prefill_attn<64>(m, s, layer, n, p0, qc, qf, out, st);
        case 128: return launch_prefill_attn<128>(m, s, layer, n, p0, qc, qf, out, st);
        default: return cudaErrorInvalidValue;
    }
}

// ------------------------------------------------------------------------------------------ host orchestration
// Large dynamic shared memory for every tensor-core kernel instantiation this file launches; called at state set-up
// (never inside a stream capture).
template <class Epi>
static cudaError_t tc_attrs_for() {
    cudaError_t e = cudaSuccess;
    auto set = [&](const void *f) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    };
    set((const void *)k_gemm_tc<FMT_Q8, FMT_Q8, Epi>);
    set((const void *)k_gemm_tc<FMT_Q4, FMT_Q8, Epi>);
    set((const void *)k_gemm_tc<FMT_Q4, FMT_Q4, Epi>);
    set((const void *)k_gemm_tc<FMT_BF16, FMT_BF16, Epi>);
    set((const void *)k_gemm_tc<FMT_F16, FMT_F16, Epi>);
    return e;
}

cudaError_t tc_init_attrs() {
    cudaError_t e = tc_attrs_for<PieceQKV>();
    if (e == cudaSuccess) e = tc_attrs_for<TokResid>();
    if (e == cudaSuccess) e = tc_attrs_for<TokGateUp>();
    if (e == cudaSuccess) e = tc_attrs_for<TokStore>();
    const int D[4] = {16, 32, 64, 128};
    const void *fn[4] = {(const void *)k_prefill_attn<16>, (const void *)k_prefill_attn<32>,
                         (const void *)k_prefill_attn<64>, (const void *)k_prefill_attn<128>};
    for (int i = 0; i < 4 && e == cudaSuccess; ++i)
        e = cudaFuncSetAttribute(fn[i], cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * 64 * (D[i] + 8) * 2);
    return e;
}
bool piece_supported(const v3g_model *m, const v3g_state *s) {
    const ModelDev &md = m->host;
    if (!s->pf.x || s->pf.cap < 1) return false;
    auto ok = [](const MatW &w) { return w.fmt == FMT_Q8 || w.fmt == FMT_Q4 || w.fmt == FMT_BF16 || w.fmt == FMT_F16; };
    for (int l = 0; l < md.n_layers; ++l) {
        const LayerW &L = md.layers[l];
        if (!ok(L.q) || !ok(L.k) || !ok(L.v) || !ok(L.o) || !ok(L.gu) || !ok(L.down)) return false;
    }
    return true;
}

// n tokens per sequence (ids row b at dev_ids + b ld, columns i0 ..), starting at host position p0; the piece stays
// inside one window chunk.  want_lm: the last token's logits into s.logits and its greedy token into tok_in.
cudaError_t launch_piece(const v3g_model *m, v3g_state *s, const int32_t *dev_ids, int64_t ld, int64_t i0, int n,
                         int64_t p0, bool want_lm, cudaStream_t st) {
    const ModelDev &md = m->host;
    const StateDev &sd = s->host;
    const PfBuf &pf = s->pf;
    const int B = s->B, T = B * n;
    const bool boundary = p0 > 0 && p0 % md.W == 0;
    int *status = &sd.step->status;
    cudaError_t e;
#define PF_TRY(x)                               \
    do {                                        \
        if ((e = (x)) != cudaSuccess) return e; \
    } while (0)
    if (boundary) {   // the boundary kernels read each sequence's boundary token from tok_in (k_pin)
        PF_TRY(cudaMemcpy2DAsync(sd.tok_in, sizeof(int32_t), dev_ids + i0, (size_t)ld * sizeof(int32_t), sizeof(int32_t),
                                 (size_t)B, cudaMemcpyDeviceToDevice, st));
        PF_TRY(launch_boundary(m, s, st));
    }
    const int slices = std::max(1, std::min(32, (n * md.d) / (256 * 64)));   // about 64 embedding values a thread
    k_piece_begin<<<dim3(B, slices), 256, (size_t)n * 3 * sizeof(int), st>>>(m->dev, s->dev, dev_ids, ld, i0, n, p0,
                                                                               boundary ? 0 : 1, pf.x);
    PF_TRY(cudaGetLastError());
    const int HD = md.H * md.D;
    const bool any_seg = md.seg_n_feat > 0 && s->seg_budget > 0;
    for (int l = 0; l < md.n_layers; ++l) {
        const LayerW &L = md.layers[l];
        for (int fi = 0; fi < md.seg_n_feat && any_seg; ++fi)
            if (md.seg_layers[fi] == l)   // scorer features: residual stream entering this layer, every token
                PF_TRY(cudaMemcpy2DAsync(pf.feat + (size_t)fi * md.d, (size_t)sd.feat_dim * 4, pf.x, (size_t)md.d * 4,
                                         (size_t)md.d * 4, (size_t)T, cudaMemcpyDeviceToDevice, st));
        PF_TRY(tc_prep(pf.x, md.d, T, md.d, L.ln1, md.rms_eps, pf.x16, pf.ldx16, pf.xscale, st));
        {
            const MatW *mats[3] = {&L.q, &L.k, &L.v};
            PieceQKV epi{s->host, md.rope, md.rope_pos0, l, n, p0, L.bq, L.bk, L.bv, pf.qc, pf.qf};
            PF_TRY(tc_gemm(mats, 3, pf.x16, pf.ldx16, pf.xscale, T, status, m->n_sm, epi, st, &pf.sk));
        }
        PF_TRY(prefill_attention(m, s, l, n, p0, st));
        PF_TRY(tc_prep(pf.attn, HD, T, HD, nullptr, 0.f, pf.x16, pf.ldx16, pf.xscale, st));
        {
            const MatW *mats[1] = {&L.o};
            TokResid epi{pf.x, md.d, md.d};
            PF_TRY(tc_gemm(mats, 1, pf.x16, pf.ldx16, pf.xscale, T, status, m->n_sm, epi, st, &pf.sk));
        }
        PF_TRY(tc_prep(pf.x, md.d, T, md.d, L.ln2, md.rms_eps, pf.x16, pf.ldx16, pf.xscale, st));
        {
            const MatW *mats[1] = {&L.gu};
            TokGateUp epi{pf.h, md.F};
            PF_TRY(tc_gemm(mats, 1, pf.x16, pf.ldx16, pf.xscale, T, status, m->n_sm, epi, st, &pf.sk));
        }
        PF_TRY(tc_prep(pf.h, md.F, T, md.F, nullptr, 0.f, pf.x16, pf.ldx16, pf.xscale, st));
        {
            const MatW *mats[1] = {&L.down};
            TokResid epi{pf.x, md.d, md.d};
            PF_TRY(tc_gemm(mats, 1, pf.x16, pf.ldx16, pf.xscale, T, status, m->n_sm, epi, st, &pf.sk));
        }
    }
    if (any_seg) {
        k_piece_scan<<<dim3((sd.feat_dim + 255) / 256, B), 256, 0, st>>>(s->dev, n, pf.feat, pf.hin);
        k_piece_lnstat<<<T, SCORER_THREADS, 0, st>>>(s->dev, n, pf.feat, pf.hin, pf.stat);
        k_piece_fc1<<<dim3((md.seg_hidden + 7) / 8, (T + PF_FC1_TOK - 1) / PF_FC1_TOK), SCORER_THREADS, 0, st>>>(
            m->dev, s->dev, T, pf.feat, pf.hin, pf.stat, pf.z);
        k_piece_score<<<T, SCORER_THREADS, 0, st>>>(m->dev, s->dev, n, p0, pf.z);
        PF_TRY(cudaGetLastError());
    }
    if (want_lm) {   // the last token of every sequence: rows (b n + n - 1) of x, stride n d
        PF_TRY(launch_lm_head(m, s, pf.x + (size_t)(n - 1) * md.d, n * md.d, st));
        PF_TRY(launch_argmax_only(m, s, st));
    }
    k_piece_finish<<<1, 256, 0, st>>>(s->dev, n, want_lm ? 1 : 0);
    PF_TRY(cudaGetLastError());
#undef PF_TRY
    return cudaSuccess;
}

// One decode step of a batch of B > 8 sequences with every projection on the tensor-core GEMM (N = B tokens, so
// each weight byte is read once per step): the step kernels of v3g_step.cu for the token bookkeeping, chunk
// boundary, split-KV attention, segment scorer and argmax, the GEMMs for QKV (fused bias / RoPE / KV writes), O,
// gate/up and down, and the tied lm head.  Positions come from the device state: the sequence can be captured.
cudaError_t launch_step_tc(const v3g_model *m, v3g_state *s, bool boundary, bool want_lm, cudaStream_t st) {
    const ModelDev &md = m->host;
    const StateDev &sd = s->host;
    const PfBuf &pf = s->pf;
    const int B = s->B, HD = md.H * md.D;
    const bool any_seg = md.seg_n_feat > 0 && s->seg_budget > 0;
    int *status = &sd.step->status;
    cudaError_t e;
#define TS_TRY(x)                               \
    do {                                        \
        if ((e = (x)) != cudaSuccess) return e; \
    } while (0)
    TS_TRY(launch_step_begin(m, s, boundary, st));
    for (int l = 0; l < md.n_layers; ++l) {
        const LayerW &L = md.layers[l];
        for (int fi = 0; fi < md.seg_n_feat && any_seg; ++fi)
            if (md.seg_layers[fi] == l)   // scorer features: residual stream entering this layer
                TS_TRY(cudaMemcpy2DAsync(sd.feat + (size_t)fi * md.d, (size_t)sd.feat_dim * 4, sd.x, (size_t)md.d * 4,
                                         (size_t)md.d * 4, (size_t)B, cudaMemcpyDeviceToDevice, st));
        TS_TRY(tc_prep(sd.x, md.d, B, md.d, L.ln1, md.rms_eps, pf.x16, pf.ldx16, pf.xscale, st));
        {
            const MatW *mats[3] = {&L.q, &L.k, &L.v};
            PieceQKV epi{s->host, md.rope, md.rope_pos0, l, 1, -1, L.bq, L.bk, L.bv, sd.q_cur, sd.q_far};
            TS_TRY(tc_gemm(mats, 3, pf.x16, pf.ldx16, pf.xscale, B, status, m->n_sm, epi, st, &pf.sk));
        }
        TS_TRY(launch_attention(m, s, l, false, st));
        TS_TRY(tc_prep(sd.attn, HD, B, HD, nullptr, 0.f, pf.x16, pf.ldx16, pf.xscale, st));
        {
            const MatW *mats[1] = {&L.o};
            TokResid epi{sd.x, md.d, md.d};
            TS_TRY(tc_gemm(mats, 1, pf.x16, pf.ldx16, pf.xscale, B, status, m->n_sm, epi, st, &pf.sk));
        }
        TS_TRY(tc_prep(sd.x, md.d, B, md.d, L.ln2, md.rms_eps, pf.x16, pf.ldx16, pf.xscale, st));
        {
            const MatW *mats[1] = {&L.gu};
            TokGateUp epi{sd.hbuf, md.F};
            TS_TRY(tc_gemm(mats, 1, pf.x16, pf.ldx16, pf.xscale, B, status, m->n_sm, epi, st, &pf.sk));
        }
        TS_TRY(tc_prep(sd.hbuf, md.F, B, md.F, nullptr, 0.f, pf.x16, pf.ldx16, pf.xscale, st));
        {
            const MatW *mats[1] = {&L.down};
            TokResid epi{sd.x, md.d, md.d};
            TS_TRY(tc_gemm(mats, 1, pf.x16, pf.ldx16, pf.xscale, B, status, m->n_sm, epi, st, &pf.sk));
        }
    }
    if (any_seg) TS_TRY(launch_scorer(m, s, st));
    if (want_lm) {
        TS_TRY(tc_prep(sd.x, md.d, B, md.d, md.norm, md.rms_eps, pf.x16, pf.ldx16, pf.xscale, st));
        const MatW *mats[1] = {&md.embed};
        TokStore epi{sd.logits, md.vocab, md.vocab};
        TS_TRY(tc_gemm(mats, 1, pf.x16, pf.ldx16, pf.xscale, B, status, m->n_sm, epi, st, &pf.sk));
    }
    TS_TRY(launch_argmax_finish(m, s, want_lm, false, st));
#undef TS_TRY
    return cudaSuccess;
}

// the decode attention of `layer` as the state's step runs it (kernel-level timing entry v3g_attention)
cudaError_t launch_step_attention(const v3g_model *m, v3g_state *s, int layer, cudaStream_t st) {
    return launch_attention(m, s, layer, false, st);
}

bool step_tc_supported(const v3g_model *m, const v3g_state *s) {
    const ModelDev &md = m->host;
    auto ok = [](const MatW &w) { return w.fmt == FMT_Q8 || w.fmt == FMT_Q4 || w.fmt == FMT_BF16 || w.fmt == FMT_F16; };
    if (!s->pf.x16 || s->pf.cap < s->B || !ok(md.embed)) return false;
    for (int l = 0; l < md.n_layers; ++l) {
        const LayerW &L = md.layers[l];
        if (!ok(L.q) || !ok(L.k) || !ok(L.v) || !ok(L.o) || !ok(L.gu) || !ok(L.down)) return false;
    }
    return true;
}

}  // namespace v3g
