// Output side of the token loop on the device, one CTA per logit row:
//
// * Top-k + temperature sampling: the reference's v3_sample_topk (runtime/vault3.c:3204-3230, declared
//   runtime/vault3.h:221).
//     temp <= 0 or k <= 1: the greedy token (first maximum, v3_argmax, runtime/vault3.c:3198-3202);
//     otherwise, with k capped at 64: the k largest logits, ordered by value (descending) and, among equal values,
//     by index (ascending) -- the order the reference's insertion list produces -- then
//       p[j] = expf_ref((val[j] - val[0]) / temp),  sum = p[0] + p[1] + ... (in order),
//       x = xorshift64(rng) (13, 7, 17; a zero state starts from 0x9E3779B97F4A7C15), rng <- x,
//       r = ((x >> 40) & 0xFFFFFF) / 2^24 * sum, and the first j with (r -= p[j]) <= 0 gives the token.
//   expf_ref is the reference's own exponential (v3_expf, runtime/vault3.c:104-114: Cody-Waite reduction with a
//   degree-7 polynomial) restated with explicitly rounded operations; the whole draw runs on one thread in the
//   reference's operation order.
//
// * The CAAI output governor (runtime/vault3.c:2814-3194): k_govern masks the candidates whose bytes would complete
//   a forbidden pattern, k_gov_commit appends the chosen token to each sequence's stream; the host builds the rules.
//
// Selection (both): every logit becomes the 64-bit key (order-preserving float bits << 32) | (2^32 - 1 - index),
// the key of the greedy token in k_argmax_partial, so "larger key" = "larger value, or equal value and smaller
// index" (-0.0 equals +0.0).  The k-th largest key among the eligible logits is found by an 8-pass radix select
// (8 bits per pass, shared-memory histograms) and the keys at or above it are collected.  No global scratch.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/vault_b200.h"
#include "v3g.cuh"
#include "v3g_gov.cuh"
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

__device__ __forceinline__ uint32_t key_index(uint64_t key) { return 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFu); }

struct SelectSmem {
    unsigned int hist[256];
    uint64_t sel[SAMPLE_KMAX];
    uint64_t prefix;
    int need, cnt;
};

// The keys of the min(kk, #eligible) largest eligible logits of a row, in sm.sel[0..n) in no particular order;
// returns n (the same on every thread).  kk <= SAMPLE_KMAX.  Entered and left by the whole CTA.
template <class Eligible>
__device__ int select_top_keys(const float *lg, uint32_t vocab, uint32_t kk, Eligible eligible, SelectSmem &sm) {
    const int tid = threadIdx.x, nt = blockDim.x;
    if (tid == 0) {
        sm.prefix = 0ull;
        sm.need = (int)kk;
        sm.cnt = 0;
    }
    // radix select of the need-th largest key, 8 bits per pass from the top
    for (int pass = 0; pass < 8; ++pass) {
        const int shift = 56 - 8 * pass;
        for (int b = tid; b < 256; b += nt) sm.hist[b] = 0u;
        __syncthreads();
        const uint64_t pre = sm.prefix;
        for (uint32_t i = tid; i < vocab; i += nt) {
            const float v = lg[i];
            if (!eligible(v)) continue;
            const uint64_t key = logit_key(v, i);
            if (pass == 0 || (key >> (shift + 8)) == (pre >> (shift + 8)))
                atomicAdd(&sm.hist[(unsigned)(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            if (pass == 0) {   // fewer eligible logits than k: take them all
                unsigned int total = 0u;
                for (int b = 0; b < 256; ++b) total += sm.hist[b];
                if ((unsigned)sm.need > total) sm.need = (int)total;
            }
            int digit = 0;
            if (sm.need > 0) {
                unsigned int cum = 0u;
                for (int b = 255; b >= 0; --b) {
                    if (cum + sm.hist[b] >= (unsigned)sm.need) {
                        digit = b;
                        sm.need -= (int)cum;
                        break;
                    }
                    cum += sm.hist[b];
                }
            }
            sm.prefix = pre | ((uint64_t)digit << shift);
        }
        __syncthreads();
    }
    // the keys at or above the selected one: exactly min(k, #eligible) of them (keys are distinct)
    const uint64_t kth = sm.prefix;
    const bool any = sm.need > 0;
    for (uint32_t i = tid; i < vocab && any; i += nt) {
        const float v = lg[i];
        if (!eligible(v)) continue;
        const uint64_t key = logit_key(v, i);
        if (key >= kth) {
            const int slot = atomicAdd(&sm.cnt, 1);
            if (slot < SAMPLE_KMAX) sm.sel[slot] = key;
        }
    }
    __syncthreads();
    return sm.cnt < SAMPLE_KMAX ? sm.cnt : SAMPLE_KMAX;
}

// tokens[row] gets the draw; out (when not null) also gets it at out[row * out_ld] (the generation token sink)
__global__ void __launch_bounds__(SAMPLE_THREADS) k_sample_topk(const float *logits, uint32_t vocab, uint64_t ld,
                                                               uint32_t k, float temp, uint64_t *rng,
                                                               int32_t *tokens, int32_t *out, int64_t out_ld) {
    const int tid = threadIdx.x, nt = blockDim.x;
    const float *lg = logits + (size_t)blockIdx.x * ld;
    __shared__ SelectSmem sm;
    __shared__ uint64_t sorted[SAMPLE_KMAX];
    __shared__ unsigned long long best;
    auto emit = [&](int32_t tok) {
        tokens[blockIdx.x] = tok;
        if (out) out[(int64_t)blockIdx.x * out_ld] = tok;
    };
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
        if (tid == 0) emit(best ? (int32_t)key_index(best) : 0);
        return;
    }
    const uint32_t kk = k > (uint32_t)SAMPLE_KMAX ? (uint32_t)SAMPLE_KMAX : k;
    const int n = select_top_keys(lg, vocab, kk, [](float v) { return v == v; }, sm);
    if (tid < n) {   // rank by counting larger keys
        const uint64_t mine = sm.sel[tid];
        int rank = 0;
        for (int j = 0; j < n; ++j) rank += sm.sel[j] > mine ? 1 : 0;
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
    const float v0 = lg[key_index(sorted[0])];
    for (int j = 0; j < n; ++j) {
        idx[j] = (int32_t)key_index(sorted[j]);
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

// ------------------------------------------------------------------------------------------------------ governor
struct TokBytes {
    const uint8_t *pool;
    const uint32_t *off;
    const uint16_t *len;
    uint32_t vocab;
};

// The decoded bytes of one base64 / hex tail complete a rule within their last `bound` canonical bytes
// (runtime/vault3.c:3080-3083 and :3121-3124).
__device__ bool gov_decoded_hits(const v3g_gov_rules_t &g, const uint8_t *dec, uint32_t dl, uint32_t bound) {
    uint8_t dh[V3G_GOV_HIST_CAP], rem[4];
    uint32_t dhl = 0, rl = 0;
    gov_feed(dh, dhl, V3G_GOV_HIST_CAP, rem, rl, dec, dl);
    return gov_match(g, dh, dhl, dhl > bound ? dhl - bound : 0);
}

// The stream's raw tail followed by the candidate's bytes ends in a base64 or hex run whose decoding completes a rule
// (runtime/vault3.c:3032-3131): base64 at the 4 group phases over the last <= 128 symbols (line breaks skipped, up
// to two '=' stripped), hex at the 2 nibble phases over the last <= 192 digits (separators and 0x prefixes skipped).
__device__ bool gov_encoded_tail_hits(const v3g_gov_rules_t &g, const v3g_gov_stream_t &s, const uint8_t *tb,
                                      uint32_t tbl) {
    const uint32_t take = tbl < 64u ? tbl : 64u;
    bool b64 = false, hex = false;
    for (uint32_t i = 0; i < take; ++i) {
        b64 = b64 || gov_b64(tb[i]) >= 0;
        hex = hex || gov_hex(tb[i]) >= 0;
    }
    if (!b64 && !hex) return false;
    uint8_t comb[V3G_GOV_RAW_CAP + 64];
    uint32_t cl = 0;
    const uint32_t raw = s.raw_len < V3G_GOV_RAW_CAP ? s.raw_len : V3G_GOV_RAW_CAP;
    for (uint32_t i = 0; i < raw; ++i) comb[cl++] = s.raw_tail[i];
    for (uint32_t i = 0; i < take; ++i) comb[cl++] = tb[i];
    const uint32_t bound = take + 3u;
    uint8_t sym[192], dec[96];
    if (b64) {
        uint32_t end = cl;
        while (end > 0 && (comb[end - 1] == '\r' || comb[end - 1] == '\n')) --end;
        for (int eq = 0; eq < 2 && end > 0 && comb[end - 1] == '='; ++eq) --end;
        uint32_t start = end, run = 0;
        while (start > 0 && run < 128u) {
            const uint8_t ch = comb[start - 1];
            if (ch == '\r' || ch == '\n') {
                --start;
            } else if (gov_b64(ch) >= 0) {
                --start;
                ++run;
            } else {
                break;
            }
        }
        if (run >= 8u) {
            uint32_t ns = 0;
            for (uint32_t i = start; i < end && ns < 128u; ++i) {
                const int v = gov_b64(comb[i]);
                if (v >= 0) sym[ns++] = (uint8_t)v;
            }
            for (uint32_t ph = 0; ph < 4u && ph + 6u <= ns; ++ph) {
                uint32_t left = ns - ph, p = ph, dl = 0;
                while (left >= 4u && dl + 3u <= sizeof(dec)) {
                    const uint32_t v = ((uint32_t)sym[p] << 18) | ((uint32_t)sym[p + 1] << 12) |
                                       ((uint32_t)sym[p + 2] << 6) | (uint32_t)sym[p + 3];
                    dec[dl++] = (uint8_t)(v >> 16);
                    dec[dl++] = (uint8_t)(v >> 8);
                    dec[dl++] = (uint8_t)v;
                    p += 4;
                    left -= 4;
                }
                if (left == 3u && dl + 2u <= sizeof(dec)) {
                    const uint32_t v = ((uint32_t)sym[p] << 18) | ((uint32_t)sym[p + 1] << 12) | ((uint32_t)sym[p + 2] << 6);
                    dec[dl++] = (uint8_t)(v >> 16);
                    dec[dl++] = (uint8_t)(v >> 8);
                } else if (left == 2u && dl + 1u <= sizeof(dec)) {
                    dec[dl++] = (uint8_t)((((uint32_t)sym[p] << 18) | ((uint32_t)sym[p + 1] << 12)) >> 16);
                }
                if (gov_decoded_hits(g, dec, dl, bound)) return true;
            }
        }
    }
    if (hex) {
        uint32_t start = cl, run = 0;
        while (start > 0 && run < 192u) {
            const uint8_t ch = comb[start - 1];
            if (gov_hex(ch) >= 0) {
                --start;
                ++run;
            } else if (gov_hex_sep(ch)) {
                --start;
            } else {
                break;
            }
        }
        if (run >= 8u) {
            uint32_t nn = 0;
            for (uint32_t i = start; i < cl && nn < 192u;) {
                if (comb[i] == '0' && i + 2 < cl && (comb[i + 1] == 'x' || comb[i + 1] == 'X') && gov_hex(comb[i + 2]) >= 0) {
                    i += 2;   // a 0x prefix
                    continue;
                }
                const int v = gov_hex(comb[i]);
                if (v >= 0) sym[nn++] = (uint8_t)v;
                ++i;
            }
            for (uint32_t ph = 0; ph < 2u && ph + 8u <= nn; ++ph) {
                uint32_t dl = 0;
                for (uint32_t p = ph; p + 1 < nn && dl < sizeof(dec); p += 2) dec[dl++] = (uint8_t)((sym[p] << 4) | sym[p + 1]);
                if (gov_decoded_hits(g, dec, dl, bound)) return true;
            }
        }
    }
    return false;
}

// Would emitting these bytes after the stream complete a rule (runtime/vault3.c:3157-3175)?  At most the last 31
// history bytes are kept ahead of the candidate's bytes.
__device__ bool gov_candidate_hits(const v3g_gov_rules_t &g, const v3g_gov_stream_t &s, const uint8_t *tb,
                                   uint32_t tbl) {
    uint8_t h[V3G_GOV_HIST_CAP], rem[4];
    uint32_t hl = s.hist_len < V3G_GOV_HIST_CAP ? s.hist_len : V3G_GOV_HIST_CAP;
    uint32_t rl = s.utf8_len < 4u ? s.utf8_len : 3u;
    const uint32_t drop = hl > 31u ? hl - 31u : 0u;
    for (uint32_t i = drop; i < hl; ++i) h[i - drop] = s.hist[i];
    hl -= drop;
    for (uint32_t i = 0; i < rl; ++i) rem[i] = s.utf8_rem[i];
    const uint32_t prev = hl;
    gov_feed(h, hl, V3G_GOV_HIST_CAP, rem, rl, tb, tbl);
    return gov_match(g, h, hl, prev) || gov_encoded_tail_hits(g, s, tb, tbl);
}

// v3_govern_logits per row: up to 4 passes; each selects the top kk logits above -3e38 (as they stand when the pass
// starts) and masks every candidate whose bytes hit a rule; a pass that masks nothing ends the row.
__global__ void __launch_bounds__(SAMPLE_THREADS) k_govern(TokBytes tok, v3g_gov_rules_t rules,
                                                          const v3g_gov_stream_t *streams, float *logits,
                                                          uint64_t ld, uint32_t kk) {
    float *lg = logits + (size_t)blockIdx.x * ld;
    __shared__ SelectSmem sm;
    __shared__ int masked;
    const v3g_gov_stream_t &s = streams[blockIdx.x];
    for (int pass = 0; pass < 4; ++pass) {
        if (threadIdx.x == 0) masked = 0;
        const int n = select_top_keys(lg, tok.vocab, kk, [](float v) { return v > -3.0e38f; }, sm);
        if ((int)threadIdx.x < n) {
            const uint32_t id = key_index(sm.sel[threadIdx.x]);
            const uint32_t len = tok.len[id];
            if (len > 0 && gov_candidate_hits(rules, s, tok.pool + tok.off[id], len)) {
                lg[id] = -3.4e38f;
                masked = 1;
            }
        }
        __syncthreads();
        const bool again = masked != 0;
        __syncthreads();   // every thread has read `masked` before the next pass clears it
        if (!again) break;
    }
}

// v3_gov_commit per row (one thread each)
__global__ void k_gov_commit(TokBytes tok, uint32_t n_rules, int eos, int im_end, int im_start,
                             v3g_gov_stream_t *streams, const int32_t *tokens, uint32_t rows) {
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= rows || n_rules == 0) return;
    v3g_gov_stream_t &s = streams[b];
    const int id = tokens[b];
    if (id == eos || id == im_end || id == im_start) {
        s.hist_len = s.utf8_len = s.raw_len = 0;
        return;
    }
    if (id < 0 || (uint32_t)id >= tok.vocab || tok.len[id] == 0) return;
    const uint8_t *tb = tok.pool + tok.off[id];
    const uint32_t tbl = tok.len[id];
    uint32_t hl = s.hist_len < V3G_GOV_HIST_CAP ? s.hist_len : V3G_GOV_HIST_CAP;
    uint32_t rl = s.utf8_len < 4u ? s.utf8_len : 3u;
    gov_feed(s.hist, hl, V3G_GOV_HIST_CAP, s.utf8_rem, rl, tb, tbl);
    s.hist_len = hl;
    s.utf8_len = rl;
    uint32_t raw = s.raw_len < V3G_GOV_RAW_CAP ? s.raw_len : V3G_GOV_RAW_CAP;
    for (uint32_t i = 0; i < tbl; ++i) {
        if (raw < V3G_GOV_RAW_CAP) {
            s.raw_tail[raw++] = tb[i];
        } else {
            for (uint32_t j = 1; j < V3G_GOV_RAW_CAP; ++j) s.raw_tail[j - 1] = s.raw_tail[j];
            s.raw_tail[V3G_GOV_RAW_CAP - 1] = tb[i];
        }
    }
    s.raw_len = raw;
}

static TokBytes tok_bytes(const v3g_model *m) {
    return TokBytes{m->host.tok_pool, m->host.tok_off, m->host.tok_len, (uint32_t)m->host.vocab};
}

cudaError_t launch_govern(const v3g_model *m, const v3g_gov_rules_t &rules, const v3g_gov_stream_t *streams,
                          float *logits, uint32_t rows, uint64_t ld, uint32_t top_k_guard, cudaStream_t st) {
    if (rules.n_rules == 0 || rows == 0) return cudaSuccess;
    uint32_t kk = (top_k_guard == 0 || top_k_guard > (uint32_t)SAMPLE_KMAX) ? (uint32_t)SAMPLE_KMAX : top_k_guard;
    if (kk > (uint32_t)m->host.vocab) kk = (uint32_t)m->host.vocab;
    k_govern<<<rows, SAMPLE_THREADS, 0, st>>>(tok_bytes(m), rules, streams, logits, ld, kk);
    return cudaGetLastError();
}

cudaError_t launch_gov_commit(const v3g_model *m, const v3g_gov_rules_t &rules, v3g_gov_stream_t *streams,
                              const int32_t *tokens, uint32_t rows, cudaStream_t st) {
    if (rules.n_rules == 0 || rows == 0) return cudaSuccess;
    k_gov_commit<<<(rows + 127) / 128, 128, 0, st>>>(tok_bytes(m), rules.n_rules, (int)m->eos_id, m->host.im_end_id,
                                                     m->host.im_start_id, streams, tokens, rows);
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

// ------------------------------------------------------------------------------------------ governor rules (host)
extern "C" void v3g_gov_init(v3g_gov_rules_t *g) {
    if (g) memset(g, 0, sizeof(*g));
}

extern "C" int v3g_gov_add_rule(v3g_gov_rules_t *g, const uint8_t *pat, size_t len) {
    if (!g || !pat || len == 0) return V3G_E_SIZE;
    uint8_t canon[V3G_GOV_RULE_CAP], rem[4];
    uint32_t cl = 0, rl = 0;
    gov_feed(canon, cl, V3G_GOV_RULE_CAP, rem, rl, pat, len);
    if (cl < 4) return V3G_E_SIZE;
    const uint32_t nr = g->n_rules < V3G_GOV_MAX_RULES ? g->n_rules : V3G_GOV_MAX_RULES;
    for (uint32_t r = 0; r < nr; ++r)
        if (g->rule_len[r] == cl && memcmp(g->rules[r], canon, cl) == 0) return V3G_OK;
    if (nr >= V3G_GOV_MAX_RULES) return V3G_E_LIMIT;
    memcpy(g->rules[nr], canon, cl);
    g->rule_len[nr] = cl;
    g->n_rules = nr + 1;
    return V3G_OK;
}

// ASCII-case-insensitive substring test (the cue is lower-case)
static bool contains_ci(const uint8_t *s, size_t n, const char *cue) {
    const size_t m = strlen(cue);
    for (size_t i = 0; i + m <= n; ++i) {
        size_t k = 0;
        for (; k < m; ++k) {
            const uint8_t c = s[i + k];
            if ((c >= 'A' && c <= 'Z' ? (uint8_t)(c + 32) : c) != (uint8_t)cue[k]) break;
        }
        if (k == m) return true;
    }
    return false;
}

// v3_gov_arm_system (runtime/vault3.c:2970-3013): only a prompt that states a prohibition arms the governor; it
// then forbids syscall_exec when named, and every quoted literal ('...', "...", `...`) of 5..31 bytes that holds
// '_' or '(' -- with a trailing '(' also without it, and without its underscores.
extern "C" void v3g_gov_arm_system(v3g_gov_rules_t *g, const uint8_t *text, size_t len) {
    if (!g) return;
    v3g_gov_init(g);
    if (!text || len == 0) return;
    static const char *const cues[] = {"never", "forbid", "prohibit", "must not", "do not output", "do not emit"};
    bool prohibits = false;
    for (const char *c : cues) prohibits = prohibits || contains_ci(text, len, c);
    if (!prohibits) return;
    if (contains_ci(text, len, "syscall_exec")) {
        v3g_gov_add_rule(g, reinterpret_cast<const uint8_t *>("syscall_exec"), 12);
        v3g_gov_add_rule(g, reinterpret_cast<const uint8_t *>("syscallexec"), 11);
    }
    for (size_t i = 0; i < len; ++i) {
        const uint8_t q = text[i];
        if (q != '\'' && q != '"' && q != '`') continue;
        size_t j = i + 1;
        bool marked = false;
        while (j < len && text[j] != q && j - i - 1 < V3G_GOV_RULE_CAP) {
            marked = marked || text[j] == '_' || text[j] == '(';
            ++j;
        }
        const size_t n = j - i - 1;
        if (!(j < len && text[j] == q && marked && n >= 5 && n < V3G_GOV_RULE_CAP)) continue;
        const uint8_t *lit = text + i + 1;
        v3g_gov_add_rule(g, lit, n);
        const bool call = lit[n - 1] == '(';
        if (call && n >= 6) v3g_gov_add_rule(g, lit, n - 1);
        uint8_t bare[V3G_GOV_RULE_CAP];
        size_t bn = 0;
        for (size_t k = 0; k < (call ? n - 1 : n); ++k)
            if (lit[k] != '_') bare[bn++] = lit[k];
        if (bn >= 5) v3g_gov_add_rule(g, bare, bn);
        i = j;
    }
}

extern "C" int v3g_govern_logits(const v3g_model *m, const v3g_gov_rules_t *rules, const v3g_gov_stream_t *dev_streams,
                                 float *dev_logits, uint32_t rows, uint64_t ld, uint32_t top_k_guard, void *stream) {
    if (!m || !rules || !dev_streams || !dev_logits) return v3g_fail(V3G_E_ARG, "v3g_govern_logits: null pointer");
    if (ld < (uint64_t)m->host.vocab) return v3g_fail(V3G_E_ARG, "v3g_govern_logits: ld below the vocabulary");
    const cudaError_t e = launch_govern(m, *rules, dev_streams, dev_logits, rows, ld, top_k_guard, (cudaStream_t)stream);
    return e == cudaSuccess ? V3G_OK : v3g_fail(V3G_E_CUDA, cudaGetErrorString(e));
}

extern "C" int v3g_gov_commit(const v3g_model *m, const v3g_gov_rules_t *rules, v3g_gov_stream_t *dev_streams,
                              const int32_t *dev_tokens, uint32_t rows, void *stream) {
    if (!m || !rules || !dev_streams || !dev_tokens) return v3g_fail(V3G_E_ARG, "v3g_gov_commit: null pointer");
    const cudaError_t e = launch_gov_commit(m, *rules, dev_streams, dev_tokens, rows, (cudaStream_t)stream);
    return e == cudaSuccess ? V3G_OK : v3g_fail(V3G_E_CUDA, cudaGetErrorString(e));
}
