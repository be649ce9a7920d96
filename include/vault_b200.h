/* vault_b200.h -- C ABI of the B200 (sm_100a) VAULT v3 decode/prefill engine.
 *
 * Drop-in boundary for the reference's inference path.  Each entry point names the reference interface it
 * replaces (paths inside the batteryphil/VAULT checkout):
 *   - the freestanding C runtime API   runtime/vault3.h  (v3_load, v3_state_*, v3_step, v3_set_*, v3_argmax)
 *   - the Python streaming API          src/vault_v3_model.py  (VAULTv3ForCausalLM.new_state / prefill / step)
 *
 * Conventions (same as runtime/vault3.h):
 *   - integer status codes, 0 = success, negative = error (values -1..-12 keep the V3_E_* meanings);
 *   - the model file is a caller-owned host buffer (64-byte aligned), validated before anything is uploaded;
 *   - the inference state lives in a caller-owned DEVICE arena whose size is queried first; no entry point
 *     that advances the stream allocates memory;
 *   - every GPU operation is enqueued on the caller's cudaStream_t (passed as void*, NULL = legacy stream);
 *   - a state is not thread-safe; different states may be driven from different threads / streams.
 * No torch types cross this boundary: plain pointers, sizes and integers only.
 */
#ifndef VAULT_B200_H
#define VAULT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define V3G_API __attribute__((visibility("default")))
#else
#define V3G_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes: -1..-12 as runtime/vault3.h:35-49 */
enum {
    V3G_OK = 0,
    V3G_E_SIZE = -1,
    V3G_E_MAGIC = -2,
    V3G_E_CRC = -3,
    V3G_E_BOUNDS = -4,
    V3G_E_DTYPE = -5,
    V3G_E_MISSING = -6,
    V3G_E_SHAPE = -7,
    V3G_E_ARENA = -8,
    V3G_E_TOKENIZER = -9,
    V3G_E_LIMIT = -10,
    V3G_E_ALIGN = -11,
    V3G_E_NAN = -12,
    V3G_E_CUDA = -20,        /* a CUDA call failed (message in v3g_last_error) */
    V3G_E_ARG = -21,         /* invalid argument (null pointer, batch / budget out of range, ...) */
    V3G_E_UNSUPPORTED = -22, /* valid file or request this engine does not run (message says why) */
    V3G_E_DEVICE = -23       /* the device raised a status bit (see v3g_status) */
};

/* device status bits reported by v3g_status */
enum {
    V3G_STATUS_RESONANCE = 1, /* shingle-resonance bias would be active (src/vault_v3_model.py:1643-1716); not run */
    V3G_STATUS_BOUNDS = 2,    /* a token id or position left its valid range (clamped; the step's output is invalid) */
    V3G_STATUS_TIMEOUT = 4    /* a grid barrier of the persistent decode kernel gave up waiting (output invalid) */
};

/* v3g_state_init flags */
enum {
    V3G_STATE_PER_SEQ_MEMORY = 1, /* batch > 1: give every sequence its own auto-pin + segment memory (the reference
                                     runs those only at batch 1, src/vault_v3_model.py:1944,2222) */
    V3G_STATE_NO_AUTOPIN = 2,     /* keep n_pin = n_sink (runtime/vault3_host.c --no-autopin) */
    V3G_STATE_NO_GRAPHS = 4,      /* launch kernels directly instead of replaying captured CUDA graphs */
    V3G_STATE_NO_PERSISTENT = 8,  /* run a step as one GEMV kernel per layer phase (8 batch rows per pass) instead of
                                     the persistent kernel (batch <= 8) or the tensor-core GEMM step (batch > 8) */
    V3G_STATE_TOKEN_PREFILL = 16, /* v3g_prefill streams the prompt one decode step per token instead of the chunked
                                     tensor-core prefill */
    V3G_STATE_FP16_ACTIVATIONS = 32 /* decode GEMVs take each activation as one fp16 part (11 bits) instead of a high
                                       and a low part (about 22 bits) at batch <= 4: faster, less precise */
};

typedef struct v3g_model v3g_model;
typedef struct v3g_state v3g_state;

typedef struct {
    uint32_t vocab_size, d_model, n_layers, n_heads, n_kv_heads, head_dim, d_ff, window;
    float rms_eps, rope_theta;
    uint32_t bos_id, eos_id, im_start_id, im_end_id, pad_id, weight_format, flags, n_sink;
    uint32_t seg_budget, seg_hidden, seg_min, seg_max, seg_n_feat, seg_layers[4];
    uint32_t sink_cap;                /* sink rows per layer = max(1, n_sink, max_sink) */
    uint64_t step_weight_bytes;       /* file bytes of every weight read by one decode step, lm head included */
    uint64_t lm_head_bytes;           /* file bytes of the tied lm head */
    uint64_t scorer_bytes;            /* file bytes of the segment scorer (read when segment memory is on) */
    uint64_t device_bytes;            /* device memory held by the model */
} v3g_model_info;

/* CAAI output governor (runtime/vault3.h:191-216).  The rules are built on the host (v3g_gov_add_rule,
 * v3g_gov_arm_system) and passed by value to the device calls; the stream state (canonical history of the emitted
 * text, an unfinished UTF-8 sequence, the raw byte tail) is one v3g_gov_stream_t per sequence in device memory,
 * all zero at the start of a stream. */
#define V3G_GOV_MAX_RULES 8
#define V3G_GOV_RULE_CAP 32
#define V3G_GOV_HIST_CAP 64
#define V3G_GOV_RAW_CAP 96
typedef struct {
    uint32_t n_rules;                                   /* 0: the governor is off */
    uint32_t rule_len[V3G_GOV_MAX_RULES];
    uint8_t rules[V3G_GOV_MAX_RULES][V3G_GOV_RULE_CAP];  /* canonical patterns */
} v3g_gov_rules_t;
typedef struct {
    uint32_t hist_len, utf8_len, raw_len, reserved;
    uint8_t hist[V3G_GOV_HIST_CAP];
    uint8_t utf8_rem[4];
    uint8_t raw_tail[V3G_GOV_RAW_CAP];
    uint8_t pad[12];
} v3g_gov_stream_t;

/* Parse + validate a VLT3 buffer (same rules as v3_load, runtime/vault3.c:273-455; runtime/vault3.h:89) and
 * upload it to `device`, re-tiled for the decode kernels.  verify_crc = 1 also checks every tensor CRC32.
 * max_sink: cap of the ChatML auto-pinned prefix (the Python reference's VAULTv3Config.max_sink, default 512;
 * 0 selects 512).  The loader allocates the model's device memory itself (freed by v3g_free). */
V3G_API int v3g_load(v3g_model **out, const uint8_t *buf, uint64_t size, int verify_crc, int device, uint32_t max_sink);
/* Validate a VLT3 buffer on the host only (no device call): the checks and status codes v3g_load applies before it
 * uploads anything.  The Python reader (vault_b200.vlt3.read_vlt3, the counterpart of tools/vlt3.py:453-545
 * read_vlt3) validates through it, so both loaders accept and reject the same files. */
V3G_API int v3g_validate(const uint8_t *buf, uint64_t size, int verify_crc);
/* The same two calls on a file path: the file is mapped read-only (mmap, page-aligned) for the length of the call
 * and read in place, with no host copy (runtime/vault3_host.c maps its model file the same way).  A missing or
 * unmappable file gives V3G_E_ARG, an empty one V3G_E_SIZE; otherwise the codes of v3g_load / v3g_validate. */
V3G_API int v3g_load_file(v3g_model **out, const char *path, int verify_crc, int device, uint32_t max_sink);
V3G_API int v3g_validate_file(const char *path, int verify_crc);
V3G_API int v3g_model_get_info(const v3g_model *m, v3g_model_info *out);
V3G_API void v3g_free(v3g_model *m);

/* Device-arena size for `batch` sequences with a segment bank of up to max_seg_budget rows each
 * (runtime/vault3.h:153 v3_state_arena_size_ex).  Returns 0 on invalid arguments. */
V3G_API size_t v3g_state_arena_size(const v3g_model *m, uint32_t batch, uint32_t max_seg_budget);
/* Bind a state to a caller-owned device arena (256-byte aligned) and reset it (runtime/vault3.h:155
 * v3_state_init_ex).  batch > 1 without V3G_STATE_PER_SEQ_MEMORY follows the reference's batched step: no
 * auto-pin, no segment memory, n_pin = n_sink (src/vault_v3_model.py:2177-2220). */
V3G_API int v3g_state_init(v3g_state **out, const v3g_model *m, void *dev_arena, size_t arena_size, uint32_t batch,
                   uint32_t max_seg_budget, uint32_t flags);
V3G_API void v3g_state_free(v3g_state *s);
V3G_API int v3g_state_reset(v3g_state *s, void *stream);                           /* runtime/vault3.h:157 */
V3G_API int v3g_set_pinned(v3g_state *s, uint32_t n_pin, void *stream);            /* runtime/vault3.h:158 */
V3G_API int v3g_set_seg_budget(v3g_state *s, uint32_t budget, void *stream);       /* runtime/vault3.h:159 */
V3G_API uint64_t v3g_state_pos(const v3g_state *s);                                /* VAULTv3State.pos */

/* Feed one token per sequence (device int32 [batch]); optionally write fp32 logits [batch, vocab] and the greedy
 * (first-max) next token [batch] to device memory.  Replaces v3_step (runtime/vault3.h:161) and
 * VAULTv3ForCausalLM.step (src/vault_v3_model.py:2214).  Ids outside [0, vocab) are replaced by pad_id. */
V3G_API int v3g_step(v3g_state *s, const int32_t *dev_tokens, float *dev_logits, int32_t *dev_next, void *stream);
/* Same with HOST buffers (uint32 tokens in, fp32 logits / uint32 next token out; either output may be NULL):
 * copies in, steps, copies out and synchronizes `stream`.  The v3_step calling convention for C callers. */
V3G_API int v3g_step_host(v3g_state *s, const uint32_t *tokens, float *logits, uint32_t *next, void *stream);
/* Stream n_tokens ids per sequence (device int32, row b at dev_ids + b * ld) through the state, computing the
 * lm head only for the last one (src/vault_v3_model.py:2163 prefill; the chunk-recurrent forward :1938-2116).
 * The prompt runs in window-aligned pieces (each layer's projections as tensor-core GEMMs over all of a piece's
 * tokens, one block-window attention launch, the segment scorer over every token of the piece) unless
 * V3G_STATE_TOKEN_PREFILL is set or a weight matrix is stored as F32 (those models stream token by token). */
V3G_API int v3g_prefill(v3g_state *s, const int32_t *dev_ids, uint32_t n_tokens, uint64_t ld, float *dev_logits,
                int32_t *dev_next, void *stream);
/* Greedy decode on the device: feeds dev_first [batch], then each step's argmax, for n_steps steps, writing the
 * produced tokens to dev_out (row b at dev_out + b * ld).  No host round trip between steps. */
V3G_API int v3g_generate(v3g_state *s, const int32_t *dev_first, uint32_t n_steps, int32_t *dev_out, uint64_t ld,
                 void *stream);
/* Sampled decode on the device, the generation loop of runtime/vault3_host.c:586-606 with --temp / --topk: feeds
 * dev_first [batch], then for n_steps steps draws each sequence's next token from that step's logits with the
 * v3g_sample_topk rule (k capped at 64; temp <= 0 or k <= 1 is greedy), writing the tokens to dev_out (row b at
 * dev_out + b * ld) and advancing the per-sequence xorshift states dev_rng [batch].  With gov (rules, n_rules > 0)
 * and dev_gov (stream states [batch]) each step's logits are first masked by v3g_govern_logits with the loop's
 * guard (16 when temp <= 0 or k < 16, else min(k, 64)) and each drawn token is committed by v3g_gov_commit.  No
 * host round trip between steps; all n_steps run (the loop's stop at <|im_end|> / BOS is the caller's).  The
 * loop's repetition penalty is not applied. */
V3G_API int v3g_generate_sampled(v3g_state *s, const int32_t *dev_first, uint32_t n_steps, int32_t *dev_out,
                                 uint64_t ld, uint32_t k, float temp, uint64_t *dev_rng, const v3g_gov_rules_t *gov,
                                 v3g_gov_stream_t *dev_gov, void *stream);
/* Synchronize `stream` and read the sticky device status bits (V3G_STATUS_*); clears them when clear != 0. */
V3G_API int v3g_status(v3g_state *s, uint32_t *bits, int clear, void *stream);
/* Asynchronous form of v3g_status for callers that poll between steps: enqueues on `stream` a copy of the sticky
 * status bits into dst (device memory or pinned host memory, 4 bytes) and returns without synchronizing; the value
 * is valid once the stream has passed the copy. */
V3G_API int v3g_status_copy(v3g_state *s, uint32_t *dst, void *stream);

/* Snapshot of one sequence's streaming bookkeeping (VAULTv3State fields, src/vault_v3_model.py:974-1011);
 * mem_pos / mem_score receive up to `cap` bank entries in chronological order.  Synchronizes `stream`. */
typedef struct {
    int32_t n_pin, pin_locked, mem_cnt, n_uniq_segs, seg_id_offset, ema_ready, seg_budget;
    uint64_t pos;
} v3g_seq_info_t;
V3G_API int v3g_seq_info(v3g_state *s, uint32_t b, v3g_seq_info_t *info, int64_t *mem_pos, float *mem_score, uint32_t cap,
                 void *stream);

/* Kernel-level entry points (tests and the kernel sweep).  tensor_id uses the VLT3 ids of tools/vlt3.py:34-57. */
V3G_API int v3g_dequant(const v3g_model *m, uint32_t tensor_id, float *dev_out, void *stream);
V3G_API int v3g_gemv(const v3g_model *m, uint32_t tensor_id, const float *dev_x, uint32_t batch, float *dev_y, void *stream);
/* Tensor-core GEMM of one stored weight matrix against n_tok fp32 activation rows: dev_y[t, r] = sum_k W[r, k]
 * dev_x[t, k] (row t of dev_x has the matrix's K entries; dev_y rows have the matrix's row count, gate/up as
 * [gate; up]).  The kernel the chunked prefill and the batched decode step run for every projection: weights
 * dequantized to fp16 in shared memory, tcgen05 MMA into tensor memory.  It is the many-token form of the
 * reference's row_dot / matvec (runtime/vault3.c:499-624) and nn.Linear (src/vault_v3_model.py:1036-1039).
 * dev_work: caller-owned device workspace (256-byte aligned) of v3g_gemm_work_size bytes. */
V3G_API size_t v3g_gemm_work_size(const v3g_model *m, uint32_t tensor_id, uint32_t n_tok);
V3G_API int v3g_gemm(const v3g_model *m, uint32_t tensor_id, const float *dev_x, uint32_t n_tok, float *dev_y,
                     void *dev_work, size_t work_bytes, void *stream);
/* One launch of the decode attention of `layer` (the kernel the state's step uses) for every sequence at the state's
 * current position (the
 * keys of src/vault_v3_model.py:1072-1139 / runtime/vault3.c:1967-2032: sinks, bank, previous and current chunk),
 * reading the queries the last step left in the state: for timing the kernel alone (kernel sweep). */
V3G_API int v3g_attention(v3g_state *s, uint32_t layer, void *stream);
/* One launch of the persistent decode kernel (every layer of the current position, plus the lm head when want_lm)
 * on a state whose steps use it, without the step's token bookkeeping: for timing the kernel alone.  It rewrites
 * the current position's activations and KV rows, so reset the state before decoding again. */
V3G_API int v3g_decode_pass(v3g_state *s, int want_lm, void *stream);

/* Greedy (first-maximum) token of each of `rows` logit rows (row b at dev_logits + b * ld, `vocab` entries, NaN
 * never selected, -0.0 equal to +0.0, token 0 for a row that is all NaN), written to dev_tokens[rows] -- the selection v3g_step makes, for callers that hold logits but
 * may not allocate device memory (their framework's allocator owns the device memory, or cudaMalloc's implicit
 * device synchronisation is not acceptable in their token loop).  It has no counterpart in the reference.
 * Allocates nothing: its scratch is a fixed device array of V3G_NOALLOC_MAX_ROWS 8-byte keys that every GPU loading
 * the library holds until exit; more rows fail with V3G_E_LIMIT.  It runs on the current device; its first call
 * on a device looks up the array's device address, so make that first call before any stream capture.  All calls
 * share the array (cleared at the start of each call): calls that overlap on the GPU race. */
/* Top-k (k <= 64) + temperature sampling of `rows` logit rows (row b at dev_logits + b * ld, `vocab` entries) with
 * a caller-held xorshift64 state per row (dev_rng[rows], updated in place): v3_sample_topk (runtime/vault3.h:221,
 * runtime/vault3.c:3204-3230) on the device, same candidate order (value, then lower index), the reference's own
 * exponential and the same draw.  temp <= 0 or k <= 1 gives the greedy token and leaves dev_rng untouched (it may
 * then be NULL).  NaN logits are never candidates; a row without a finite logit gives token 0.  Tokens go to
 * dev_tokens[rows]. */
V3G_API int v3g_sample_topk(const float *dev_logits, uint32_t rows, uint32_t vocab, uint64_t ld, uint32_t k, float temp,
                            uint64_t *dev_rng, int32_t *dev_tokens, void *stream);

/* Governor rules (host only, no device call).  v3g_gov_init: no rules (v3_gov_init).  v3g_gov_add_rule: canonicalize
 * pat and add it unless present (v3_gov_add_rule, runtime/vault3.c:2933-2957): V3G_E_SIZE when the canonical form is
 * shorter than 4 bytes, V3G_E_LIMIT when 8 rules are held.  v3g_gov_arm_system: reset, then derive the rules from a
 * system prompt that states a prohibition (v3_gov_arm_system, runtime/vault3.c:2970-3013). */
V3G_API void v3g_gov_init(v3g_gov_rules_t *g);
V3G_API int v3g_gov_add_rule(v3g_gov_rules_t *g, const uint8_t *pat, size_t len);
V3G_API void v3g_gov_arm_system(v3g_gov_rules_t *g, const uint8_t *sys_text, size_t len);
/* Mask, in place, every candidate token whose bytes would complete a rule (forward, reversed, or inside a base64 /
 * hex tail) after that row's stream: v3_govern_logits (runtime/vault3.c:3133-3181) per row, up to 4 passes over the
 * top-k (k = top_k_guard, 0 or > 64 -> 64) logits above -3e38, a masked logit becoming -3.4e38.  Rows at
 * dev_logits + b * ld with the model's vocabulary; dev_streams[rows].  Logits are taken to be NaN-free. */
V3G_API int v3g_govern_logits(const v3g_model *m, const v3g_gov_rules_t *rules, const v3g_gov_stream_t *dev_streams,
                              float *dev_logits, uint32_t rows, uint64_t ld, uint32_t top_k_guard, void *stream);
/* Append each row's chosen token to its stream (v3_gov_commit, runtime/vault3.c:3183-3194): EOS, <|im_start|> and
 * <|im_end|> reset the stream; nothing happens while rules->n_rules == 0. */
V3G_API int v3g_gov_commit(const v3g_model *m, const v3g_gov_rules_t *rules, v3g_gov_stream_t *dev_streams,
                           const int32_t *dev_tokens, uint32_t rows, void *stream);

/* Host tokenizer of a VLT3 file's VTOK blob (runtime/vault3.h:162-188 v3_tok_init / v3_encode_ex / v3_encode;
 * v3_token_bytes :189): byte-level BPE behind the Qwen2 pre-tokenizer, UAX #15 NFC on spans holding bytes >= 0xCC,
 * special tokens (<|im_start|> ...) matched as whole strings when allow_special != 0.  Same ids as the reference for
 * the same text; V3G_E_SIZE with the first max_out ids in out when more would follow.  v3g_tokenizer_create
 * validates buf as v3g_validate does (without the CRC pass; buf 64-byte aligned as for v3g_load) and keeps its own
 * copy of the blob.  Host only. */
typedef struct v3g_tokenizer v3g_tokenizer;
V3G_API int v3g_tokenizer_create(v3g_tokenizer **out, const uint8_t *buf, uint64_t size);
V3G_API void v3g_tokenizer_free(v3g_tokenizer *t);
V3G_API int v3g_encode_ex(v3g_tokenizer *t, const uint8_t *text, size_t len, uint32_t *out, size_t max_out,
                          size_t *n_out, int allow_special);
V3G_API int v3g_encode(v3g_tokenizer *t, const uint8_t *text, size_t len, uint32_t *out, size_t max_out, size_t *n_out);
V3G_API int v3g_token_bytes(const v3g_tokenizer *t, uint32_t id, const uint8_t **bytes, uint32_t *len);

#define V3G_NOALLOC_MAX_ROWS 4096
V3G_API int v3g_argmax_noalloc(const float *dev_logits, uint32_t rows, uint32_t vocab, uint64_t ld, int32_t *dev_tokens,
                               void *stream);

V3G_API const char *v3g_error_string(int code);
V3G_API const char *v3g_last_error(void);   /* detail of the last failure on this thread */

#ifdef __cplusplus
}
#endif
#endif /* VAULT_B200_H */
