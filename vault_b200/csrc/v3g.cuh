// Internal definitions shared by the VAULT v3 B200 engine translation units.
//
// Device data layouts
// -------------------
// Weight matrices are re-tiled once at load time ("repack") into 16-row tiles whose bytes are already in
// mma.sync m16n8k16 A-fragment order (weights are the A operand, activations of up to 8 sequences the B
// operand), so a decode GEMV streams each tile with one 16-byte load per lane and feeds the tensor core without
// shared-memory staging:
//   Q8_0 : 16 rows x 32 k (one block)  = 512 B codes + 32 B fp16 scales   (544 B, 34/32 B per weight as in the file)
//   Q4_0 : 16 rows x 64 k (two blocks) = 512 B nibbles + 64 B fp16 scales (576 B, 18/32 B per weight as in the file)
//   BF16 / F16 : 16 rows x 16 k = 512 B of fp16 (BF16 weights are stored as fp16 times a per-matrix power of two
//                2^s chosen so that max|w| 2^s lies in [2^14, 2^15): exact for every |w| >= max|w| 2^-32)
//   F32  : 16 rows x 16 k, three fp16 planes hi/mid/lo with w 2^s = hi + 2^-11 mid + 2^-22 lo exactly (1536 B)
// Lane L = 4g + t of a warp owns tile rows g and g+8 and, for every 16-wide k step s of the tile, the k offsets
// 16s + {2t, 2t+1, 2t+8, 2t+9}.  Q8_0 codes are stored biased (q + 128) so one byte-permute turns two of them into
// the fp16 integers 1152 + q; Q4_0 nibbles n become 1024 + n with one mask; the constant offsets are removed after
// the tensor core with the activation block sums.  The tensor-core result hands lane (g,t) the outputs of tile
// rows g and g+8 for batch rows 2t and 2t+1.  Fused QKV tiles place RoPE partners (i, i + D/2) at tile rows
// (r, r+8) and gate/up tiles place gate_f and up_f there, so each lane holds both operands of its RoPE rotation /
// SiLU product in registers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace v3g {

enum WFmt : int { FMT_F32 = 0, FMT_F16 = 1, FMT_BF16 = 2, FMT_Q8 = 8, FMT_Q4 = 9 };

constexpr int TILE_ROWS = 16;
__host__ __device__ constexpr int tile_k(int fmt) { return fmt == FMT_Q8 ? 32 : (fmt == FMT_Q4 ? 64 : 16); }
__host__ __device__ constexpr int tile_bytes(int fmt) {
    return fmt == FMT_Q8 ? 544 : (fmt == FMT_Q4 ? 576 : (fmt == FMT_F32 ? 1536 : 512));
}
// every tile format enters the tensor core as fp16 (kind f16 with fp32 accumulation); activations are fp16 too
constexpr float F32_MID = 1.0f / 2048.0f, F32_LO = 1.0f / 4194304.0f;   // 2^-11, 2^-22 plane weights

// KV cache element: fp16 (10 mantissa bits; K/V magnitudes stay far inside its range)
typedef __half kv_t;

enum RowMap : int { ROWS_IDENTITY = 0, ROWS_ROPE_PAIRS = 1, ROWS_GATE_UP = 2 };

struct MatW {
    const uint8_t *tiles = nullptr;  // [n_rtiles][n_ktiles][tile_bytes]
    int fmt = 0;
    int rows = 0;                    // logical output rows (gate/up: 2 * d_ff)
    int cols = 0;                    // K
    int n_rtiles = 0, n_ktiles = 0;
    int rowmap = ROWS_IDENTITY;
    uint64_t file_bytes = 0;         // payload bytes of the source tensor(s) in the VLT3 file
    float wscale = 1.f;              // tile values x wscale = weights (2^-s for BF16 / F32 tiles, else 1)
    int dexp = 0;                    // Q8_0 / Q4_0: the tensor-core GEMM dequantizes to fp16 q d 2^dexp (no subnormals)
};

constexpr int MAX_LAYERS = 64;
constexpr int MAX_SEG_FEAT = 4;
constexpr int MAX_SINK = 512;
constexpr int MAX_SEG_BUDGET = 16384;
constexpr int GEMV_MB = 8;             // batch rows per GEMV pass (mma rows 0..7)
constexpr int GEMV_THREADS = 256;
constexpr int ATT_KEYS_PER_CTA = 64;   // split-KV chunk
constexpr int ATT_MERGE_MAX = 4;        // persistent kernel: up to this many splits are merged by their reader
__host__ __device__ constexpr int att_part_stride(int D) { return D + 4; }   // partial row: o[D], m, l, 2 pad
constexpr int ATT_THREADS = 128;
constexpr int GEMV_MAX_SMEM = 220 * 1024;   // launch-time cap (below the 227 KB opt-in minus static smem)

struct LayerW {
    MatW q, k, v, o, gu, down;
    const float *ln1, *ln2, *bq, *bk, *bv;
};

struct ModelDev {
    int vocab, d, n_layers, H, G, D, F, W;
    float rms_eps, rope_theta;
    int pad_id, im_start_id, im_end_id, newline_id, system_id, n_sink, sink_cap, max_sink;
    int seg_n_feat, seg_hidden, seg_min, seg_max, seg_budget_default;
    int seg_layers[MAX_SEG_FEAT];
    LayerW layers[MAX_LAYERS];
    MatW embed;                      // tied embedding / lm head
    const float *norm;
    // segment scorer (F32, row-major as in the file)
    const float *sc_ln_w, *sc_ln_b, *sc_w1, *sc_b1, *sc_w2, *sc_b2;
    // RoPE table: rows for positions [rope_pos0, rope_pos0 + rope_rows), each D/2 cos then D/2 sin (fp32)
    const float *rope;
    int rope_pos0, rope_rows;
    // token tables
    const uint8_t *tier;             // [vocab] segment-break tier 0..3
    const uint32_t *tok_off;         // [vocab] byte offset in tok_pool (0xFFFFFFFF = no bytes)
    const uint16_t *tok_len;         // [vocab]
    const uint8_t *tok_pool;
};

// Per-sequence control block (device resident; mirrors the scalar fields of src/vault_v3_model.py:974-1011)
struct SeqCtl {
    int32_t n_pin, pin_locked, saw_im_start, awaiting_sys_nl;
    int32_t ema_ready, mem_cnt, n_uniq_segs, seg_id_offset;
    int32_t cur_seg_id, seg_len, bank_par, seg_budget;
    int32_t seg_on, auto_pin, last_im_end, pad0;
};

// Step-level control (device resident, shared by the batch: the reference keeps one st.pos per batch)
struct StepCtl {
    int64_t pos;             // absolute token count before the current step
    const int32_t *ids;      // token source for prefill (nullptr: tok_in)
    int64_t ids_ld;          // row stride of ids
    int64_t ids_idx;         // next column of ids
    int32_t *out_tokens;     // greedy token sink (nullptr: none)
    int64_t out_ld, out_idx;
    int32_t status;          // sticky error bits (STATUS_*)
    int32_t want_logits;
};

enum : int32_t {
    STATUS_RESONANCE = 1,    // shingle-resonance bias would be active: unsupported, results diverge from reference
    STATUS_BOUNDS = 2,       // an internal index check failed
    STATUS_TIMEOUT = 4,      // a bounded grid-barrier wait gave up (results of the step are invalid)
};

struct StateDev {
    int B, W, G, D, H, sink_cap, seg_cap, feat_dim, max_splits;
    uint64_t lb_stride;          // bytes of one (layer, sequence) KV block
    uint8_t *kv;                 // [layer][seq] KV blocks
    // offsets inside a KV block (bytes)
    uint64_t off_ring, ring_kind_stride, ring_par_stride;   // ring[par][kind k_rot/kraw/v][G][W][D]
    uint64_t off_sink;                                      // sink[kind k_raw/k_rot/v][G][S][D]
    uint64_t off_bank, bank_par_stride, off_bank_rot;       // bank[par][kind k_raw/v][G][Bc][D]; rot[G][Bc][D]
    SeqCtl *seq;                 // [B]
    StepCtl *step;
    int32_t *tok_in;             // [B]
    int32_t *tok_ring;           // [B][2][W]
    float *sc_ring;              // [B][2][W]
    int32_t *seg_ring;           // [B][2][W]
    int64_t *mem_pos;            // [B][2][seg_cap]
    float *mem_score;            // [B][2][seg_cap]
    int32_t *mem_tok, *mem_seg;  // [B][2][seg_cap]
    int32_t *mem_src;            // [B][seg_cap]  gather source: >=0 old bank slot, <0: -(t+1) prev-chunk row
    float *ema, *feat;           // [B][feat_dim]
    float *x;                    // [B][d] residual stream
    float *attn;                 // [B][H*D]
    float *hbuf;                 // [B][F]
    float *q_cur, *q_far;        // [B][H][D]
    float *att_part;             // [B][G][max_splits][grp][att_part_stride(D)]
    uint32_t *att_cnt;           // [B][G]
    float *logits;               // [B][V]
    unsigned long long *amax;    // [B]
    float *sc_z;                 // [B][2][seg_hidden]
    unsigned int *bar;           // grid-barrier counter of the persistent decode kernel (zeroed every step)
};

// Optional timeline of the persistent decode kernel (compile with -DV3G_MK_TRACE): per phase and CTA, %globaltimer
// at the phase start (0), after the activation prologue (1), after the phase's work (2), after the grid barrier (3),
// the producer's first copy of the phase (4), and inside the prologue after the loads (5) and the block barrier (6).
// Read back with v3g_mk_trace_read (the copy of v3g_step.cu, where the kernel lives).
#ifdef V3G_MK_TRACE
constexpr int MK_TRACE_PH = 512, MK_TRACE_CTA = 160, MK_TRACE_EV = 8;
static __device__ unsigned long long g_mk_trace[MK_TRACE_PH][MK_TRACE_CTA][MK_TRACE_EV];   // per translation unit
__device__ __forceinline__ unsigned long long mk_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
#define MK_TRACE(p, ev)                                                                                \
    do {                                                                                               \
        if ((p) >= 0 && (p) < MK_TRACE_PH && blockIdx.x < MK_TRACE_CTA) g_mk_trace[p][blockIdx.x][ev] = mk_now(); \
    } while (0)
#else
#define MK_TRACE(p, ev) \
    do {                \
    } while (0)
#endif

constexpr int KIND_KROT = 0, KIND_KRAW = 1, KIND_V = 2;   // ring kinds
constexpr int SINK_KRAW = 0, SINK_KROT = 1, SINK_V = 2;   // sink kinds
constexpr int BANK_KRAW = 0, BANK_V = 1;                  // bank kinds

__device__ __forceinline__ uint64_t ring_off(const StateDev &s, int par, int kind, int g, int t) {
    return s.off_ring + (uint64_t)par * s.ring_par_stride + (uint64_t)kind * s.ring_kind_stride +
           ((uint64_t)g * s.W + t) * s.D * 2ull;
}
__device__ __forceinline__ uint64_t sink_off(const StateDev &s, int kind, int g, int j) {
    return s.off_sink + (((uint64_t)kind * s.G + g) * s.sink_cap + j) * s.D * 2ull;
}
__device__ __forceinline__ uint64_t bank_off(const StateDev &s, int par, int kind, int g, int j) {
    return s.off_bank + (uint64_t)par * s.bank_par_stride + (((uint64_t)kind * s.G + g) * s.seg_cap + j) * s.D * 2ull;
}
__device__ __forceinline__ uint64_t bank_rot_off(const StateDev &s, int g, int j) {
    return s.off_bank_rot + ((uint64_t)g * s.seg_cap + j) * s.D * 2ull;
}
__device__ __forceinline__ kv_t *kvp(const StateDev &s, int layer, int b, uint64_t off) {
    return reinterpret_cast<kv_t *>(s.kv + ((uint64_t)layer * s.B + b) * s.lb_stride + off);
}

__device__ __forceinline__ const float *rope_row(const ModelDev &m, int64_t pos) {
    return m.rope + (pos - m.rope_pos0) * (int64_t)m.D;
}

// ------------------------------------------------------------------------------------------ small device helpers
__device__ __forceinline__ uint4 ldg_stream16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldg_stream8(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

// barrier over the first n threads of the CTA (named barrier 1, n a multiple of 32): kernels whose every thread
// takes part pass blockDim.x, the persistent decode kernel passes its consumer warps only
__device__ __forceinline__ void sync_threads(int n) { asm volatile("bar.sync 1, %0;" ::"r"(n) : "memory"); }

// D (16 x 8, fp32) += A (16 x 16, fp16, row) * B (16 x 8, fp16, col): one warp-wide tensor-core step
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// order-preserving float -> uint32 (larger float -> larger key); -0.0 maps to the key of +0.0, so the two compare
// equal and the first-index tie rule of v3_argmax (runtime/vault3.c:3198-3202) holds for them too.  NaN-free
// inputs assumed (callers skip NaN).
__device__ __forceinline__ uint32_t float_key(float f) {
    uint32_t u = __float_as_uint(f);
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float kv2f(kv_t v) { return __half2float(v); }
__device__ __forceinline__ kv_t f2kv(float v) { return __float2half_rn(v); }

// Programmatic dependent launch: every kernel of a decode step is launched with programmatic stream serialization,
// so it may start while its predecessor drains.  Before griddep_wait() a kernel touches only immutable data
// (weights); griddep_wait() returns once the predecessor grid has completed and its writes are visible.
// Launched without the attribute, both are no-ops.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// host: launch `k` with the programmatic-serialization attribute (pdl = true) on stream st
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(bool pdl, void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

// element (tile row r, k) of a re-tiled matrix as fp32 (exact inverse of the repack); wscale = MatW::wscale
__device__ __forceinline__ float tile_value(const uint8_t *tiles, int fmt, int n_ktiles, float wscale, int p, int k) {
    const int TK = tile_k(fmt);
    const int rt = p / TILE_ROWS, r = p % TILE_ROWS, kt = k / TK, kk = k % TK;
    const int g = r & 7, s = kk >> 4, w16 = kk & 15;
    const int t = (w16 & 7) >> 1, half = w16 & 1;
    const int reg = ((r >> 3) & 1) | ((w16 & 8) ? 2 : 0);
    const int lane = 4 * g + t, e = 2 * reg + half;
    const uint8_t *tb = tiles + ((size_t)rt * n_ktiles + kt) * tile_bytes(fmt);
    if (fmt == FMT_Q8 || fmt == FMT_Q4) {
        const int blk = kk >> 5;
        const uint32_t sw = fmt == FMT_Q8 ? *reinterpret_cast<const uint32_t *>(tb + 512 + g * 4)
                                          : *reinterpret_cast<const uint32_t *>(tb + 512 + g * 8 + 4 * blk);
        const float d = __half2float(__ushort_as_half((uint16_t)(r < 8 ? (sw & 0xFFFF) : (sw >> 16))));
        if (fmt == FMT_Q8) return (float)((int)tb[lane * 16 + 8 * s + e] - 128) * d;
        const uint32_t word = *reinterpret_cast<const uint32_t *>(tb + lane * 16 + 4 * s);
        return (float)((int)((word >> (4 * reg + 16 * half)) & 15u) - 8) * d;
    }
    const int off = lane * 16 + 2 * e;
    const float hi = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t *>(tb + off)));
    if (fmt != FMT_F32) return hi * wscale;
    const float mid = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t *>(tb + 512 + off)));
    const float lo = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t *>(tb + 1024 + off)));
    return ((hi + mid * F32_MID) + lo * F32_LO) * wscale;
}

// logical (tile-order) row p of a re-tiled matrix -> (source matrix, source row); false for padding rows
__host__ __device__ __forceinline__ bool map_tile_row(int rowmap, int head_dim, int src_rows, int p, int &src,
                                                      int &row) {
    src = 0;
    if (rowmap == ROWS_ROPE_PAIRS) {   // tile j of a head: rows 8j..8j+7 then their partners 8j+D/2..
        const int D = head_dim, head = p / D, w = p % D, j = w >> 4, r = w & 15;
        row = head * D + 8 * j + (r & 7) + ((r & 8) ? D / 2 : 0);
    } else if (rowmap == ROWS_GATE_UP) {   // tile rt: gate rows 8rt..8rt+7 then up rows 8rt..8rt+7
        src = (p >> 3) & 1;
        row = (p >> 4) * 8 + (p & 7);
    } else {
        row = p;
    }
    return row < src_rows;
}

// ChatML system-prompt auto-pin state machine for one token (src/vault_v3_model.py:2224-2252)
__device__ inline void auto_pin_update(const ModelDev &m, SeqCtl &q, int64_t pos, int tid) {
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


}  // namespace v3g
