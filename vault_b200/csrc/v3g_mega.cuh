// Persistent decode kernel: every layer of one decode step (and the lm head) in ONE cooperative launch, one CTA
// per SM (8 consumer warps + 1 producer warp), phases separated by bounded grid barriers.
//
// Phase list (host-built, per state): for every layer [QKV GEMV, attention, O GEMV, gate/up GEMV, down GEMV], then
// the lm-head GEMV.  A GEMV phase is a flat sequence of T weight tiles (segment by segment, row tile by row tile,
// k tile by k tile -- exactly the order of the tile buffers in HBM).  CTA c owns the whole row tiles
// [c NR / G, (c+1) NR / G) and its 8 consumer warps cut the CTA's contiguous tile range into equal pieces, so
// every warp streams one contiguous byte range per phase and no row tile is ever split between SMs.
//
// Weight bytes reach shared memory through bulk asynchronous copies (cp.async.bulk, completion on an mbarrier) into
// a ring of `slots` chunk buffers per consumer warp.  The producer warp issues every copy (lane i feeds consumer
// warp i; a full / empty mbarrier pair per slot), so consumers only wait, compute and release; because weights
// never change the producer runs ahead ACROSS phase boundaries -- while the consumers wait at a grid barrier, run a
// prologue or attention, the copies for the coming GEMV phases keep HBM busy.  The chunk streams are walked from a
// compact per-phase table held in shared memory, so no bookkeeping touches global memory.
//
// The kernel is compiled per pair of tile formats (FA, FB): every segment of every GEMV phase uses one of the two
// (all Q8_0; Hybrid-Q4_0 = Q4_0 + Q8_0; all BF16; all F16; all F32), so the inner loops carry no format switch.
//
// Row tiles that one warp covers completely go straight to the fused epilogue.  A row tile split between warps of
// the CTA is finished at the end of the phase: every warp leaves its partial in shared memory and the warp where
// the row tile starts sums the pieces in warp order (deterministic) and runs the epilogue.
//
// Attention phases spread the (sequence, KV head, key chunk) work items over the CTAs (v3g_attn.cuh).
// This header is included at the end of v3g_step.cu, after the epilogue functors it instantiates.
#pragma once
#include "v3g_attn.cuh"
#include "v3g_gemv.cuh"

namespace v3g {

enum : int { MK_GEMV = 0, MK_ATTN = 1 };
enum : int { MK_EPI_QKV = 0, MK_EPI_RESID = 1, MK_EPI_GATEUP = 2, MK_EPI_STORE = 3 };
constexpr int MK_WARPS = GEMV_THREADS / 32;            // consumer warps
constexpr int MK_CT = MK_WARPS * 32;                    // consumer threads (named-barrier count)
constexpr int MK_THREADS = MK_CT + 32;                  // + the producer warp
constexpr int MK_MAX_SLOTS = 16;
constexpr int MK_CHUNK = 8;                             // tiles per chunk (F32: 3)
constexpr int MK_GROUP = 4;                             // tiles computed together (register budget)
constexpr int MK_SLOT_BYTES = MK_CHUNK * 576;           // 8 Q4_0 / Q8_0 / 16-bit tiles or 3 F32 tiles
constexpr uint32_t MK_WAIT_LIMIT = 1u << 22;
constexpr int MK_OWN_TILES = 4;                         // residual / bias row tiles a CTA keeps in shared memory

__host__ __device__ constexpr int mk_cap(int fmt) { return fmt == FMT_F32 ? MK_SLOT_BYTES / 1536 : MK_CHUNK; }

// full description of one phase (read by the CTA from a shared-memory copy while the phase runs)
struct alignas(16) MkPhase {
    GemvArgs a;
    int fmts[3];
    int kind, epi, layer;
    int tbase[4];         // flat tile index where segment s starts; tbase[n_seg] = T
    int rbase[3];         // flat row-tile index where segment s starts (ticket counters)
    const float *bq, *bk, *bv;
    float *out;
    int out_ld, out_rows;
    // norm weights of the NEXT phase (nullptr when it has no RMSNorm or they cannot be staged): this phase copies
    // them into shared memory while it runs, so the next prologue does not wait on them
    const float *next_norm;
    int next_k;
    int norm_staged;      // the previous phase staged this phase's norm weights
    int attn_in;          // the input is the attention output: merge split partials while loading (MkXLoad)
};

// chunk-stream view of one phase; the whole table lives in shared memory for the kernel's lifetime
struct MkLite {
    const uint8_t *tiles[3];
    int tbase[4];
    union {
        int rbase[4];     // host table: flat row-tile index where segment s starts; rbase[n_seg] = row tiles
        int own[4];       // a CTA's shared copy, from kernel start: [own[0], own[1]) = the CTA's flat tile range
    };
    int kt[3];            // k tiles per row tile of segment s
    int8_t kind, n_seg;
    int8_t fmt[3];
    int8_t pad[7];
};
static_assert(sizeof(MkLite) == 80, "MkLite is one 80-byte record");

struct MkCfg {
    int slots;            // ring depth per consumer warp
    int xr_bytes;         // activation / attention region at the start of dynamic shared memory
    int ph_off, lite_off, part_off, misc_off, nw_off, ring_off, bar_off;   // shared-memory offsets (bytes); bar_off:
                                                                            // full, then empty barriers
    int x_rtiles, x_ld;   // row tiles of the residual stream (d / 16, rounded up) and its row stride (d)
    const MkLite *lite;   // global copy of the lite table (n_phases records)
};

// per-step constants every phase reads, copied to shared memory once at kernel start: the state descriptor, each
// sequence's visible key span, the RoPE rows of positions c and W + c, and the step position
struct alignas(16) MkMisc {
    StateDev sd;
    KeySpan ks[GEMV_MB];
    float rope[2][128];
    int64_t pos;
    // the residual rows x[b, 16 r .. 16 r + 15] of the row tiles r in [own_r0, own_r0 + own_n) that this CTA owns in
    // the O and down phases (they own the same d-row tiles): kept here so the residual add reads no global memory
    float xown[MK_OWN_TILES][16][GEMV_MB];
    int own_r0, own_n;
    // biases of the CTA's QKV row tiles, refreshed at each QKV phase (16 per row tile, tile-row order)
    float qkv_bias[MK_OWN_TILES][16];
    int bias_r0, bias_n;
    // 1 from the CTA's arrival at a grid barrier until the next phase's activation prologue is done: the producer
    // issues no copies meanwhile, so the ring's refill does not queue in front of the prologue's loads
    volatile int quiet;
};

// activation loader of the persistent kernel's prologues: for the phase after attention, a sequence whose keys
// fell into 2 .. ATT_MERGE_MAX splits has only partials, merged here; everything else reads a.x
template <int D>
struct MkXLoad {
    const StateDev *s;
    const KeySpan *ks;
    int attn_in;
    __device__ __forceinline__ void operator()(const GemvArgs &a, int b, int u, bool vec, int n, float (&v)[8]) const {
        const int ns = (ks[b].total + ATT_KPC - 1) / ATT_KPC;
        if (attn_in && ns >= 2 && ns <= ATT_MERGE_MAX) attn_merged8<D>(*s, b, u * 8, ns, v);
        else load8<true>(a.x + (size_t)(a.b0 + b) * a.x_ld + u * 8, vec, n, v);
    }
};

// residual epilogue of the persistent kernel: x[b, row] += y, from the CTA's shared copy when it owns the row tile
struct MkEpiResid {
    float *x;
    int ld, rows;
    float (*xown)[16][GEMV_MB];
    int r0, n;
    __device__ void operator()(int, int rt, int g, int b, float y0, float y1) const {
        const int r = TILE_ROWS * rt + g, rl = rt - r0;
        if (rl >= 0 && rl < n) {
            const float v0 = xown[rl][g][b] + y0, v1 = xown[rl][g + 8][b] + y1;
            xown[rl][g][b] = v0;
            xown[rl][g + 8][b] = v1;
            if (r < rows) x[(size_t)b * ld + r] = v0;
            if (r + 8 < rows) x[(size_t)b * ld + r + 8] = v1;
        } else {   // L1-bypassing read: other SMs updated x in earlier phases
            if (r < rows) x[(size_t)b * ld + r] = __ldcg(&x[(size_t)b * ld + r]) + y0;
            if (r + 8 < rows) x[(size_t)b * ld + r + 8] = __ldcg(&x[(size_t)b * ld + r + 8]) + y1;
        }
    }
};

// shared-memory record of the split row tiles of one phase: per warp, a head piece (row tile begun by an earlier
// warp) and a tail piece (row tile begun here, continued by later warps)
struct MkPart {
    float v[MK_WARPS][2][32][4];
    int head_row[MK_WARPS];   // flat row tile of the head piece, -1 when none, -2 when the warp has no tiles
};

// ---------------------------------------------------------------------------------------------------------------
// bulk-copy ring primitives
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// L2 policy for streamed weights: evict first, so the weight stream (read once per step) does not push the
// activations, KV rows and counters that the phases hand each other out of L2
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// expect `bytes` on bar and copy them global -> shared (a plain CTA-local bulk copy of this GPU's memory) under L2 policy pol
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar, uint64_t pol) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(pol)
        : "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(done)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return done != 0;
}

// bounded wait for the completion of phase `parity` of bar; false when the limit ran out
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < MK_WAIT_LIMIT; ++i) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// ---------------------------------------------------------------------------------------------------------------
// per-warp chunk stream over all GEMV phases
// ---------------------------------------------------------------------------------------------------------------
struct MkCur {
    int p, si;            // phase (n_phases when exhausted) and segment of the next chunk
    int pend;             // 1: the range in phase p - 1 ended; the next range is searched from phase p (mk_grid_sync)
    int t, t1, send;      // next flat tile, end of this warp's range in phase p, end of the run in segment si
    int tl;               // tile index of t inside segment si
    int r, kt, KT;        // row tile / k tile of tl, k tiles per row tile
    int fmt;
    const uint8_t *tiles; // tile buffer of segment si
};

// flat tile index of the first tile of flat row tile R
__device__ __forceinline__ int mk_row_tile(const MkLite &L, int R) {
    int si = 0;
    while (si + 1 < L.n_seg && R >= L.rbase[si + 1]) ++si;
    return L.tbase[si] + (R - L.rbase[si]) * L.kt[si];
}

// CTA c (of G) owns the whole row tiles [c NR / G, (c+1) NR / G) of phase L: its flat tile range, computed once
// per phase at kernel start (it replaces rbase in the CTA's shared copy of the table)
__device__ __forceinline__ void mk_own_range(MkLite &L, int c, int G) {
    const int NR = L.rbase[L.n_seg];
    const int lo = mk_row_tile(L, (int)((int64_t)c * NR / G)), hi = mk_row_tile(L, (int)((int64_t)(c + 1) * NR / G));
    L.own[0] = lo;
    L.own[1] = hi;
}

// tile range [t0, t1) of consumer warp wi in phase L (L.own = the CTA's range).  A CTA range of fewer than two
// chunks per warp is cut at whole chunks (some warps then get none): a full chunk runs the fast path and costs
// little more than a partial one, and fewer pieces meet in the combine.
__device__ __forceinline__ void mk_range(const MkLite &L, int wi, int &t0, int &t1) {
    const int lo = L.own[0], n = L.own[1] - lo;
    if (n < 2 * MK_CHUNK * MK_WARPS) {
        const int nc = (n + MK_CHUNK - 1) / MK_CHUNK;
        t0 = lo + min(n, wi * nc / MK_WARPS * MK_CHUNK);
        t1 = lo + min(n, (wi + 1) * nc / MK_WARPS * MK_CHUNK);
    } else {
        t0 = lo + wi * n / MK_WARPS;
        t1 = lo + (wi + 1) * n / MK_WARPS;
    }
}

__device__ __forceinline__ void mk_seg(const MkLite &L, MkCur &c) {
    c.send = L.tbase[c.si + 1] < c.t1 ? L.tbase[c.si + 1] : c.t1;
    c.tl = c.t - L.tbase[c.si];
    c.KT = L.kt[c.si];
    c.r = c.tl / c.KT;
    c.kt = c.tl - c.r * c.KT;
    c.fmt = L.fmt[c.si];
    c.tiles = L.tiles[c.si];
}

__device__ __forceinline__ void mk_enter(const MkLite *lite, int n_phases, int wi, MkCur &c, int p) {
    c.pend = 0;
    for (; p < n_phases; ++p) {
        const MkLite &L = lite[p];
        if (L.kind != MK_GEMV) continue;
        int t0, t1;
        mk_range(L, wi, t0, t1);
        if (t0 >= t1) continue;
        c.p = p;
        c.t = t0;
        c.t1 = t1;
        c.si = 0;
        while (c.si + 1 < L.n_seg && c.t >= L.tbase[c.si + 1]) ++c.si;
        mk_seg(L, c);
        return;
    }
    c.p = n_phases;
}

__device__ __forceinline__ int mk_chunk_n(const MkCur &c) {
    const int cap = mk_cap(c.fmt);
    return c.send - c.t < cap ? c.send - c.t : cap;
}

// move the cursor past the n tiles of its current chunk.  LAZY: at the end of the range only mark the cursor
// pending (phase p + 1, searched later) -- the consumer warps look up their next range while they wait at the grid
// barrier instead of before the phase's closing combine
template <bool LAZY>
__device__ __forceinline__ void mk_advance(const MkLite *lite, int n_phases, int wi, MkCur &c, int n) {
    c.t += n;
    if (c.t >= c.t1) {
        if (LAZY) {
            ++c.p;
            c.pend = 1;
        } else {
            mk_enter(lite, n_phases, wi, c, c.p + 1);
        }
    } else if (c.t >= c.send) {
        ++c.si;
        mk_seg(lite[c.p], c);
    } else {
        c.tl += n;
        c.kt += n;
        while (c.kt >= c.KT) {
            c.kt -= c.KT;
            ++c.r;
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// row-tile results
// ---------------------------------------------------------------------------------------------------------------
template <class Epi>
__device__ __forceinline__ void mk_emit(const Epi &epi, int B, int si, int r, int lane, float y0, float y1, float y2,
                                        float y3) {
    const int g = lane >> 2, t = lane & 3;
    if (2 * t < B) epi(si, r, g, 2 * t, y0, y2);
    if (2 * t + 1 < B) epi(si, r, g, 2 * t + 1, y1, y3);
}

// ---------------------------------------------------------------------------------------------------------------
// tile arithmetic on shared-memory chunks
// ---------------------------------------------------------------------------------------------------------------
// Activations: xq = this lane's fragment records (row g of the converted activations, row 0 for lanes of absent
// batch rows g >= B: the tensor-core columns they feed are never read, quad position t), xbs = records per 32-wide
// k block (4 B); bq = bsum + 2t.  See XFrag for the record layout.

// one tile at tb (shared memory) with k tile kt, accumulated into acc (rows g, g+8 x batch 2t, 2t+1)
template <int FMT>
__device__ __forceinline__ void mk_tile(const uint8_t *tb, int kt, const uint4 *xq, int xbs, const float *bq,
                                        int lane, float (&acc)[4]) {
    const int g = lane >> 2;
    const uint4 q = *reinterpret_cast<const uint4 *>(tb + lane * 16);
    if constexpr (FMT == FMT_Q8) {
        const uint32_t sc = *reinterpret_cast<const uint32_t *>(tb + 512 + g * 4);
        const uint4 xv = xq[kt * xbs];
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(d, q8_pair(q.x, 0x4140u), q8_pair(q.x, 0x4342u), q8_pair(q.y, 0x4140u), q8_pair(q.y, 0x4342u), xv.x,
                 xv.y);
        mma16816(d, q8_pair(q.z, 0x4140u), q8_pair(q.z, 0x4342u), q8_pair(q.w, 0x4140u), q8_pair(q.w, 0x4342u), xv.z,
                 xv.w);
        const float2 S = *reinterpret_cast<const float2 *>(bq + kt * GEMV_MB);
        const float2 ds = h2f2(sc);
        acc[0] = fmaf(ds.x, fmaf(-1152.f, S.x, d[0]), acc[0]);
        acc[1] = fmaf(ds.x, fmaf(-1152.f, S.y, d[1]), acc[1]);
        acc[2] = fmaf(ds.y, fmaf(-1152.f, S.x, d[2]), acc[2]);
        acc[3] = fmaf(ds.y, fmaf(-1152.f, S.y, d[3]), acc[3]);
    } else if constexpr (FMT == FMT_Q4) {
        const uint2 sc = *reinterpret_cast<const uint2 *>(tb + 512 + g * 8);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w}, scw[2] = {sc.x, sc.y};
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
            const uint4 xv = xq[(2 * kt + blk) * xbs];
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(d, q4_pair<0>(w[2 * blk]), q4_pair<4>(w[2 * blk]), q4_pair<8>(w[2 * blk]), q4_pair<12>(w[2 * blk]),
                     xv.x, xv.y);
            mma16816(d, q4_pair<0>(w[2 * blk + 1]), q4_pair<4>(w[2 * blk + 1]), q4_pair<8>(w[2 * blk + 1]),
                     q4_pair<12>(w[2 * blk + 1]), xv.z, xv.w);
            const float2 S = *reinterpret_cast<const float2 *>(bq + (2 * kt + blk) * GEMV_MB);
            const float2 ds = h2f2(scw[blk]);
            acc[0] = fmaf(ds.x, fmaf(-1032.f, S.x, d[0]), acc[0]);
            acc[1] = fmaf(ds.x, fmaf(-1032.f, S.y, d[1]), acc[1]);
            acc[2] = fmaf(ds.y, fmaf(-1032.f, S.x, d[2]), acc[2]);
            acc[3] = fmaf(ds.y, fmaf(-1032.f, S.y, d[3]), acc[3]);
        }
    } else {   // 16-wide k tiles: one k16 step, half of a block record
        const uint2 xv = reinterpret_cast<const uint2 *>(xq + (kt >> 1) * xbs)[kt & 1];
        if constexpr (FMT == FMT_F32) {   // planes accumulate apart, then hi + 2^-11 mid + 2^-22 lo
            const uint4 m = *reinterpret_cast<const uint4 *>(tb + 512 + lane * 16);
            const uint4 l = *reinterpret_cast<const uint4 *>(tb + 1024 + lane * 16);
            float dm[4] = {0.f, 0.f, 0.f, 0.f}, dl[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(acc, q.x, q.y, q.z, q.w, xv.x, xv.y);
            mma16816(dm, m.x, m.y, m.z, m.w, xv.x, xv.y);
            mma16816(dl, l.x, l.y, l.z, l.w, xv.x, xv.y);
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = fmaf(dm[i], F32_MID, fmaf(dl[i], F32_LO, acc[i]));
        } else {   // fp16 tiles (F16 files, BF16 weights stored as scaled fp16)
            mma16816(acc, q.x, q.y, q.z, q.w, xv.x, xv.y);
        }
    }
}

// MK_GROUP consecutive tiles of one row tile: every shared load first, then the tensor-core chains
template <int FMT>
__device__ __forceinline__ void mk_chunk_fast(const uint8_t *sb, int kt, const uint4 *xq, int xbs, const float *bq,
                                              int lane, float (&acc)[4]) {
    constexpr int TB = tile_bytes(FMT), N = MK_GROUP;
    const int g = lane >> 2;
    uint4 q[N];
    uint2 sc[N];
    uint32_t b0[N][4], b1[N][4];   // B fragments of each tile's k16 steps (Q4: 4, Q8: 2, 16-bit: 1)
#pragma unroll
    for (int i = 0; i < N; ++i) {
        q[i] = *reinterpret_cast<const uint4 *>(sb + i * TB + lane * 16);
        if constexpr (FMT == FMT_Q8) {
            sc[i].x = *reinterpret_cast<const uint32_t *>(sb + i * TB + 512 + g * 4);
            const uint4 xv = xq[(kt + i) * xbs];
            b0[i][0] = xv.x;
            b1[i][0] = xv.y;
            b0[i][1] = xv.z;
            b1[i][1] = xv.w;
        } else if constexpr (FMT == FMT_Q4) {
            sc[i] = *reinterpret_cast<const uint2 *>(sb + i * TB + 512 + g * 8);
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                const uint4 xv = xq[(2 * (kt + i) + blk) * xbs];
                b0[i][2 * blk] = xv.x;
                b1[i][2 * blk] = xv.y;
                b0[i][2 * blk + 1] = xv.z;
                b1[i][2 * blk + 1] = xv.w;
            }
        } else {
            const uint2 xv = reinterpret_cast<const uint2 *>(xq + ((kt + i) >> 1) * xbs)[(kt + i) & 1];
            b0[i][0] = xv.x;
            b1[i][0] = xv.y;
        }
    }
    if constexpr (FMT == FMT_Q8) {
        float d[N][4];
#pragma unroll
        for (int i = 0; i < N; ++i) {
            d[i][0] = d[i][1] = d[i][2] = d[i][3] = 0.f;
            const uint32_t w[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
#pragma unroll
            for (int s = 0; s < 2; ++s)
                mma16816(d[i], q8_pair(w[2 * s], 0x4140u), q8_pair(w[2 * s], 0x4342u), q8_pair(w[2 * s + 1], 0x4140u),
                         q8_pair(w[2 * s + 1], 0x4342u), b0[i][s], b1[i][s]);
        }
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const float2 S = *reinterpret_cast<const float2 *>(bq + (kt + i) * GEMV_MB);
            const float2 ds = h2f2(sc[i].x);
            acc[0] = fmaf(ds.x, fmaf(-1152.f, S.x, d[i][0]), acc[0]);
            acc[1] = fmaf(ds.x, fmaf(-1152.f, S.y, d[i][1]), acc[1]);
            acc[2] = fmaf(ds.y, fmaf(-1152.f, S.x, d[i][2]), acc[2]);
            acc[3] = fmaf(ds.y, fmaf(-1152.f, S.y, d[i][3]), acc[3]);
        }
    } else if constexpr (FMT == FMT_Q4) {
        float d[N][2][4];
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const uint32_t w[4] = {q[i].x, q[i].y, q[i].z, q[i].w};
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                d[i][blk][0] = d[i][blk][1] = d[i][blk][2] = d[i][blk][3] = 0.f;
                mma16816(d[i][blk], q4_pair<0>(w[2 * blk]), q4_pair<4>(w[2 * blk]), q4_pair<8>(w[2 * blk]),
                         q4_pair<12>(w[2 * blk]), b0[i][2 * blk], b1[i][2 * blk]);
                mma16816(d[i][blk], q4_pair<0>(w[2 * blk + 1]), q4_pair<4>(w[2 * blk + 1]), q4_pair<8>(w[2 * blk + 1]),
                         q4_pair<12>(w[2 * blk + 1]), b0[i][2 * blk + 1], b1[i][2 * blk + 1]);
            }
        }
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const uint32_t scw[2] = {sc[i].x, sc[i].y};
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                const float2 S = *reinterpret_cast<const float2 *>(bq + (2 * (kt + i) + blk) * GEMV_MB);
                const float2 ds = h2f2(scw[blk]);
                acc[0] = fmaf(ds.x, fmaf(-1032.f, S.x, d[i][blk][0]), acc[0]);
                acc[1] = fmaf(ds.x, fmaf(-1032.f, S.y, d[i][blk][1]), acc[1]);
                acc[2] = fmaf(ds.y, fmaf(-1032.f, S.x, d[i][blk][2]), acc[2]);
                acc[3] = fmaf(ds.y, fmaf(-1032.f, S.y, d[i][blk][3]), acc[3]);
            }
        }
    } else {   // fp16 tiles: independent accumulators, summed at the end
        float d[N][4];
#pragma unroll
        for (int i = 0; i < N; ++i) {
            d[i][0] = d[i][1] = d[i][2] = d[i][3] = 0.f;
            mma16816(d[i], q[i].x, q[i].y, q[i].z, q[i].w, b0[i][0], b1[i][0]);
        }
#pragma unroll
        for (int i = 0; i < N; ++i) {
            acc[0] += d[i][0];
            acc[1] += d[i][1];
            acc[2] += d[i][2];
            acc[3] += d[i][3];
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// consumer warps
// ---------------------------------------------------------------------------------------------------------------
struct MkRing {
    const uint8_t *buf;   // slot 0 of this warp's ring (slots * MK_SLOT_BYTES)
    uint32_t full, empty; // shared addresses of this warp's first full / empty mbarrier
    int slots;
    int slot;             // slot of the next chunk
    uint32_t phase;       // parity of the next chunk's use of its slot
    MkCur cons;
    bool dead;            // a wait ran out: stop computing (the step is reported invalid)
};

// One GEMV phase for one consumer warp.  Every consumer warp of the CTA calls it (the closing combine synchronises
// them); warps without tiles in the phase only take part in the combine.
template <int FA, int FB, class Epi>
__device__ __forceinline__ void mk_consume(const MkPhase &P, const Epi &epi, MkRing &R, const MkLite *lite,
                                           int n_phases, int p, int cta, int G, int wi, const uint4 *xq,
                                           const float *bq, const float *s_scale, MkPart &part, int *status,
                                           int lane) {
    const int t = lane & 3, B = P.a.B, xbs = 4 * gemv_xrows(B, P.a.lo);
    const float sc0 = 2 * t < B ? s_scale[2 * t] : 0.f, sc1 = 2 * t + 1 < B ? s_scale[2 * t + 1] : 0.f;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int cur_si = -1, cur_r = -1;
    int tail_si = -1, tail_r = -1;   // split row tile begun in this warp, finished after the phase
    int t0w = 0, t1w = 0;
    mk_range(lite[p], wi, t0w, t1w);
    if (lane == 0) part.head_row[wi] = t0w < t1w ? -1 : -2;
    auto flush = [&]() {   // the finished piece of row tile (cur_si, cur_r)
        gemv_fold_lo(P.a.lo, acc);
        const float ws = P.a.seg[cur_si].wscale, s0 = sc0 * ws, s1 = sc1 * ws;
        const float y0 = acc[0] * s0, y1 = acc[1] * s1, y2 = acc[2] * s0, y3 = acc[3] * s1;
        const int KT = P.a.seg[cur_si].n_ktiles;
        const int rs = P.tbase[cur_si] + cur_r * KT, re = rs + KT;
        if (rs >= t0w && re <= t1w) {
            mk_emit(epi, B, cur_si, cur_r, lane, y0, y1, y2, y3);
            return;
        }
        const int slot = rs < t0w ? 0 : 1;
        *reinterpret_cast<float4 *>(part.v[wi][slot][lane]) = make_float4(y0, y1, y2, y3);
        if (slot == 0) {
            if (lane == 0) part.head_row[wi] = P.rbase[cur_si] + cur_r;
        } else {
            tail_si = cur_si;
            tail_r = cur_r;
        }
    };
    while (R.cons.p == p) {
        const int n = mk_chunk_n(R.cons), si = R.cons.si, KT = R.cons.KT;
        int r = R.cons.r, kt = R.cons.kt;
        const bool fa = FA == FB || R.cons.fmt == FA;
        if (!R.dead && !mbar_wait(R.full + R.slot * 8, R.phase)) {
            R.dead = true;
            if (lane == 0) atomicOr(status, STATUS_TIMEOUT);
        }
        const uint8_t *sb = R.buf + R.slot * MK_SLOT_BYTES;
        if (r != cur_r || si != cur_si) {
            if (cur_r >= 0) flush();
            cur_r = r;
            cur_si = si;
            acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        }
        if (!R.dead) {
            constexpr bool F32A = FA == FMT_F32, F32B = FB == FMT_F32;
            const int tbytes = fa ? tile_bytes(FA) : tile_bytes(FB);
            if (n == MK_CHUNK && kt + MK_CHUNK <= KT && !(fa ? F32A : F32B)) {   // whole chunk in one row tile
#pragma unroll
                for (int g0 = 0; g0 < MK_CHUNK; g0 += MK_GROUP) {
                    if (fa) mk_chunk_fast<F32A ? FMT_Q8 : FA>(sb + g0 * tbytes, kt + g0, xq, xbs, bq, lane, acc);
                    else mk_chunk_fast<F32B ? FMT_Q8 : FB>(sb + g0 * tbytes, kt + g0, xq, xbs, bq, lane, acc);
                }
                kt += MK_CHUNK;
                if (kt == KT) kt = 0;
            } else for (int i = 0; i < n;) {   // groups of MK_GROUP tiles inside one row tile, single tiles otherwise
                if (i > 0 && kt == 0) {
                    flush();
                    cur_r = ++r;
                    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
                }
                if (i + MK_GROUP <= n && kt + MK_GROUP <= KT && !(fa ? F32A : F32B)) {
                    if (fa) mk_chunk_fast<F32A ? FMT_Q8 : FA>(sb + i * tbytes, kt, xq, xbs, bq, lane, acc);
                    else mk_chunk_fast<F32B ? FMT_Q8 : FB>(sb + i * tbytes, kt, xq, xbs, bq, lane, acc);
                    i += MK_GROUP;
                    kt += MK_GROUP;
                } else {
                    if (fa) mk_tile<FA>(sb + i * tbytes, kt, xq, xbs, bq, lane, acc);
                    else mk_tile<FB>(sb + i * tbytes, kt, xq, xbs, bq, lane, acc);
                    ++i;
                    ++kt;
                }
                if (kt == KT) kt = 0;
            }
            __syncwarp();   // every tile byte of the slot is in registers: release it to the producer
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(R.empty + R.slot * 8) : "memory");
        }
        if (++R.slot == R.slots) {
            R.slot = 0;
            R.phase ^= 1u;
        }
        mk_advance<true>(lite, n_phases, wi, R.cons, n);
    }
    if (cur_r >= 0) flush();
    sync_threads(MK_CT);   // every piece of every split row tile is in shared memory
    if (tail_r >= 0) {     // this warp began the row tile: add the later warps' pieces in order, then the epilogue
        const int row = P.rbase[tail_si] + tail_r;
        float4 y = *reinterpret_cast<const float4 *>(part.v[wi][1][lane]);
        for (int v = wi + 1; v < MK_WARPS; ++v) {
            const int hr = part.head_row[v];
            if (hr == -2) continue;   // a warp without tiles inside the row tile
            if (hr != row) break;
            const float4 q = *reinterpret_cast<const float4 *>(part.v[v][0][lane]);
            y.x += q.x;
            y.y += q.y;
            y.z += q.z;
            y.w += q.w;
        }
        mk_emit(epi, B, tail_si, tail_r, lane, y.x, y.y, y.z, y.w);
    }
}

// Every epilogue of the kernel behind one runtime switch, built from the shared-memory phase descriptor at each
// call and kept out of line.  Epilogues run once per row tile, so the switch and the call cost little, while ONE
// compact copy of the consume loop then serves every GEMV phase: its instructions stay cached from phase to phase
// instead of four inlined copies evicting one another (measured: 1745 -> 1650 us per 1.5B Q8_0 token).
struct MkEpiAny {
    const MkPhase *P;
    const ModelDev *mp;
    MkMisc *ms;
    __device__ __noinline__ void operator()(int si, int rt, int g, int b, float y0, float y1) const {
        switch (P->epi) {
            case MK_EPI_QKV: {
                const EpiQKV e{mp,          &ms->sd,     P->layer, P->bq, P->bk, P->bv, ms->rope[0],
                               ms->rope[1], ms->pos,     &ms->qkv_bias[0][0], ms->bias_r0, ms->bias_n,
                               P->rbase[1], P->rbase[2]};
                e(si, rt, g, b, y0, y1);
                break;
            }
            case MK_EPI_RESID: {
                const MkEpiResid e{P->out, P->out_ld, P->out_rows, ms->xown, ms->own_r0, ms->own_n};
                e(si, rt, g, b, y0, y1);
                break;
            }
            case MK_EPI_GATEUP: {
                const EpiGateUp e{P->out, P->out_rows};
                e(si, rt, g, b, y0, y1);
                break;
            }
            default: {
                const EpiStore e{P->out, P->out_ld, P->out_rows};
                e(si, rt, g, b, y0, y1);
                break;
            }
        }
    }
};

template <int FA, int FB>
__device__ __forceinline__ void mk_consume_epi(const MkPhase &P, const ModelDev *mp, MkMisc &ms, MkRing &R,
                                               const MkLite *lite, int n_phases, int p, int cta, int G, int wi,
                                               const uint4 *xq, const float *bq, const float *s_scale,
                                               MkPart &part, int *status, int lane) {
    const MkEpiAny e{&P, mp, &ms};
    mk_consume<FA, FB>(P, e, R, lite, n_phases, p, cta, G, wi, xq, bq, s_scale, part, status, lane);
}

// ---------------------------------------------------------------------------------------------------------------
// producer warp: lane i streams consumer warp i's chunks into its ring, a slot as soon as the consumer released it
// (empty barrier), until the stream ends; then waits (bounded) until its last copies have landed
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mk_produce(const MkLite *lite, int n_phases, int c, int G, const MkCfg &cfg,
                                           uint8_t *smem, const StateDev *sp) {
    const int lane = threadIdx.x & 31;
    if (lane >= MK_WARPS) return;
    const volatile int *quiet = &reinterpret_cast<MkMisc *>(smem + cfg.misc_off)->quiet;
    uint32_t hush = 0;
    const int S = cfg.slots;
    const uint32_t buf = smem_u32(smem + cfg.ring_off + (size_t)lane * S * MK_SLOT_BYTES);
    const uint32_t full = smem_u32(smem + cfg.bar_off) + (uint32_t)(lane * S * 8);
    const uint32_t empty = full + (uint32_t)(MK_WARPS * S * 8);
    MkCur cur;
    mk_enter(lite, n_phases, lane, cur, 0);
    uint32_t slot = 0, round = 0, idle = 0;
    const uint64_t pol = l2_evict_first();
#ifdef V3G_MK_TRACE
    int traced = -1;
#endif
    while (cur.p < n_phases) {
        if (round > 0 && !mbar_test(empty + slot * 8, (round - 1) & 1u)) {   // slot still in use
            if (++idle > MK_WAIT_LIMIT) {
                atomicOr(&sp->step->status, STATUS_TIMEOUT);
                break;
            }
            __nanosleep(32);
            continue;
        }
        idle = 0;
        if (*quiet && hush < MK_WAIT_LIMIT) {   // hold the copy while the consumers load activations (bounded)
            ++hush;
            __nanosleep(64);
            continue;
        }
        hush = 0;
#ifdef V3G_MK_TRACE
        if (lane == 0 && cur.p != traced) {
            traced = cur.p;
            MK_TRACE(cur.p, 4);
        }
#endif
        const int n = mk_chunk_n(cur);
        const int tb = tile_bytes(cur.fmt);
        bulk_load(buf + slot * MK_SLOT_BYTES, cur.tiles + (size_t)cur.tl * tb, (uint32_t)(n * tb), full + slot * 8, pol);
        mk_advance<false>(lite, n_phases, lane, cur, n);
        if (++slot == (uint32_t)S) {
            slot = 0;
            ++round;
        }
    }
    // the last use of every slot: wait until its copy has landed
    for (uint32_t sl = 0; sl < (uint32_t)S; ++sl) {
        if (round == 0 && sl >= slot) continue;   // never used
        const uint32_t use = sl < slot ? round : round - 1;
        mbar_wait(full + sl * 8, use & 1u);
    }
}

// asynchronous copy of phases[p] into a shared-memory slot (consumer threads 0 .. sizeof/16 - 1)
__device__ __forceinline__ void mk_fetch_phase(const MkPhase *phases, int p, int n_phases, MkPhase *dst) {
    constexpr int N16 = (int)(sizeof(MkPhase) / 16);
    static_assert(N16 <= MK_CT, "one 16-byte piece per consumer thread");
    if (p < n_phases && (int)threadIdx.x < N16)
        cp_async16(reinterpret_cast<uint8_t *>(dst) + threadIdx.x * 16,
                   reinterpret_cast<const uint8_t *>(phases + p) + threadIdx.x * 16);
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// bounded grid barrier over the consumer warps: every CTA arrives once per phase on a counter zeroed at the start
// of the step; a wait that exceeds its iteration limit records STATUS_TIMEOUT and returns (results then invalid).
// Between the CTA's arrival and the wait each consumer warp moves a pending chunk cursor to its next range.
__device__ __forceinline__ void mk_grid_sync(unsigned int *bar, unsigned int target, int *status, const MkLite *lite,
                                             int n_phases, int wi, MkCur &cur) {
    sync_threads(MK_CT);
    if (threadIdx.x == 0)   // release-add (the CTA's writes, ordered by the barrier above)
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
    if (cur.pend) mk_enter(lite, n_phases, wi, cur, cur.p);
    if (threadIdx.x == 0) {   // acquire-poll
        unsigned int v = 0;
        for (uint32_t spins = 0;; ++spins) {
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
            if (v >= target) break;
            if (spins > MK_WAIT_LIMIT) {
                atomicOr(status, STATUS_TIMEOUT);
                break;
            }
        }
    }
    sync_threads(MK_CT);
}

template <int D, int FA, int FB>
__global__ void __launch_bounds__(MK_THREADS, 1) k_decode(const ModelDev *mp, const StateDev *sp,
                                                          const MkPhase *phases, int n_phases, float scale,
                                                          MkCfg cfg) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int c = blockIdx.x, G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    MkPhase *ph_s = reinterpret_cast<MkPhase *>(smem + cfg.ph_off);
    MkLite *lite = reinterpret_cast<MkLite *>(smem + cfg.lite_off);
    // the lite table (immutable), the first two phase descriptors and the ring barriers
    for (int i = threadIdx.x; i < n_phases * (int)(sizeof(MkLite) / 16); i += blockDim.x)
        cp_async16(reinterpret_cast<uint8_t *>(lite) + i * 16, reinterpret_cast<const uint8_t *>(cfg.lite) + i * 16);
    if (warp < MK_WARPS) {
        mk_fetch_phase(phases, 0, n_phases, ph_s);
        mk_fetch_phase(phases, 1, n_phases, ph_s + 1);
    }
    const uint32_t bars = smem_u32(smem + cfg.bar_off);
    for (int i = threadIdx.x; i < 2 * MK_WARPS * cfg.slots; i += blockDim.x)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bars + i * 8) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    for (int p = threadIdx.x; p < n_phases; p += blockDim.x)   // this CTA's tile range of every GEMV phase
        if (lite[p].kind == MK_GEMV) mk_own_range(lite[p], c, G);
    if (threadIdx.x == 0) reinterpret_cast<MkMisc *>(smem + cfg.misc_off)->quiet = 0;
    __syncthreads();
    if (warp == MK_WARPS) {   // weights are immutable: the producer streams from the very start
        mk_produce(lite, n_phases, c, G, cfg, smem, sp);
        return;
    }
    // per-step constants into shared memory (state descriptor, then position, key spans and RoPE rows)
    MkMisc &misc = *reinterpret_cast<MkMisc *>(smem + cfg.misc_off);
    griddep_wait();
    static_assert(sizeof(StateDev) % 4 == 0, "word copy");
    for (int i = threadIdx.x; i < (int)(sizeof(StateDev) / 4); i += MK_CT)
        reinterpret_cast<uint32_t *>(&misc.sd)[i] = __ldcg(reinterpret_cast<const uint32_t *>(sp) + i);
    const float *rope_tab = mp->rope;
    const int rope_pos0 = mp->rope_pos0;
    sync_threads(MK_CT);
    const StateDev &st = misc.sd;
    int *status = &st.step->status;
    const int64_t pos = __ldcg(&st.step->pos);
    if ((int)threadIdx.x < st.B) misc.ks[threadIdx.x] = key_span(st, threadIdx.x, pos);
    {
        const int cpos = (int)(pos % st.W);
        for (int i = threadIdx.x; i < 2 * D; i += MK_CT) {
            const int row = i / D;
            const int64_t rp = (row ? st.W + cpos : cpos) - rope_pos0;
            misc.rope[row][i - row * D] = __ldg(rope_tab + rp * D + (i - row * D));
        }
    }
    if (threadIdx.x == 0) misc.pos = pos;
    {   // the residual row tiles this CTA owns in the O and down phases
        const int r0 = (int)((int64_t)c * cfg.x_rtiles / G), r1 = (int)((int64_t)(c + 1) * cfg.x_rtiles / G);
        const int n = r1 - r0 <= MK_OWN_TILES ? r1 - r0 : 0;
        if (threadIdx.x == 0) {
            misc.own_r0 = r0;
            misc.own_n = n;
        }
        for (int i = threadIdx.x; i < n * 16 * GEMV_MB; i += MK_CT) {
            const int b = i % GEMV_MB, rr = (i / GEMV_MB) % 16, rl = i / (16 * GEMV_MB);
            const int row = (r0 + rl) * 16 + rr;
            misc.xown[rl][rr][b] = (b < st.B && row < cfg.x_ld) ? __ldcg(&st.x[(size_t)b * cfg.x_ld + row]) : 0.f;
        }
    }
    sync_threads(MK_CT);
    MkRing R;
    R.slots = cfg.slots;
    R.buf = smem + cfg.ring_off + (size_t)warp * cfg.slots * MK_SLOT_BYTES;
    R.full = bars + (uint32_t)(warp * cfg.slots * 8);
    R.empty = R.full + (uint32_t)(MK_WARPS * cfg.slots * 8);
    R.slot = 0;
    R.phase = 0;
    R.dead = false;
    mk_enter(lite, n_phases, warp, R.cons, 0);
    MkPart &part = *reinterpret_cast<MkPart *>(smem + cfg.part_off);
    const int n_kv = st.G, ms = st.max_splits, Bst = st.B;
    unsigned int *gbar = st.bar;
    constexpr bool BSUM = fmt_int(FA) || fmt_int(FB);
    float *s_red = reinterpret_cast<float *>(smem);
    float *s_scale = s_red + 136;
    float *bsum = s_scale + GEMV_MB;
    for (int p = 0; p < n_phases; ++p) {
        const MkPhase &P = ph_s[p & 1];
        if (threadIdx.x == 0) MK_TRACE(p, 0);
        if (P.kind == MK_ATTN) {
            const int n_items = Bst * n_kv * ms;
            for (int i = c; i < n_items; i += G) {
                const int split = i % ms, g = (i / ms) % n_kv, b = i / (ms * n_kv);
                attn_item<D>(st, misc.ks[b], P.layer, scale, split, g, b, pos, *reinterpret_cast<AttnSmem<D> *>(smem),
                             MK_CT, true);
            }
        } else {
            uint16_t *xs = reinterpret_cast<uint16_t *>(bsum + (BSUM ? P.a.nblk * GEMV_MB : 0));
            if (P.epi == MK_EPI_QKV && threadIdx.x >= MK_CT - 32) {   // the last warp stages this CTA's biases
                const int NR = P.a.total_rtiles;
                const int r0 = (int)((int64_t)c * NR / G), r1 = (int)((int64_t)(c + 1) * NR / G);
                const int n = r1 - r0 <= MK_OWN_TILES ? r1 - r0 : 0;
                for (int i = threadIdx.x - (MK_CT - 32); i < n * 16; i += 32) {
                    const int R = r0 + i / 16, tr = i % 16;
                    const int si = R >= P.rbase[2] ? 2 : (R >= P.rbase[1] ? 1 : 0), rt = R - P.rbase[si];
                    const int row = (rt / (D / TILE_ROWS)) * D + 8 * (rt % (D / TILE_ROWS)) + (tr & 7) + (tr & 8 ? D / 2 : 0);
                    misc.qkv_bias[i / 16][tr] = __ldg((si == 0 ? P.bq : (si == 1 ? P.bk : P.bv)) + row);
                }
                if (threadIdx.x == MK_CT - 32) {
                    misc.bias_r0 = r0;
                    misc.bias_n = n;
                }
            }
            float *nw_s = reinterpret_cast<float *>(smem + cfg.nw_off);
            // a CTA without row tiles in this phase converts nothing (CTA 0 still captures scorer features)
            if (lite[p].own[1] > lite[p].own[0] || (P.a.feat && c == 0))
                gemv_prologue<BSUM, 5>(P.a, xs, s_scale, s_red, bsum, MK_CT, P.norm_staged ? nw_s : nullptr,
                                       MkXLoad<D>{&misc.sd, misc.ks, P.attn_in}, p);
            if (threadIdx.x == 0) misc.quiet = 0;   // activations are in place: the ring may refill
            if (P.next_norm) {   // stage the next phase's norm weights while this one streams (landed by the barrier)
                for (int i = threadIdx.x; i < P.next_k / 4; i += MK_CT) cp_async16(nw_s + 4 * i, P.next_norm + 4 * i);
                asm volatile("cp.async.commit_group;" ::: "memory");
            }
            if (threadIdx.x == 0) MK_TRACE(p, 1);
            const int g = lane >> 2, t = lane & 3;
            const uint4 *xq = reinterpret_cast<const uint4 *>(xs) + gemv_rec_row(P.a.B, P.a.lo, g) * 4 + t;
            mk_consume_epi<FA, FB>(P, mp, misc, R, lite, n_phases, p, c, G, warp, xq, bsum + 2 * t, s_scale, part,
                                   status, lane);
        }
        if (threadIdx.x == 0) MK_TRACE(p, 2);
        if (p + 1 < n_phases) {
            asm volatile("cp.async.wait_all;" ::: "memory");   // descriptor p + 1 is in place after the barrier
            if (threadIdx.x == 0 && lite[p + 1].kind == MK_GEMV) misc.quiet = 1;
            mk_grid_sync(gbar, (unsigned int)(p + 1) * (unsigned int)G, status, lite, n_phases, warp, R.cons);
            if (threadIdx.x == 0) MK_TRACE(p, 3);
            mk_fetch_phase(phases, p + 2, n_phases, ph_s + (p & 1));   // slot of phase p, now unused
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    griddep_launch();
}

}  // namespace v3g
