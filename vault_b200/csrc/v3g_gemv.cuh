// Decode GEMV: y[b, :] = W x[b, :] for up to 8 batch rows per pass, weights streamed once from HBM.
//
// Weights are the A operand of mma.sync m16n8k16 (16-row tiles, see v3g.cuh), activations the B operand (batch
// rows = the 8 columns).  Each CTA (8 warps) owns 8/WK row tiles and the WK warps of a row tile split its k tiles.
// A warp issues the loads of its first weight tiles before it waits for the previous kernel (programmatic
// dependent launch) and before the activation prologue, then streams double-buffered batches of tiles.  The
// prologue converts the activation rows once per CTA into shared memory -- fp16 with a per-row power-of-two scale
// -- and, for integer weights, the fp32 sum of every 32-wide block of the converted activations.  Every tile
// format is fp16 on the tensor core (BF16 / F32 weights as scaled fp16 planes, see v3g.cuh); integer codes enter
// it as exact fp16 integers
// C + q (C = 1152 for Q8_0 via one byte-permute, C = 1032 for Q4_0 via one mask); each block result is corrected
// by -C * blocksum and scaled by its fp16 block scale in fp32.  Partial sums of the WK warps are reduced in shared
// memory in a fixed order (deterministic), then a fused epilogue consumes (y[row g], y[row g+8]) in registers.
#pragma once
#include "v3g.cuh"

namespace v3g {

constexpr int PRO_PLAIN = 0, PRO_RMSNORM = 1;
constexpr int GEMV_U = 4;   // tiles per batch (two batches in flight)

struct GemvSeg {
    const uint8_t *tiles;
    int n_rtiles, n_ktiles;
    float wscale;     // MatW::wscale of this segment (applied with the activation scale)
};

struct GemvArgs {
    GemvSeg seg[3];
    int n_seg;
    int seg_base;     // segment index reported to the epilogue for seg[0]
    int total_rtiles;
    int K;            // logical K
    int kpx;          // padded K + 8 (kept for the host plan; the converted activations use nblk 32-blocks)
    int nblk;         // 32-wide blocks of the padded K (block sums)
    int B;            // batch rows in this pass (<= GEMV_MB)
    int lo;           // tensor-core column of the first low activation part (gemv_lo), 0: one fp16 part per row
    int b0;           // first batch row of this pass
    int wk;           // warps per row tile
    const float *x;   // fp32 activations, row b at x + (b0 + b) * x_ld
    int x_ld;
    int prologue;
    const float *norm_w;
    float eps;
    float *feat;      // optional copy of the raw input rows (scorer features), row b at feat + (b0 + b) * feat_ld
    int feat_ld;
};

__host__ __device__ constexpr bool fmt_int(int fmt) { return fmt == FMT_Q8 || fmt == FMT_Q4; }

// Activation precision.  A batch of B <= 4 rows leaves tensor-core columns free, so every activation row enters as
// two fp16 parts -- high part x_h = fp16(x), low part x_l = fp16(x - x_h), about 22 significant bits together --
// in columns b (high) and P + b (low), P = 1, 2 or 4; the two columns are added after the tensor core.  Larger
// batches keep one fp16 part per row (11 bits); a state may also ask for one part at any batch (GemvArgs::lo = 0).
// gemv_lo(B) = P (0: no low parts), gemv_xrows(B, P) = record rows.
__host__ __device__ constexpr int gemv_lo(int B) { return B == 1 ? 1 : (B == 2 ? 2 : (B <= 4 ? 4 : 0)); }
__host__ __device__ constexpr int gemv_xrows(int B, int P) { return P ? 2 * P : B; }
// record row read by the lanes of tensor-core column g: its own row when it holds data, else row 0 (the columns of
// absent rows are computed and never read)
__device__ __forceinline__ int gemv_rec_row(int B, int P, int g) {
    if (P) return (g < 2 * P && (g & (P - 1)) < B) ? g : 0;
    return g < B ? g : 0;
}
// add the low-part columns into the high-part columns of a lane's accumulators (rows g, g+8 x columns 2t, 2t+1);
// every lane of the warp must call it together
__device__ __forceinline__ void gemv_fold_lo(int P, float (&acc)[4]) {
    if (P == 1) {
        acc[0] += acc[1];
        acc[2] += acc[3];
    } else if (P) {
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], P >> 1);
    }
}
__host__ __device__ constexpr float fmt_offset(int fmt) { return fmt == FMT_Q8 ? 1152.f : 1032.f; }

__device__ __forceinline__ float2 h2f2(uint32_t h) {
    __half2 v = *reinterpret_cast<__half2 *>(&h);
    return __half22float2(v);
}
// two +128-biased codes (bytes selected by `sel`) -> fp16x2 {1024 + u} = {1152 + q}, exact
__device__ __forceinline__ uint32_t q8_pair(uint32_t w, uint32_t sel) { return __byte_perm(w, 0x64646464u, sel); }
// nibbles at bits [sh, sh+4) and [sh+16, sh+20) -> fp16x2 {1024 + n} = {1032 + (n - 8)}, exact
template <int SH>
__device__ __forceinline__ uint32_t q4_pair(uint32_t w) {
    return ((w >> SH) & 0x000F000Fu) | 0x64006400u;
}

struct TileRegs {
    uint4 q;        // codes / hi plane
    uint2 s;        // block scales (Q8: .x; Q4: .x, .y)
    uint4 m, l;     // mid / lo planes (F32)
};

template <int FMT>
__device__ __forceinline__ void load_tile(TileRegs &r, const uint8_t *tb, int lane) {
    r.q = ldg_stream16(tb + lane * 16);
    if constexpr (FMT == FMT_Q8) {
        r.s.x = __ldg(reinterpret_cast<const unsigned int *>(tb + 512 + (lane >> 2) * 4));
    } else if constexpr (FMT == FMT_Q4) {
        r.s = __ldg(reinterpret_cast<const uint2 *>(tb + 512 + (lane >> 2) * 8));
    } else if constexpr (FMT == FMT_F32) {
        r.m = ldg_stream16(tb + 512 + lane * 16);
        r.l = ldg_stream16(tb + 1024 + lane * 16);
    }
}

// Converted activations in shared memory are fragment-major: for each 32-wide k block, each batch row b and each
// lane quad position t one 16-byte record {x[2t..], x[2t+8..], x[2t+16..], x[2t+24..]} (fp16 pairs), i.e. the
// tensor-core B fragments of the block's two k16 steps for lane (g = b, t), record index (blk * B + b) * 4 + t.  A
// lane reads a Q8 tile's activations with one 16-byte load (64 bytes per quad: one wavefront, no bank conflicts for
// any batch size).  XFrag addresses one lane's records: base = record of block 0, stride = records per block (4 B).
struct XFrag {
    const uint4 *base;   // nullptr: batch row absent (fragments read as zero)
    int stride;
    __device__ __forceinline__ uint4 blk(int i) const { return base ? base[i * stride] : make_uint4(0u, 0u, 0u, 0u); }
    // fragments (b0, b1) of absolute k16 step j
    __device__ __forceinline__ void step(int j, uint32_t &b0, uint32_t &b1) const {
        if (base) {
            const uint2 v = reinterpret_cast<const uint2 *>(base + (j >> 1) * stride)[j & 1];
            b0 = v.x;
            b1 = v.y;
        } else {
            b0 = 0u;
            b1 = 0u;
        }
    }
};

template <int FMT>
__device__ __forceinline__ void compute_tile(const TileRegs &r, int kt, const XFrag &xf, const float *bsum, int t,
                                             float (&acc)[4]) {
    const uint32_t w[4] = {r.q.x, r.q.y, r.q.z, r.q.w};
    if constexpr (FMT == FMT_Q8) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const uint4 xv = xf.blk(kt);
        mma16816(d, q8_pair(w[0], 0x4140u), q8_pair(w[0], 0x4342u), q8_pair(w[1], 0x4140u), q8_pair(w[1], 0x4342u),
                 xv.x, xv.y);
        mma16816(d, q8_pair(w[2], 0x4140u), q8_pair(w[2], 0x4342u), q8_pair(w[3], 0x4140u), q8_pair(w[3], 0x4342u),
                 xv.z, xv.w);
        const float2 S = *reinterpret_cast<const float2 *>(bsum + kt * GEMV_MB + 2 * t);   // batch 2t, 2t+1
        const float2 ds = h2f2(r.s.x);                                                   // rows g, g+8
        acc[0] = fmaf(ds.x, fmaf(-1152.f, S.x, d[0]), acc[0]);
        acc[1] = fmaf(ds.x, fmaf(-1152.f, S.y, d[1]), acc[1]);
        acc[2] = fmaf(ds.y, fmaf(-1152.f, S.x, d[2]), acc[2]);
        acc[3] = fmaf(ds.y, fmaf(-1152.f, S.y, d[3]), acc[3]);
    } else if constexpr (FMT == FMT_Q4) {
        const uint32_t sc[2] = {r.s.x, r.s.y};
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            const uint4 xv = xf.blk(2 * kt + blk);
            mma16816(d, q4_pair<0>(w[2 * blk]), q4_pair<4>(w[2 * blk]), q4_pair<8>(w[2 * blk]), q4_pair<12>(w[2 * blk]),
                     xv.x, xv.y);
            mma16816(d, q4_pair<0>(w[2 * blk + 1]), q4_pair<4>(w[2 * blk + 1]), q4_pair<8>(w[2 * blk + 1]),
                     q4_pair<12>(w[2 * blk + 1]), xv.z, xv.w);
            const float2 S = *reinterpret_cast<const float2 *>(bsum + (2 * kt + blk) * GEMV_MB + 2 * t);
            const float2 ds = h2f2(sc[blk]);
            acc[0] = fmaf(ds.x, fmaf(-1032.f, S.x, d[0]), acc[0]);
            acc[1] = fmaf(ds.x, fmaf(-1032.f, S.y, d[1]), acc[1]);
            acc[2] = fmaf(ds.y, fmaf(-1032.f, S.x, d[2]), acc[2]);
            acc[3] = fmaf(ds.y, fmaf(-1032.f, S.y, d[3]), acc[3]);
        }
    } else if constexpr (FMT == FMT_F32) {   // planes accumulate apart, then hi + 2^-11 mid + 2^-22 lo
        uint32_t b0, b1;
        xf.step(kt, b0, b1);
        float dm[4] = {0.f, 0.f, 0.f, 0.f}, dl[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(acc, w[0], w[1], w[2], w[3], b0, b1);
        mma16816(dm, r.m.x, r.m.y, r.m.z, r.m.w, b0, b1);
        mma16816(dl, r.l.x, r.l.y, r.l.z, r.l.w, b0, b1);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = fmaf(dm[i], F32_MID, fmaf(dl[i], F32_LO, acc[i]));
    } else {
        uint32_t b0, b1;
        xf.step(kt, b0, b1);
        mma16816(acc, w[0], w[1], w[2], w[3], b0, b1);
    }
}

template <int FMT>
__device__ __forceinline__ void prefetch_tiles(TileRegs (&pre)[GEMV_U], const uint8_t *tp, int nkt, int lane) {
#pragma unroll
    for (int u = 0; u < GEMV_U; ++u)
        if (u < nkt) load_tile<FMT>(pre[u], tp + (size_t)u * tile_bytes(FMT), lane);
}

// stream nkt tiles starting at tp (the first GEMV_U already in `pre`), double-buffered
template <int FMT>
__device__ __forceinline__ void stream_tiles(TileRegs (&pre)[GEMV_U], const uint8_t *tp, int kt0, int nkt,
                                             const XFrag &xf, const float *bsum, int lane, float (&acc)[4]) {
    constexpr int TB = tile_bytes(FMT);
    const int t = lane & 3;
    for (int i = 0; i < nkt; i += GEMV_U) {
        TileRegs nxt[GEMV_U];
#pragma unroll
        for (int u = 0; u < GEMV_U; ++u)
            if (i + GEMV_U + u < nkt) load_tile<FMT>(nxt[u], tp + (size_t)(i + GEMV_U + u) * TB, lane);
#pragma unroll
        for (int u = 0; u < GEMV_U; ++u)
            if (i + u < nkt) compute_tile<FMT>(pre[u], kt0 + i + u, xf, bsum, t, acc);
#pragma unroll
        for (int u = 0; u < GEMV_U; ++u) pre[u] = nxt[u];
    }
}

// 2^e for an integer e in [-126, 127], built from its exponent bits (exact)
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

// 8 consecutive fp32 values of a row: two 16-byte loads when the row is made of whole 16-byte-aligned 32-blocks,
// else guarded scalar loads (zero past n).  L2: L1-bypassing loads (activations written by other SMs).
template <bool L2>
__device__ __forceinline__ void load8(const float *p, bool vec, int n, float (&v)[8]) {
    if (vec) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float4 q = L2 ? __ldcg(reinterpret_cast<const float4 *>(p) + j) : reinterpret_cast<const float4 *>(p)[j];
            v[4 * j] = q.x;
            v[4 * j + 1] = q.y;
            v[4 * j + 2] = q.z;
            v[4 * j + 3] = q.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = j < n ? (L2 ? __ldcg(p + j) : p[j]) : 0.f;
    }
}

// default activation loader of gemv_prologue: 8 values of row b at quarter block u, read from a.x
struct XPlain {
    __device__ __forceinline__ void operator()(const GemvArgs &a, int b, int u, bool vec, int n, float (&v)[8]) const {
        load8<true>(a.x + (size_t)(a.b0 + b) * a.x_ld + u * 8, vec, n, v);
    }
};

// Convert the pass's activation rows once per CTA into shared memory: RMSNorm (optional), fp16 with a per-row
// power-of-two scale (largest |x| scaled into (2^13, 2^14]); s_scale[b] receives the scale to undo and, with
// BSUM, bsum[blk * 8 + b] the fp32 sum of converted 32-wide block blk of row b.  Work items are quarter blocks
// (8 values; the four quarters of a block sit in adjacent lanes), so a 1536-wide row keeps 192 threads busy: one
// stats pass and one convert pass.  A thread keeps its first items in registers between the passes -- CACHE of
// them without RMSNorm, one item and its norm weights (in the last cache slot) with it -- so such rows cost one
// round trip to L2.  nw_s: optional shared-memory copy of the norm weights (a.norm_w); xl: the loader of the
// activation values (XPlain reads a.x).
template <bool BSUM, int CACHE = 0, class XL = XPlain>
__device__ inline void gemv_prologue(const GemvArgs &a, uint16_t *xs, float *s_scale, float *s_red, float *bsum,
                                     int nt, const float *nw_s = nullptr, const XL &xl = XL(), int trace_p = -1) {
    const int tid = threadIdx.x, nw = nt / 32;
    const bool norm = a.prologue == PRO_RMSNORM;
    const bool vec = (a.K & 31) == 0 && (a.x_ld & 3) == 0;
    const int nb = (a.K + 31) >> 5, nq = 4 * nb, items = a.B * nq;
    const int xr = gemv_xrows(a.B, a.lo), lo = a.lo;
    const float *nwp = nw_s ? nw_s : a.norm_w;
    const float inv_k = 1.0f / (float)a.K;
    float ss[GEMV_MB], mx[GEMV_MB];
#pragma unroll
    for (int b = 0; b < GEMV_MB; ++b) {
        ss[b] = 0.f;
        mx[b] = 0.f;
    }
    constexpr int NC = CACHE > 1 ? CACHE : 2;
    float vc[NC][8];
    float (&wc)[8] = vc[NC - 1];                // norm weights of the first item (RMSNorm)
    const int ncache = CACHE == 0 ? 0 : (norm ? 1 : CACHE);
    auto stats = [&](int b, const float (&v)[8], const float (&w)[8]) {
        float s2a = 0.f, s2b = 0.f, ma = 0.f, mb = 0.f;   // two chains each
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            s2a = fmaf(v[j], v[j], s2a);
            s2b = fmaf(v[j + 1], v[j + 1], s2b);
            ma = fmaxf(ma, fabsf(norm ? v[j] * w[j] : v[j]));
            mb = fmaxf(mb, fabsf(norm ? v[j + 1] * w[j + 1] : v[j + 1]));
        }
        const float s2 = s2a + s2b, m = fmaxf(ma, mb);
#pragma unroll
        for (int bb = 0; bb < GEMV_MB; ++bb)
            if (bb == b) {
                ss[bb] += s2;
                mx[bb] = fmaxf(mx[bb], m);
            }
    };
#pragma unroll
    for (int k = 0; k < CACHE; ++k) {   // cached items: loads of all of them in flight together
        const int it = tid + k * nt;
        if (k < ncache && it < items) {
            const int b = it / nq, u = it - b * nq, n = a.K - u * 8;
            xl(a, b, u, vec, n, vc[k]);
            if (k == 0 && norm) load8<false>(nwp + u * 8, vec, n, wc);
        }
    }
#pragma unroll
    for (int k = 0; k < CACHE; ++k) {
        const int it = tid + k * nt;
        if (k < ncache && it < items) stats(it / nq, vc[k], wc);
    }
    for (int it = tid + ncache * nt; it < items; it += nt) {
        const int b = it / nq, u = it - b * nq, n = a.K - u * 8;
        float v[8], w[8];
        xl(a, b, u, vec, n, v);
        if (norm) load8<false>(nwp + u * 8, vec, n, w);
        stats(b, v, w);
    }
#pragma unroll
    for (int b = 0; b < GEMV_MB; ++b) {
        if (b < a.B) {   // warp partials: the sum and max shuffle chains interleave
            float S = ss[b], M = mx[b];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                S += __shfl_xor_sync(0xffffffffu, S, o);
                M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            }
            if ((tid & 31) == 0) {
                s_red[b * 8 + (tid >> 5)] = S;
                s_red[64 + b * 8 + (tid >> 5)] = M;
            }
        }
    }
    if (tid == 0) MK_TRACE(trace_p, 5);
    sync_threads(nt);
    if (tid == 0) MK_TRACE(trace_p, 6);
    // every thread derives the multiplier of the rows it converts (same arithmetic everywhere: no second sync);
    // threads b < B also publish the scale the GEMV undoes.  Warp partials are summed in warp order.
    auto row_mul = [&](int b, float &scale) {
        float S = 0.f, Mx = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {   // nt <= 256: at most 8 warp partials, all loads in flight
            if (w < nw) {
                S += s_red[b * 8 + w];
                Mx = fmaxf(Mx, s_red[64 + b * 8 + w]);
            }
        }
        const float inv = norm ? rsqrtf(S * inv_k + a.eps) : 1.0f;
        // largest |x| scaled into (2^13, 2^14]: e = frexp exponent - 14, read from the exponent bits (the row
        // maximum is a finite non-negative float; a zero or subnormal maximum keeps e = 0)
        const int be = (__float_as_int(Mx * inv) >> 23) & 0xff;
        int e = be > 0 ? be - 140 : 0;
        e = e < -126 ? -126 : (e > 126 ? 126 : e);
        scale = pow2i(e);
        return inv * pow2i(-e);   // multiplier applied before rounding to 16 bits
    };
    int cb = -1;          // row whose multiplier cmul holds (threads convert few distinct rows: compute each once)
    float cmul = 0.f;
    if (tid < a.B) {
        float sc;
        cmul = row_mul(tid, sc);
        cb = tid;
        s_scale[tid] = sc;
    }
    uint32_t *xw = reinterpret_cast<uint32_t *>(xs);
    auto convert = [&](bool act, int b, int u, int n, const float (&v)[8], const float (&w)[8]) {
        float bs = 0.f, bsl = 0.f;
        if (act) {
            if (a.feat && blockIdx.x == 0) {
                float *f = a.feat + (size_t)(a.b0 + b) * a.feat_ld + u * 8;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (j < n) f[j] = v[j];
            }
            if (b != cb) {
                float unused;
                cmul = row_mul(b, unused);
                cb = b;
            }
            const float mul = cmul;
            // quarter u of block u / 4 holds the fp16 pairs t = 0..3 of word (u & 3) in the records (block, row, t);
            // the low parts of row b go to record row lo + b
            uint32_t *dst = xw + ((size_t)(u >> 2) * xr + b) * 16 + (u & 3);
            float bs2 = 0.f;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float x0 = (norm ? v[2 * t] * w[2 * t] : v[2 * t]) * mul;
                const float x1 = (norm ? v[2 * t + 1] * w[2 * t + 1] : v[2 * t + 1]) * mul;
                const __half2 hv = __floats2half2_rn(x0, x1);
                const float2 back = __half22float2(hv);
                if (t & 1) bs2 += back.x + back.y;
                else bs += back.x + back.y;
                dst[4 * t] = *reinterpret_cast<const uint32_t *>(&hv);
                if (lo) {
                    const __half2 lv = __floats2half2_rn(x0 - back.x, x1 - back.y);
                    const float2 lb = __half22float2(lv);
                    bsl += lb.x + lb.y;
                    dst[lo * 16 + 4 * t] = *reinterpret_cast<const uint32_t *>(&lv);
                }
            }
            bs += bs2;
        }
        if (BSUM) {   // the four quarters of a block sit in adjacent lanes (warp-uniform call)
            bs += __shfl_xor_sync(0xffffffffu, bs, 1);
            bs += __shfl_xor_sync(0xffffffffu, bs, 2);
            if (act && (u & 3) == 0) bsum[(u >> 2) * GEMV_MB + b] = bs;
            if (lo) {
                bsl += __shfl_xor_sync(0xffffffffu, bsl, 1);
                bsl += __shfl_xor_sync(0xffffffffu, bsl, 2);
                if (act && (u & 3) == 0) bsum[(u >> 2) * GEMV_MB + lo + b] = bsl;
            }
        }
    };
    int base = 0;
#pragma unroll
    for (int k = 0; k < CACHE; ++k) {
        if (k >= ncache || base >= items) break;
        const int it = base + tid;
        const bool act = it < items;
        const int b = act ? it / nq : 0, u = act ? it - b * nq : 0, n = a.K - u * 8;
        convert(act, b, u, n, vc[k], wc);
        base += nt;
    }
    for (; base < items; base += nt) {   // warp-uniform trip count
        const int it = base + tid;
        const bool act = it < items;
        const int b = act ? it / nq : 0, u = act ? it - b * nq : 0, n = a.K - u * 8;
        float v[8], w[8];
        if (act) {
            xl(a, b, u, vec, n, v);
            if (norm) load8<false>(nwp + u * 8, vec, n, w);
        }
        convert(act, b, u, n, v, w);
    }
    // zero the records and block sums of padding blocks (tiles may extend past K).  Absent batch rows (b >= B) have
    // no records: their lanes read row 0, whose tensor-core columns are computed and never read.
    for (int idx = nb * xr * 4 + tid; idx < a.nblk * xr * 4; idx += nt)
        reinterpret_cast<uint4 *>(xs)[idx] = make_uint4(0u, 0u, 0u, 0u);
    if (BSUM)
        for (int idx = nb * GEMV_MB + tid; idx < a.nblk * GEMV_MB; idx += nt) bsum[idx] = 0.f;
    sync_threads(nt);
}

template <int FA, int FB, class Epi>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(GemvArgs a, Epi epi) {
    constexpr bool BSUM = fmt_int(FA) || fmt_int(FB);
    extern __shared__ __align__(16) uint8_t smem[];
    float *s_red = reinterpret_cast<float *>(smem);                  // 136 floats
    float *s_scale = s_red + 136;                                    // GEMV_MB
    float *s_part = s_scale + GEMV_MB;                               // [8 warps][32 lanes][4]
    float *bsum = s_part + 8 * 32 * 4;                               // [nblk][GEMV_MB]
    uint16_t *xs = reinterpret_cast<uint16_t *>(bsum + (BSUM ? a.nblk * GEMV_MB : 0));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rtc = 8 / a.wk;
    const int rs = warp / a.wk, kw = warp % a.wk;
    const int gr = blockIdx.x * rtc + rs;
    const bool active = gr < a.total_rtiles;
    int si = 0, rt = gr, k0 = 0, nkt = 0;
    const uint8_t *tp = nullptr;
    if (active) {
        while (si < a.n_seg - 1 && rt >= a.seg[si].n_rtiles) {
            rt -= a.seg[si].n_rtiles;
            ++si;
        }
        const GemvSeg &sg = a.seg[si];
        const int KT = sg.n_ktiles;
        k0 = (kw * KT) / a.wk;
        nkt = ((kw + 1) * KT) / a.wk - k0;
        tp = sg.tiles + ((size_t)rt * KT + k0) * (si == 0 ? tile_bytes(FA) : tile_bytes(FB));
    }
    // weights do not depend on earlier kernels: start streaming before waiting for them
    TileRegs pre[GEMV_U];
    if (active) {
        if (si == 0) prefetch_tiles<FA>(pre, tp, nkt, lane);
        else prefetch_tiles<FB>(pre, tp, nkt, lane);
    }
    griddep_wait();
    griddep_launch();
    gemv_prologue<BSUM, 5>(a, xs, s_scale, s_red, bsum, blockDim.x);

    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (active) {
        const int g = lane >> 2;
        const XFrag xf{reinterpret_cast<const uint4 *>(xs) + gemv_rec_row(a.B, a.lo, g) * 4 + (lane & 3),
                       4 * gemv_xrows(a.B, a.lo)};
        if (si == 0) stream_tiles<FA>(pre, tp, k0, nkt, xf, bsum, lane, acc);
        else stream_tiles<FB>(pre, tp, k0, nkt, xf, bsum, lane, acc);
    }
    if (a.wk > 1) {
        *reinterpret_cast<float4 *>(&s_part[(warp * 32 + lane) * 4]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        __syncthreads();
        if (kw == 0) {
            acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
            for (int w = 0; w < a.wk; ++w) {
                const float4 p = *reinterpret_cast<const float4 *>(&s_part[((warp + w) * 32 + lane) * 4]);
                acc[0] += p.x;
                acc[1] += p.y;
                acc[2] += p.z;
                acc[3] += p.w;
            }
        }
    }
    if (active && kw == 0) {
        gemv_fold_lo(a.lo, acc);
        const int g = lane >> 2, t = lane & 3;
        const int sg = si + a.seg_base;
        const float ws = a.seg[si].wscale;
        if (2 * t < a.B) {
            const float sc = s_scale[2 * t] * ws;
            epi(sg, rt, g, a.b0 + 2 * t, acc[0] * sc, acc[2] * sc);
        }
        if (2 * t + 1 < a.B) {
            const float sc = s_scale[2 * t + 1] * ws;
            epi(sg, rt, g, a.b0 + 2 * t + 1, acc[1] * sc, acc[3] * sc);
        }
    }
}

inline size_t gemv_smem_bytes(const GemvArgs &a, bool bsum) {
    return (136 + GEMV_MB + 8 * 32 * 4 + (bsum ? a.nblk * GEMV_MB : 0)) * sizeof(float) +
           (size_t)gemv_xrows(a.B, a.lo) * a.nblk * 64;
}

// Host helper: choose the k split so the launch covers the GPU, fill the launch parameters.
void gemv_plan(GemvArgs &a, const int *fmts, int n_sm, int &grid, size_t &smem);

}  // namespace v3g
