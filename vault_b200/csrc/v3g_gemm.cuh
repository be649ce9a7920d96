// Tensor-core (tcgen05) GEMM over the engine's quantized weight tiles, for work with many tokens per weight row:
// chunked prefill and batched decode.
//
//   Y[token, row] = epilogue( sum_k W[row, k] * X[token, k] )
//
// W is one or more re-tiled weight matrices of the same K (v3g.cuh tile formats; several matrices are stacked row
// tile after row tile, e.g. q | k | v), X the activations of n_tok tokens as fp16 rows [n_tok, K] with a per-token
// power-of-two scale (k_tc_prep writes them).  The weights are the MMA's A operand (M = 128 rows = 8 row tiles per
// CTA tile), the tokens its B operand (N = bn tokens, 16..256), the fp32 accumulator lives in tensor memory.
//
// One persistent CTA per SM walks the (128-row, bn-token) output tiles with warp-specialised roles:
//   warp 0      producer: for every 64-wide k stage, one TMA box of the weights (the segment's row-tile buffer viewed
//               as [row tiles] x [stored bytes / 8] 8-byte elements; box = the CTA tile's 8 row tiles x one stage's
//               stored bytes) and one TMA box of the bn x 64 fp16 activations (128-byte swizzle), both completing on
//               the stage's `full` mbarrier.  A CTA tile that straddles two stacked matrices falls back to one bulk
//               copy per row tile (lanes 0-7) plus the activation box (lane 8);
//   warps 2-9   converters (one per row tile): dequantize the stage's weight bytes into the A operand (fp16, K-major, 128-byte
//               swizzle) -- Q8_0 codes and Q4_0 nibbles times their fp16 block scale (times a per-matrix power of two
//               that keeps small scales out of the fp16 subnormal range), 16-bit tiles copied -- then fence the
//               writes to the async proxy and arrive on `conv`;
//   warp 1      allocates 512 TMEM columns (two accumulator buffers) and issues, from one thread, the four
//               tcgen05.mma (K = 16 each) of every stage, committing the stage's `empty` barrier (its buffers may be
//               refilled) and, after a tile's last stage, the buffer's `acc_full` barrier;
//   warps 10-13 epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes 32 (w % 4) ..), scale each token's
//               column by its activation scale and the matrix's weight scale, and hand (row g, row g+8) pairs of a
//               16-row tile to the fused epilogue -- the partners of the RoPE / gate-up row order sit 8 lanes apart;
//               then release the accumulator buffer (`acc_empty`).
// An epilogue functor provides
//   chunk(seg, rt, g, tok0, nv, y0[8], y1[8])     tokens tok0 .. tok0 + nv - 1 of rows (g, g + 8) of row tile rt
//   operator()(seg, rt, g, tok, y0, y1)           one token (the split-K reduction)
// chunk() issues its global reads for all nv tokens before its first write: the reads cannot be reordered across
// the writes by the compiler (they may alias), so a per-token loop would pay one L2 round trip per token.
// Few output tiles (small batches) split K over up to 16 CTAs per tile: each split writes an fp32 partial, and a
// second kernel over all (row pair, token) outputs adds the splits in order (deterministic) and runs the epilogue.
// Every wait is bounded: a wait that runs out records status bit 4 (timeout) and its role stops.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>

#include "v3g.cuh"
#include "v3g_tc.cuh"

namespace v3g {

constexpr int TC_BM = 128;            // weight rows per CTA tile (8 row tiles)
constexpr int TC_BK = 64;             // k per stage (one 128-byte swizzled row)
constexpr int TC_CONV_WARPS = 8;      // one per row tile of the CTA tile
constexpr int TC_THREADS = 32 * (2 + TC_CONV_WARPS + 4);   // producer, MMA, converters, 4 epilogue warps
constexpr int TC_EPI_CHUNK = 8;   // tokens per epilogue chunk() call
constexpr int TC_MAX_STAGES = 8;
constexpr int TC_TMEM_COLS = 512;
// split-K workspace of a state: tiles x splits <= SMs, so 256 SMs x 256 tokens x 128 rows of fp32 always suffice
constexpr size_t TC_SPLITK_WS_BYTES = (size_t)256 * 256 * 128 * 4;

struct TcSeg {
    const uint8_t *tiles;
    int n_rtiles, n_ktiles, fmt;
    float wscale;     // output multiplier of this matrix (16-bit tiles: MatW::wscale; integer formats: 2^-dexp)
    int dexp;         // integer formats: the converter multiplies block scales by 2^dexp
};

struct TcArgs {
    TcSeg seg[3];
    int n_seg;
    int rbase[4];     // flat row tile where segment s starts; rbase[n_seg] = total row tiles
    int m_tiles;      // ceil(total row tiles / 8)
    int K, kstages;   // logical K, ceil(K / 64)
    int n_tok, bn, n_tiles;
    int stages;
    int seg_base;          // segment index the epilogue receives for seg[0]
    int splits;            // k splits per output tile (1: no split)
    float *ws;             // split-K partials [tile][split][bn][128] (splits > 1)

    const float *xscale;   // [n_tok] multiplier undoing each token's activation scale
    int *status;           // sticky error word (bit 4: a bounded wait ran out)
    // shared-memory layout (bytes from the 1024-aligned base)
    int a_off, x_off, raw_off, bar_off, stage_a, stage_x, stage_raw;
    int raw_row;          // stored weight bytes of one row tile per stage (Q8_0: 2 x 544, Q4_0: 576, 16-bit: 4 x 512)
    int w_tma;            // 1: every CTA tile lies in one segment and its weights arrive by one TMA box per stage
};

// weight tensor maps of the segments: a segment's row-tile buffer viewed as a [row tiles] x [stored bytes / 8] array
// of 8-byte elements; one box = 8 row tiles x one stage's stored bytes (rows land tc_stage_raw_bytes(fmt) apart)
struct alignas(64) TcMaps {
    CUtensorMap w[3];
};

__host__ __device__ inline int tc_stage_raw_bytes(int fmt) {
    return fmt == FMT_Q8 ? 2 * 544 : (fmt == FMT_Q4 ? 576 : 4 * 512);
}

// ---------------------------------------------------------------------------------------------- weight converters
// byte offset inside a 128-row x 64-k SW128 operand tile of the 4-byte pair at (row p, k = 8 j + 2 t)
__device__ __forceinline__ uint32_t sw128_pair_off(int p, int j, int t) {
    return (uint32_t)(p * 128 + ((j ^ (p & 7)) << 4) + 4 * t);
}

// fp16x2 {1152 + q0, 1152 + q1} (biased codes through the byte-permute of v3g_gemv.cuh) -> {q0 d, q1 d} rounded
__device__ __forceinline__ uint32_t q8_dequant_pair(uint32_t w, uint32_t sel, __half2 d2) {
    const uint32_t v = __byte_perm(w, 0x64646464u, sel);
    __half2 h = *reinterpret_cast<const __half2 *>(&v);
    h = __hsub2(h, __float2half2_rn(1152.f));
    h = __hmul2(h, d2);
    return *reinterpret_cast<const uint32_t *>(&h);
}
template <int SH>
__device__ __forceinline__ uint32_t q4_dequant_pair(uint32_t w, __half2 d2) {
    const uint32_t v = ((w >> SH) & 0x000F000Fu) | 0x64006400u;   // {1024 + n}
    __half2 h = *reinterpret_cast<const __half2 *>(&v);
    h = __hsub2(h, __float2half2_rn(1032.f));                      // n - 8, exact
    h = __hmul2(h, d2);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// One stored tile (this lane's 16 bytes at `tb`) into the A operand at row tile rl (0..7), k offset k0 in the
// stage (0, 16, 32 or 48 for 16-bit tiles; 0 or 32 for Q8_0; 0 for Q4_0).  tb == nullptr writes zeros (k past K).
template <int FMT>
__device__ __forceinline__ void tc_convert_tile(uint8_t *A, const uint8_t *tb, int rl, int k0, int lane, __half2 dmul) {
    const int g = lane >> 2, t = lane & 3;
    const int p0 = 16 * rl + g, p1 = p0 + 8;
    if constexpr (FMT == FMT_Q8) {
        uint4 q = make_uint4(0u, 0u, 0u, 0u);
        __half2 dg = __float2half2_rn(0.f), dh = dg;
        if (tb) {
            q = *reinterpret_cast<const uint4 *>(tb + lane * 16);
            const uint32_t sw = *reinterpret_cast<const uint32_t *>(tb + 512 + g * 4);
            const __half2 s2 = __hmul2(*reinterpret_cast<const __half2 *>(&sw), dmul);   // {d(row g), d(row g+8)}
            dg = __low2half2(s2);
            dh = __high2half2(s2);
        }
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        // lane bytes: [s (k16 step)][reg][half]; reg bit 0 = row g+8, bit 1 = k + 8
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const int j0 = (k0 >> 3) + 2 * s;
            *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p0, j0, t)) = q8_dequant_pair(w[2 * s], 0x4140u, dg);
            *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p1, j0, t)) = q8_dequant_pair(w[2 * s], 0x4342u, dh);
            *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p0, j0 + 1, t)) = q8_dequant_pair(w[2 * s + 1], 0x4140u, dg);
            *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p1, j0 + 1, t)) = q8_dequant_pair(w[2 * s + 1], 0x4342u, dh);
        }
    } else if constexpr (FMT == FMT_Q4) {
        uint4 q = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
        __half2 dg[2], dh[2];
        dg[0] = dg[1] = dh[0] = dh[1] = __float2half2_rn(0.f);
        if (tb) {
            q = *reinterpret_cast<const uint4 *>(tb + lane * 16);
            const uint2 sw = *reinterpret_cast<const uint2 *>(tb + 512 + g * 8);
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const uint32_t wb = b ? sw.y : sw.x;
                const __half2 s2 = __hmul2(*reinterpret_cast<const __half2 *>(&wb), dmul);
                dg[b] = __low2half2(s2);
                dh[b] = __high2half2(s2);
            }
        }
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        // word s = k16 step s; nibble (reg, half) at bit 4 reg + 16 half; block = s >> 1
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const int j0 = 2 * s, b = s >> 1;
            *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p0, j0, t)) = q4_dequant_pair<0>(w[s], dg[b]);
            *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p1, j0, t)) = q4_dequant_pair<4>(w[s], dh[b]);
            *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p0, j0 + 1, t)) = q4_dequant_pair<8>(w[s], dg[b]);
            *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p1, j0 + 1, t)) = q4_dequant_pair<12>(w[s], dh[b]);
        }
    } else {   // 16-bit tiles (fp16 values, already scaled): copy the fragment pairs
        uint4 q = make_uint4(0u, 0u, 0u, 0u);
        if (tb) q = *reinterpret_cast<const uint4 *>(tb + lane * 16);
        const int j0 = k0 >> 3;
        *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p0, j0, t)) = q.x;
        *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p1, j0, t)) = q.y;
        *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p0, j0 + 1, t)) = q.z;
        *reinterpret_cast<uint32_t *>(A + sw128_pair_off(p1, j0 + 1, t)) = q.w;
    }
}

// segment and segment-local row tile of flat row tile R
__device__ __forceinline__ int tc_seg_of(const TcArgs &a, int R, int &rt) {
    int s = 0;
    while (s + 1 < a.n_seg && R >= a.rbase[s + 1]) ++s;
    rt = R - a.rbase[s];
    return s;
}

template <int FA, int FB>
__device__ __forceinline__ void tc_convert_row_tile(const TcArgs &a, uint8_t *A, const uint8_t *raw_row, int R, int rl,
                                                    int ks, int lane) {
    int rt;
    const int si = tc_seg_of(a, R, rt);
    const TcSeg &sg = a.seg[si];
    const __half2 dmul = __float2half2_rn(__int_as_float((sg.dexp + 127) << 23));
    const int fmt = FA == FB ? FA : sg.fmt;
    const int tk = tile_k(fmt), per = TC_BK / tk, kt0 = ks * per;
    const int tb = tile_bytes(fmt);
    for (int i = 0; i < per; ++i) {
        const uint8_t *src = kt0 + i < sg.n_ktiles ? raw_row + i * tb : nullptr;
        if (fmt == FA) tc_convert_tile<FA>(A, src, rl, i * tk, lane, dmul);
        else tc_convert_tile<FB>(A, src, rl, i * tk, lane, dmul);
    }
}

// --------------------------------------------------------------------------------------------------- the kernel
// work item w -> output tile (mt, nt) and k-split sp (k stages [ks0, ks1))
__device__ __forceinline__ void tc_work(const TcArgs &a, int w, int &mt, int &nt, int &sp, int &ks0, int &ks1) {
    const int tile = w / a.splits;
    sp = w - tile * a.splits;
    mt = tile / a.n_tiles;
    nt = tile - mt * a.n_tiles;
    ks0 = (int)((int64_t)sp * a.kstages / a.splits);
    ks1 = (int)((int64_t)(sp + 1) * a.kstages / a.splits);
}

template <int FA, int FB, class Epi>
__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_tc(const __grid_constant__ TcArgs a,
                                                          const __grid_constant__ CUtensorMap xmap,
                                                          const __grid_constant__ TcMaps wm, Epi epi) {
    extern __shared__ uint8_t smem_raw[];
    // operand tiles need 1024-byte aligned shared-memory addresses (the swizzle reads address bits 7-9)
    uint8_t *smem = smem_raw + ((1024u - (tc::smem_addr(smem_raw) & 1023u)) & 1023u);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.stages;
    const uint32_t bars = tc::smem_addr(smem + a.bar_off);
    // barrier slots: full[S], conv[S], empty[S], acc_full[2], acc_empty[2]; then the TMEM address and a flag word
    auto FULL = [&](int s) { return bars + 8u * s; };
    auto CONV = [&](int s) { return bars + 8u * (S + s); };
    auto EMPTY = [&](int s) { return bars + 8u * (2 * S + s); };
    auto ACCF = [&](int b) { return bars + 8u * (3 * S + b); };
    auto ACCE = [&](int b) { return bars + 8u * (3 * S + 2 + b); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + a.bar_off + 8 * (3 * S + 4));
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(FULL(s), 1);
            tc::mbar_init(CONV(s), TC_CONV_WARPS);
            tc::mbar_init(EMPTY(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(ACCF(b), 1);
            tc::mbar_init(ACCE(b), 4);
        }
        tc::mbar_fence_init();
    }
    if (warp == 1) tc::tmem_alloc(tc::smem_addr(tmem_slot), TC_TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_work = a.m_tiles * a.n_tiles * a.splits;
    const int total_rt = a.rbase[a.n_seg];

    if (warp == 0) {   // ------------------------------------------------------------------------- producer
        // lane r < 8 streams row tile r of the CTA tile (its stored k tiles are contiguous); lane 8 the activations
        if (lane == 0) {
            tc::prefetch_tmap(&xmap);
            if (a.w_tma)
                for (int i = 0; i < a.n_seg; ++i) tc::prefetch_tmap(&wm.w[i]);
        }
        const uint64_t pol = tc::l2_evict_first_policy();
        int it = 0;
        bool ok = true;
        for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
            int mt, nt, sp, ks0, ks1;
            tc_work(a, w, mt, nt, sp, ks0, ks1);
            const uint8_t *base = nullptr;
            int tb = 0, nkt = 0, per = 0;
            const int R = mt * 8 + lane;
            if (lane < 8 && R < total_rt) {
                int rt;
                const TcSeg &sg = a.seg[tc_seg_of(a, R, rt)];
                tb = tile_bytes(sg.fmt);
                nkt = sg.n_ktiles;
                per = TC_BK / tile_k(sg.fmt);
                base = sg.tiles + (size_t)rt * nkt * tb;
            }
            int wseg = 0, wrt = 0;   // TMA mode: the CTA tile's segment and its first row tile there
            if (a.w_tma && mt * 8 < total_rt) wseg = tc_seg_of(a, mt * 8, wrt);
            const int wtb = tile_bytes(a.seg[wseg].fmt), wper = TC_BK / tile_k(a.seg[wseg].fmt);
            for (int ks = ks0; ks < ks1; ++ks, ++it) {
                const int s = it % S;
                if (it >= S && !tc::mbar_wait(EMPTY(s), ((it / S) - 1) & 1)) {
                    ok = false;
                    break;
                }
                if (a.w_tma) {   // two copies per stage: the weight box (8 row tiles) and the activation box
                    if (lane == 0) {
                        tc::mbar_expect_tx(FULL(s), (uint32_t)(8 * wper * wtb + a.bn * TC_BK * 2));
                        tc::tma_load_2d_hint(tc::smem_addr(smem + a.raw_off + s * a.stage_raw), &wm.w[wseg],
                                             ks * wper * wtb / 8, wrt, FULL(s), pol);
                        tc::tma_load_2d(tc::smem_addr(smem + a.x_off + s * a.stage_x), &xmap, ks * TC_BK, nt * a.bn,
                                        FULL(s));
                    }
                    continue;
                }
                const int kt0 = ks * per;
                const int n = base ? max(0, min(per, nkt - kt0)) : 0;
                int bytes = n * tb;
#pragma unroll
                for (int o = 4; o > 0; o >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, o);   // lanes 0..7
                if (lane == 0) tc::mbar_expect_tx(FULL(s), (uint32_t)(bytes + a.bn * TC_BK * 2));
                __syncwarp();
                if (n > 0)
                    tc::bulk_g2s(tc::smem_addr(smem + a.raw_off + s * a.stage_raw + lane * a.raw_row),
                                 base + (size_t)kt0 * tb, (uint32_t)(n * tb), FULL(s), pol);
                if (lane == 8)
                    tc::tma_load_2d(tc::smem_addr(smem + a.x_off + s * a.stage_x), &xmap, ks * TC_BK, nt * a.bn,
                                    FULL(s));
            }
        }
        if (!ok && lane == 0) atomicOr(a.status, 4);
    } else if (warp == 1) {   // ------------------------------------------------------------------ MMA issuer
        const uint32_t idesc = tc::idesc_f16(TC_BM, a.bn);
        int it = 0, tcount = 0;
        bool ok = true;
        for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x, ++tcount) {
            int mt, nt, sp, ks0, ks1;
            tc_work(a, w, mt, nt, sp, ks0, ks1);
            const int buf = tcount & 1;
            if (tcount >= 2 && !tc::mbar_wait(ACCE(buf), ((tcount >> 1) - 1) & 1)) {
                ok = false;
                break;
            }
            tc::tc_fence_after();
            const uint32_t d = tmem + (uint32_t)(buf * a.bn);
            for (int ks = ks0; ks < ks1; ++ks, ++it) {
                const int s = it % S;
                if (!tc::mbar_wait(CONV(s), (it / S) & 1)) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                if (lane == 0) {
                    const uint32_t sa = tc::smem_addr(smem + a.a_off + s * a.stage_a);
                    const uint32_t sx = tc::smem_addr(smem + a.x_off + s * a.stage_x);
#pragma unroll
                    for (int k16 = 0; k16 < TC_BK / 16; ++k16)
                        tc::mma_f16(d, tc::sw128_desc(sa + 32 * k16), tc::sw128_desc(sx + 32 * k16), idesc,
                                    (ks > ks0 || k16 > 0) ? 1u : 0u);
                    tc::mma_commit(EMPTY(s));
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) tc::mma_commit(ACCF(buf));
            __syncwarp();
        }
        if (!ok && lane == 0) atomicOr(a.status, 4);
    } else if (warp < 2 + TC_CONV_WARPS) {   // ---------------------------------------------------- converters
        const int rl = warp - 2;              // the row tile this warp converts
        int it = 0;
        bool ok = true;
        for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
            int mt, nt, sp, ks0, ks1;
            tc_work(a, w, mt, nt, sp, ks0, ks1);
            const int R = mt * 8 + rl;
            int row_bytes = a.raw_row;   // TMA mode: rows of the box sit one stage of the tile's format apart
            if (a.w_tma && R < total_rt) {
                int rt_unused;
                row_bytes = tc_stage_raw_bytes(a.seg[tc_seg_of(a, R, rt_unused)].fmt);
            }
            for (int ks = ks0; ks < ks1; ++ks, ++it) {
                const int s = it % S;
                if (!tc::mbar_wait(FULL(s), (it / S) & 1)) {
                    ok = false;
                    break;
                }
                if (R < total_rt)
                    tc_convert_row_tile<FA, FB>(a, smem + a.a_off + s * a.stage_a,
                                                smem + a.raw_off + s * a.stage_raw + rl * row_bytes, R, rl, ks, lane);
                tc::fence_proxy_async();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(CONV(s));
            }
        }
        if (!ok && lane == 0) atomicOr(a.status, 4);
    } else {   // ------------------------------------------------------------------------------------- epilogue
        const int q = warp & 3;                       // TMEM lane quarter this warp may read
        const int row = 32 * q + lane;                // weight row inside the CTA tile
        int tcount = 0;
        bool ok = true;
        for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x, ++tcount) {
            int mt, nt, sp, ks0, ks1;
            tc_work(a, w, mt, nt, sp, ks0, ks1);
            const int buf = tcount & 1;
            if (!tc::mbar_wait(ACCF(buf), (tcount >> 1) & 1)) {
                ok = false;
                break;
            }
            tc::tc_fence_after();
            const int R = mt * 8 + (row >> 4), tr = row & 15;
            const int g = tr & 7, hi = tr >> 3;   // lanes g and g + 8 hold the row pair (g, g + 8)
            const bool live = R < total_rt;
            int rt = 0, si = 0;
            if (live) si = tc_seg_of(a, R, rt);
            const float ws = a.seg[si].wscale;
            const int tile = mt * a.n_tiles + nt;
            if (a.splits == 1) {
                // per 16 token columns, lane g takes tokens 0-7 and lane g + 8 tokens 8-15 of the row pair
                // (g, g + 8): each swaps the other half with its partner, and the epilogue gets 8 tokens at once,
                // so that it can issue all of its global reads before its first write
                for (int c0 = 0; c0 < a.bn; c0 += 16) {
                    uint32_t v[16];
                    tc::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * a.bn + c0), v);
                    tc::tmem_ld_wait();
                    const int tok0 = nt * a.bn + c0 + 8 * hi;
                    const int nv = min(TC_EPI_CHUNK, a.n_tok - tok0);
                    float y0[TC_EPI_CHUNK], y1[TC_EPI_CHUNK];
#pragma unroll
                    for (int j = 0; j < TC_EPI_CHUNK; ++j) {
                        const float lo_v = __uint_as_float(v[j]), hi_v = __uint_as_float(v[j + 8]);
                        const float keep = hi ? hi_v : lo_v;
                        const float recv = __shfl_xor_sync(0xffffffffu, hi ? lo_v : hi_v, 8);
                        const float sc = j < nv ? __ldg(a.xscale + tok0 + j) * ws : 0.f;
                        y0[j] = (hi ? recv : keep) * sc;
                        y1[j] = (hi ? keep : recv) * sc;
                    }
                    if (live && nv > 0) epi.chunk(si + a.seg_base, rt, g, tok0, nv, y0, y1);
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(ACCE(buf));
                continue;
            }
            // split-K: this split's fp32 partial goes to the workspace ([tile][split][bn columns][128 rows], so a
            // warp writes 128 contiguous bytes per column); k_tc_splitk_reduce adds the splits in order and runs
            // the epilogue
            float *part = a.ws + ((size_t)tile * a.splits + sp) * TC_BM * a.bn + row;
            for (int c0 = 0; c0 < a.bn; c0 += 16) {
                uint32_t v[16];
                tc::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * a.bn + c0), v);
                tc::tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j) __stcg(part + (size_t)(c0 + j) * TC_BM, __uint_as_float(v[j]));
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(ACCE(buf));   // the accumulator buffer is free again
        }
        if (!ok && lane == 0) atomicOr(a.status, 4);
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TC_TMEM_COLS);
    }
}

// split-K reduction: one thread per (output tile, token column, row pair (g, g+8) of a 16-row tile), the row pairs
// fastest so that a warp reads and writes contiguous rows: the splits' partials summed in split order (deterministic),
// then the fused epilogue of the pair
template <class Epi>
__global__ void __launch_bounds__(256) k_tc_splitk_reduce(const __grid_constant__ TcArgs a, Epi epi) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t n = (int64_t)a.m_tiles * a.n_tiles * 64 * a.bn;
    if (idx >= n) return;
    const int pair = (int)(idx & 63);
    const int c = (int)((idx >> 6) % a.bn);
    const int tile = (int)(idx / ((int64_t)a.bn * 64));
    const int mt = tile / a.n_tiles, nt = tile - mt * a.n_tiles;
    const int rl = pair >> 3, g = pair & 7;
    const int R = mt * 8 + rl, tok = nt * a.bn + c;
    if (R >= a.rbase[a.n_seg] || tok >= a.n_tok) return;
    const int r0 = 16 * rl + g;
    const float *p = a.ws + (size_t)tile * a.splits * TC_BM * a.bn + (size_t)c * TC_BM + r0;
    const size_t split_stride = (size_t)TC_BM * a.bn;
    float y0 = 0.f, y1 = 0.f;
    for (int k = 0; k < a.splits; ++k) {
        y0 += __ldcg(p + k * split_stride);
        y1 += __ldcg(p + k * split_stride + 8);
    }
    int rt;
    const int si = tc_seg_of(a, R, rt);
    const float sc = __ldg(a.xscale + tok) * a.seg[si].wscale;
    epi(si + a.seg_base, rt, g, tok, y0 * sc, y1 * sc);
}

// ------------------------------------------------------------------------------------------------ host launch
// One GEMM launch: the kernel arguments, the activation tensor map and the weight-format pair of the kernel.
struct TcLaunch {
    TcArgs a;
    CUtensorMap xmap;
    TcMaps wm;
    int fa, fb;
    int grid;
    size_t smem;
};

// Fill `L` for the stacked matrices mats[0..n) (all of one K) against n_tok fp16 activation rows x16 (row stride
// ldx elements, ldx >= K, 16-byte aligned rows).  Returns cudaErrorNotSupported when a matrix is not in a
// tensor-core format (F32 tiles) or the formats do not form one kernel's pair (the caller then splits by matrix).
struct TcSplitWs {
    float *ws = nullptr;     // split-K partials
    size_t ws_bytes = 0;
};
cudaError_t tc_setup(TcLaunch &L, const MatW *const *mats, int n, const __half *x16, int ldx, const float *xscale,
                     int n_tok, int *status, int n_sm, const TcSplitWs *sk = nullptr);

template <int FA, int FB, class Epi>
cudaError_t tc_launch_t(const TcLaunch &L, const Epi &epi, cudaStream_t st) {
    static bool attr_set = false;   // large dynamic shared memory: set once per instantiation (outside capture)
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<FA, FB, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             227 * 1024);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    k_gemm_tc<FA, FB, Epi><<<L.grid, TC_THREADS, L.smem, st>>>(L.a, L.xmap, L.wm, epi);
    if (L.a.splits > 1) {
        const int64_t n = (int64_t)L.a.m_tiles * L.a.n_tiles * 64 * L.a.bn;
        k_tc_splitk_reduce<Epi><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(L.a, epi);
    }
    return cudaGetLastError();
}

template <class Epi>
cudaError_t tc_launch(const TcLaunch &L, const Epi &epi, cudaStream_t st) {
    if (L.fa == FMT_Q8 && L.fb == FMT_Q8) return tc_launch_t<FMT_Q8, FMT_Q8>(L, epi, st);
    if (L.fa == FMT_Q4 && L.fb == FMT_Q8) return tc_launch_t<FMT_Q4, FMT_Q8>(L, epi, st);
    if (L.fa == FMT_Q4 && L.fb == FMT_Q4) return tc_launch_t<FMT_Q4, FMT_Q4>(L, epi, st);
    if (L.fa == FMT_BF16 && L.fb == FMT_BF16) return tc_launch_t<FMT_BF16, FMT_BF16>(L, epi, st);
    if (L.fa == FMT_F16 && L.fb == FMT_F16) return tc_launch_t<FMT_F16, FMT_F16>(L, epi, st);
    return cudaErrorNotSupported;
}

// Stacked matrices through the tensor-core GEMM: one launch when the formats form a kernel pair, else one launch
// per matrix (the epilogue still receives the matrix index as its segment).
template <class Epi>
cudaError_t tc_gemm(const MatW *const *mats, int n, const __half *x16, int ldx, const float *xscale, int n_tok,
                    int *status, int n_sm, const Epi &epi, cudaStream_t st, const TcSplitWs *sk = nullptr) {
    TcLaunch L;
    cudaError_t e = tc_setup(L, mats, n, x16, ldx, xscale, n_tok, status, n_sm, sk);
    if (e == cudaSuccess) return tc_launch(L, epi, st);
    if (e != cudaErrorNotSupported || n == 1) return e;
    for (int i = 0; i < n; ++i) {
        e = tc_setup(L, mats + i, 1, x16, ldx, xscale, n_tok, status, n_sm, sk);
        if (e != cudaSuccess) return e;
        L.a.seg_base = i;
        e = tc_launch(L, epi, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// ------------------------------------------------------------------------------------------ activation operand
// Row r of x (fp32, stride ld_x; RMSNorm with gain norm_w when it is non-null) -> fp16 row of out (stride ldo,
// zero-padded to ldo) scaled by a power of two that puts the row's largest |value| into (2^13, 2^14]; xscale[r]
// receives the multiplier that undoes it.  One CTA per row.
__global__ void k_tc_prep(const float *x, int64_t ld_x, int K, const float *norm_w, float eps, __half *out, int ldo,
                          float *xscale);
// rows 0..n-1 of x through k_tc_prep
cudaError_t tc_prep(const float *x, int64_t ld_x, int n, int K, const float *norm_w, float eps, __half *out, int ldo,
                    float *xscale, cudaStream_t st);

}  // namespace v3g
