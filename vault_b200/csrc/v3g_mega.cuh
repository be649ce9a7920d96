// Persistent decode kernel: every layer of one decode step (and the lm head) in ONE cooperative launch, one CTA
// of 8 warps per SM, phases separated by bounded grid barriers.
//
// Phase list (host-built, per state): for every layer [QKV GEMV, attention, O GEMV, gate/up GEMV, down GEMV], then
// the lm-head GEMV.  A GEMV phase is a flat sequence of T weight tiles (segment by segment, row tile by row tile,
// k tile by k tile -- exactly the order of the tile buffers in HBM), cut into equal contiguous ranges, one per
// warp of the grid.  Every warp therefore streams one contiguous byte range per phase, all SMs stay busy even when
// a matrix has fewer row tiles than the GPU has SMs, and the load is balanced to one tile.
//
// Weight bytes reach shared memory through bulk asynchronous copies (cp.async.bulk, completion on an mbarrier) into
// a per-warp ring of `slots` chunk buffers.  Lane 0 of each warp is that warp's producer: it keeps slots-1 chunks
// in flight ahead of its own consumption, and because weights never change the producer runs ahead ACROSS phase
// boundaries -- while a CTA waits at a grid barrier or runs attention, its copies for the next GEMV phase keep
// HBM busy.  No weight bytes pass through registers until the tile is consumed.
//
// Row tiles that one warp covers completely go straight to the fused epilogue.  A row tile split between warps
// (at most at both ends of a warp's range) is written as a partial to a per-warp slot; the last warp to arrive
// (atomic ticket per row tile) sums the partials in warp order -- deterministic -- and runs the epilogue.
//
// Attention phases spread the (sequence, KV head, key chunk) work items over the CTAs (v3g_attn.cuh).
// This header is included at the end of v3g_step.cu, after the epilogue functors it instantiates.
#pragma once
#include "v3g_attn.cuh"
#include "v3g_gemv.cuh"

namespace v3g {

enum : int { MK_GEMV = 0, MK_ATTN = 1 };
enum : int { MK_EPI_QKV = 0, MK_EPI_RESID = 1, MK_EPI_GATEUP = 2, MK_EPI_STORE = 3 };
constexpr int MK_WARPS = GEMV_THREADS / 32;
constexpr int MK_MAX_SLOTS = 16;
constexpr int MK_SLOT_BYTES = 2304;       // 4 Q4_0 / Q8_0 / BF16 tiles or 1 F32 tile; multiple of 16
constexpr uint32_t MK_WAIT_LIMIT = 1u << 22;

struct MkPhase {
    GemvArgs a;
    int fmts[3];
    int kind, epi, layer;
    int64_t tbase[4];     // flat tile index where segment s starts; tbase[n_seg] = T
    int rbase[3];         // flat row-tile index where segment s starts (ticket counters)
    const float *bq, *bk, *bv;
    float *out;
    int out_ld, out_rows;
};

struct MkCfg {
    int slots;            // ring depth per warp
    int xr_bytes;         // bytes of the activation / attention region at the start of dynamic shared memory
    float *part;          // [n_warps][2][32 lanes][4] split row-tile partials
    uint32_t *cnt;        // [max row tiles] arrival tickets (zero between uses)
};

// ---------------------------------------------------------------------------------------------------------------
// bulk-copy ring primitives
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// expect `bytes` on bar and copy them global -> shared (no multicast: a plain CTA-local bulk copy)
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// bounded wait for the completion of phase `parity` of bar; false when the limit ran out
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t i = 0; i < MK_WAIT_LIMIT; ++i) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// ---------------------------------------------------------------------------------------------------------------
// per-warp chunk stream over all GEMV phases
// ---------------------------------------------------------------------------------------------------------------
struct MkCursor {
    int p;                // phase of the next chunk (n_phases when exhausted)
    int64_t t, t1;        // next flat tile and end of this warp's range in phase p
};

struct MkChunk {
    const uint8_t *src;
    int bytes, n, fmt, si;
    int64_t tl0;          // tile index of the first tile inside segment si
};

// warps that take part in a phase of T tiles (every one of them gets >= 1 tile)
__device__ __forceinline__ int mk_nw(int64_t T, int NW) { return T < (int64_t)NW ? (int)T : NW; }

__device__ __forceinline__ void mk_enter(const MkPhase *ph, int n_phases, int w, int NW, MkCursor &c, int p) {
    for (; p < n_phases; ++p) {
        const MkPhase &P = ph[p];
        if (P.kind != MK_GEMV) continue;
        const int64_t T = P.tbase[P.a.n_seg];
        const int nw = mk_nw(T, NW);
        if (w >= nw) continue;
        c.p = p;
        c.t = (int64_t)w * T / nw;
        c.t1 = (int64_t)(w + 1) * T / nw;
        return;
    }
    c.p = n_phases;
    c.t = c.t1 = 0;
}

// next chunk of the cursor's stream (requires c.p < n_phases); advances the cursor
__device__ __forceinline__ MkChunk mk_next(const MkPhase *ph, int n_phases, int w, int NW, MkCursor &c) {
    const MkPhase &P = ph[c.p];
    int si = 0;
    while (si + 1 < P.a.n_seg && c.t >= P.tbase[si + 1]) ++si;
    MkChunk k;
    k.fmt = P.fmts[si];
    k.si = si;
    const int tb = tile_bytes(k.fmt);
    const int64_t seg_end = P.tbase[si + 1] < c.t1 ? P.tbase[si + 1] : c.t1;
    const int64_t cap = MK_SLOT_BYTES / tb;
    k.n = (int)(seg_end - c.t < cap ? seg_end - c.t : cap);
    k.tl0 = c.t - P.tbase[si];
    k.src = P.a.seg[si].tiles + k.tl0 * tb;
    k.bytes = k.n * tb;
    c.t += k.n;
    if (c.t >= c.t1) mk_enter(ph, n_phases, w, NW, c, c.p + 1);
    return k;
}

// ---------------------------------------------------------------------------------------------------------------
// split row tiles
// ---------------------------------------------------------------------------------------------------------------
// warp (among nw over T tiles) whose range holds flat tile t
__device__ __forceinline__ int mk_owner(int64_t t, int64_t T, int nw) { return (int)(((t + 1) * nw - 1) / T); }

// y = this warp's (scaled) sums of row tile (si, r); complete row tiles go to the epilogue, split ones through the
// partial slots and the ticket of the row tile
template <class Epi>
__device__ __forceinline__ void mk_flush(const MkPhase &P, const Epi &epi, const MkCfg &cfg, int si, int64_t r,
                                         float (&y)[4], int w, int nw, int64_t t0w, int64_t t1w, int lane) {
    const int g = lane >> 2, t = lane & 3, B = P.a.B;
    const int KT = P.a.seg[si].n_ktiles;
    const int64_t rs = P.tbase[si] + r * KT, re = rs + KT;
    if (!(t0w <= rs && re <= t1w)) {
        const int slot = rs <= t0w ? 0 : 1;
        float *pp = cfg.part + (((size_t)w * 2 + slot) * 32 + lane) * 4;
        *reinterpret_cast<float4 *>(pp) = make_float4(y[0], y[1], y[2], y[3]);
        __threadfence();
        __syncwarp();
        const int64_t T = P.tbase[P.a.n_seg];
        const int wa = mk_owner(rs, T, nw), wb = mk_owner(re - 1, T, nw);
        uint32_t *cnt = cfg.cnt + P.rbase[si] + r;
        uint32_t ticket = 0;
        if (lane == 0) ticket = atomicAdd(cnt, 1u);
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket != (uint32_t)(wb - wa)) return;
        __threadfence();
        y[0] = y[1] = y[2] = y[3] = 0.f;
        for (int v = wa; v <= wb; ++v) {
            const int64_t sv = (int64_t)v * T / nw;
            const int sl = (v == wa && sv < rs) ? 1 : 0;
            const float4 q = __ldcg(reinterpret_cast<const float4 *>(cfg.part + (((size_t)v * 2 + sl) * 32 + lane) * 4));
            y[0] += q.x;
            y[1] += q.y;
            y[2] += q.z;
            y[3] += q.w;
        }
        if (lane == 0) *cnt = 0u;
    }
    const int rt = (int)r;
    if (2 * t < B) epi(si, rt, g, 2 * t, y[0], y[2]);
    if (2 * t + 1 < B) epi(si, rt, g, 2 * t + 1, y[1], y[3]);
}

template <int FMT>
__device__ __forceinline__ void mk_tile(const uint8_t *tb, int kt, const uint16_t *xr, const float *bsum, int lane,
                                        float (&acc)[4]) {
    TileRegs r;
    r.q = *reinterpret_cast<const uint4 *>(tb + lane * 16);
    if constexpr (FMT == FMT_Q8) {
        r.s.x = *reinterpret_cast<const uint32_t *>(tb + 512 + (lane >> 2) * 4);
    } else if constexpr (FMT == FMT_Q4) {
        r.s = *reinterpret_cast<const uint2 *>(tb + 512 + (lane >> 2) * 8);
    } else if constexpr (FMT == FMT_F32) {
        r.m = *reinterpret_cast<const uint4 *>(tb + 512 + lane * 16);
        r.l = *reinterpret_cast<const uint4 *>(tb + 1024 + lane * 16);
    }
    compute_tile<FMT>(r, kt, xr, bsum, lane & 3, acc);
}

// per-warp ring state (identical in every lane)
struct MkRing {
    uint8_t *buf;         // slots * MK_SLOT_BYTES
    uint64_t *bar;        // slots mbarriers
    int slots;
    uint32_t issued, consumed;
    MkCursor prod, cons;
    bool dead;            // a wait ran out: stop copying and computing (the step is reported invalid)
    uint32_t d0, d1;      // chunks [d0, d1) were in flight when the ring died
};

__device__ __forceinline__ void mk_issue(MkRing &R, const MkPhase *ph, int n_phases, int w, int NW, int lane) {
    if (R.dead || R.prod.p >= n_phases) return;
    const MkChunk k = mk_next(ph, n_phases, w, NW, R.prod);
    const int s = (int)(R.issued % (uint32_t)R.slots);
    if (lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // our generic reads of the slot come first
        bulk_load(R.buf + (size_t)s * MK_SLOT_BYTES, k.src, (uint32_t)k.bytes, R.bar + s);
    }
    ++R.issued;
}

template <class Epi>
__device__ __forceinline__ void mk_consume(const MkPhase &P, const Epi &epi, MkRing &R, const MkPhase *ph,
                                           int n_phases, int p, int w, int NW, const MkCfg &cfg, const uint16_t *xr,
                                           const float *bsum, const float *s_scale, int *status, int lane) {
    const int64_t T = P.tbase[P.a.n_seg];
    const int nw = mk_nw(T, NW);
    if (w >= nw) return;
    const int64_t t0w = (int64_t)w * T / nw, t1w = (int64_t)(w + 1) * T / nw;
    const int t = lane & 3, B = P.a.B;
    const float sc0 = 2 * t < B ? s_scale[2 * t] : 0.f, sc1 = 2 * t + 1 < B ? s_scale[2 * t + 1] : 0.f;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int cur_si = -1;
    int64_t cur_r = -1;
    while (R.cons.p == p) {
        const MkChunk k = mk_next(ph, n_phases, w, NW, R.cons);
        const int s = (int)(R.consumed % (uint32_t)R.slots);
        const uint32_t par = (R.consumed / (uint32_t)R.slots) & 1u;
        if (!R.dead && !mbar_wait(R.bar + s, par)) {
            R.dead = true;
            R.d0 = R.consumed;
            R.d1 = R.issued;
            if (lane == 0) atomicOr(status, STATUS_TIMEOUT);
        }
        const uint8_t *sb = R.buf + (size_t)s * MK_SLOT_BYTES;
        const int KT = P.a.seg[k.si].n_ktiles;
        int64_t r = k.tl0 / KT;
        int kt = (int)(k.tl0 - r * KT);
        const int tb = tile_bytes(k.fmt);
        for (int i = 0; i < k.n; ++i) {
            if (r != cur_r || k.si != cur_si) {
                if (cur_r >= 0) {
                    const float ws = P.a.seg[cur_si].wscale;
                    float y[4] = {acc[0] * sc0 * ws, acc[1] * sc1 * ws, acc[2] * sc0 * ws, acc[3] * sc1 * ws};
                    mk_flush(P, epi, cfg, cur_si, cur_r, y, w, nw, t0w, t1w, lane);
                }
                cur_r = r;
                cur_si = k.si;
                acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
            }
            if (!R.dead) {
                const uint8_t *tp = sb + (size_t)i * tb;
                switch (k.fmt) {   // warp-uniform
                    case FMT_Q8: mk_tile<FMT_Q8>(tp, kt, xr, bsum, lane, acc); break;
                    case FMT_Q4: mk_tile<FMT_Q4>(tp, kt, xr, bsum, lane, acc); break;
                    case FMT_BF16: mk_tile<FMT_BF16>(tp, kt, xr, bsum, lane, acc); break;
                    case FMT_F16: mk_tile<FMT_F16>(tp, kt, xr, bsum, lane, acc); break;
                    default: mk_tile<FMT_F32>(tp, kt, xr, bsum, lane, acc); break;
                }
            }
            if (++kt == KT) {
                kt = 0;
                ++r;
            }
        }
        ++R.consumed;
        __syncwarp();
        mk_issue(R, ph, n_phases, w, NW, lane);   // refill the slot just read
    }
    if (cur_r >= 0) {
        const float ws = P.a.seg[cur_si].wscale;
        float y[4] = {acc[0] * sc0 * ws, acc[1] * sc1 * ws, acc[2] * sc0 * ws, acc[3] * sc1 * ws};
        mk_flush(P, epi, cfg, cur_si, cur_r, y, w, nw, t0w, t1w, lane);
    }
}

__device__ __forceinline__ void mk_consume_epi(const MkPhase &P, const ModelDev *mp, const StateDev *sp, MkRing &R,
                                               const MkPhase *ph, int n_phases, int p, int w, int NW,
                                               const MkCfg &cfg, const uint16_t *xr, const float *bsum,
                                               const float *s_scale, int *status, int lane) {
    switch (P.epi) {
        case MK_EPI_QKV: {
            EpiQKV e{mp, sp, P.layer, P.bq, P.bk, P.bv};
            mk_consume(P, e, R, ph, n_phases, p, w, NW, cfg, xr, bsum, s_scale, status, lane);
            break;
        }
        case MK_EPI_RESID: {
            EpiResid e{P.out, P.out_ld, P.out_rows};
            mk_consume(P, e, R, ph, n_phases, p, w, NW, cfg, xr, bsum, s_scale, status, lane);
            break;
        }
        case MK_EPI_GATEUP: {
            EpiGateUp e{P.out, P.out_rows};
            mk_consume(P, e, R, ph, n_phases, p, w, NW, cfg, xr, bsum, s_scale, status, lane);
            break;
        }
        default: {
            EpiStore e{P.out, P.out_ld, P.out_rows};
            mk_consume(P, e, R, ph, n_phases, p, w, NW, cfg, xr, bsum, s_scale, status, lane);
            break;
        }
    }
}

// bounded grid barrier: every CTA arrives once per phase on a counter zeroed at the start of the step; a wait
// that exceeds its iteration limit records STATUS_TIMEOUT and returns (the step's results are then invalid)
__device__ __forceinline__ void mk_grid_sync(unsigned int *bar, unsigned int target, int *status) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(bar, 1u);
        unsigned int v = 0;
        for (uint32_t spins = 0;; ++spins) {
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
            if (v >= target) break;
            if (spins > MK_WAIT_LIMIT) {
                atomicOr(status, STATUS_TIMEOUT);
                break;
            }
            __nanosleep(32);
        }
        __threadfence();
    }
    __syncthreads();
}

template <int D>
__global__ void __launch_bounds__(GEMV_THREADS, 1) k_decode(const ModelDev *mp, const StateDev *sp,
                                                            const MkPhase *phases, int n_phases, float scale,
                                                            MkCfg cfg) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int c = blockIdx.x, G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NW = G * MK_WARPS, w = c * MK_WARPS + warp;
    MkRing R;
    R.slots = cfg.slots;
    R.buf = smem + cfg.xr_bytes + (size_t)warp * cfg.slots * MK_SLOT_BYTES;
    R.bar = reinterpret_cast<uint64_t *>(smem + cfg.xr_bytes + (size_t)MK_WARPS * cfg.slots * MK_SLOT_BYTES) +
            warp * cfg.slots;
    R.issued = R.consumed = R.d0 = R.d1 = 0;
    R.dead = false;
    if (lane == 0)
        for (int s = 0; s < R.slots; ++s) mbar_init(R.bar + s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncwarp();
    mk_enter(phases, n_phases, w, NW, R.prod, 0);
    R.cons = R.prod;
    // weights are immutable: start streaming before the previous kernel's results are needed
    for (int s = 0; s < R.slots; ++s) mk_issue(R, phases, n_phases, w, NW, lane);
    griddep_wait();
    const StateDev &st = *sp;
    int *status = &st.step->status;
    const int64_t pos = __ldcg(&st.step->pos);
    float *s_red = reinterpret_cast<float *>(smem);
    float *s_scale = s_red + 136;
    float *bsum = s_scale + GEMV_MB;
    for (int p = 0; p < n_phases; ++p) {
        const MkPhase &P = phases[p];
        if (P.kind == MK_ATTN) {
            const int n_kv = mp->G, ms = st.max_splits;
            const int n_items = st.B * n_kv * ms;
            for (int i = c; i < n_items; i += G) {
                const int split = i % ms, g = (i / ms) % n_kv, b = i / (ms * n_kv);
                attn_item<D>(*mp, st, P.layer, scale, split, g, b, pos, *reinterpret_cast<AttnSmem<D> *>(smem));
            }
        } else {
            bool bs = false;
            for (int i = 0; i < P.a.n_seg; ++i) bs = bs || fmt_int(P.fmts[i]);
            uint16_t *xs = reinterpret_cast<uint16_t *>(bsum + (bs ? P.a.nblk * GEMV_MB : 0));
            if (bs) gemv_prologue<true>(P.a, xs, s_scale, s_red, bsum);
            else gemv_prologue<false>(P.a, xs, s_scale, s_red, bsum);
            const int g = lane >> 2;
            const uint16_t *xr = g < P.a.B ? xs + g * P.a.kpx : nullptr;
            mk_consume_epi(P, mp, sp, R, phases, n_phases, p, w, NW, cfg, xr, bsum, s_scale, status, lane);
        }
        if (p + 1 < n_phases) mk_grid_sync(st.bar, (unsigned int)(p + 1) * (unsigned int)G, status);
    }
    // every issued chunk was consumed unless a wait ran out; then wait (bounded) for what was still in flight
    for (uint32_t q = R.d0; q < R.d1; ++q) mbar_wait(R.bar + q % (uint32_t)R.slots, (q / (uint32_t)R.slots) & 1u);
    griddep_launch();
}

}  // namespace v3g
