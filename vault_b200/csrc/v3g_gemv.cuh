// Decode GEMV: y[b, :] = W x[b, :] for up to 8 batch rows per pass, weights streamed once from HBM.
//
// Each CTA (8 warps) owns 8/WK row tiles; the WK warps of a row tile split its k tiles, so every matrix shape is
// spread over >= ~148 CTAs.  The activation rows are normalised (optional RMSNorm) and converted once per CTA into
// shared memory as fp16 (with a per-row power-of-two scale that keeps them in fp16 range) or bf16.  Weight tiles
// are read with 16-byte streaming loads straight into mma.sync B fragments: int8 / nibble codes become exact fp16
// integers with one byte-permute (or mask) and one packed subtract, the tensor core multiplies them with the
// activations and accumulates in fp32, and each 32-wide block sum is scaled by its fp16 scale in fp32.  Partial
// sums of the WK warps are reduced in shared memory in a fixed order (deterministic), then a fused epilogue
// consumes (y[row 2t], y[row 2t+1]) pairs in registers.
#pragma once
#include "v3g.cuh"

namespace v3g {

constexpr int PRO_PLAIN = 0, PRO_RMSNORM = 1;

struct GemvSeg {
    const uint8_t *tiles;
    int fmt, n_rtiles, n_ktiles;
};

struct GemvArgs {
    GemvSeg seg[3];
    int n_seg;
    int total_rtiles;
    int K;            // logical K
    int kpx;          // smem row pitch of the converted activations (elements)
    int B;            // batch rows in this pass (<= GEMV_MB)
    int b0;           // first batch row of this pass
    int wk;           // warps per row tile
    const float *x;   // fp32 activations, row b at x + (b0 + b) * x_ld
    int x_ld;
    int prologue;
    const float *norm_w;
    float eps;
    int xbf16;
};

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
// two signed int8 (bytes lo_sel / hi_sel of w) -> exact fp16x2 integers
__device__ __forceinline__ uint32_t q8_pair(uint32_t u_biased, uint32_t sel) {
    return hsub2_u32(__byte_perm(u_biased, 0x64646464u, sel), 0x64806480u);   // (1024 + (q+128)) - 1152
}
__device__ __forceinline__ uint32_t q4_pair(uint32_t w, int shift) {
    return hsub2_u32(((w >> shift) & 0x000F000Fu) | 0x64006400u, 0x64086408u);  // (1024 + n) - 1032
}
__device__ __forceinline__ float2 h2f2(uint32_t h) {
    __half2 v = *reinterpret_cast<__half2 *>(&h);
    return __half22float2(v);
}

// Accumulate one warp's share of a row tile: nkt consecutive k tiles starting at tile pointer `tp` whose first
// k index is kt0 * tile_k.  xr: this lane's activation row in smem (nullptr when its batch row g >= B).
template <int FMT, int U>
__device__ __forceinline__ void gemv_tiles(const uint8_t *tp, int kt0, int nkt, const uint16_t *xr, int lane,
                                           float &acc0, float &acc1) {
    constexpr int TK = tile_k(FMT), TB = tile_bytes(FMT);
    const int t = lane & 3;
    for (int i = 0; i < nkt; i += U) {
        uint4 q[U];
        uint4 sc[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (i + u < nkt) {
                const uint8_t *tb = tp + (size_t)(i + u) * TB;
                q[u] = ldg_stream16(tb + lane * 16);
                if constexpr (FMT == FMT_Q8) {
                    uint2 s2 = ldg_stream8(tb + 512 + t * 8);
                    sc[u] = make_uint4(s2.x, s2.y, 0u, 0u);
                } else if constexpr (FMT == FMT_Q4) {
                    sc[u] = ldg_stream16(tb + 512 + t * 16);
                } else if constexpr (FMT == FMT_F32) {
                    sc[u] = ldg_stream16(tb + 512 + lane * 16);               // mid plane
                }
            }
        }
        uint4 lo[U];
        if constexpr (FMT == FMT_F32) {
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (i + u < nkt) lo[u] = ldg_stream16(tp + (size_t)(i + u) * TB + 1024 + lane * 16);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (i + u >= nkt) break;
            const int kb = (kt0 + i + u) * TK;
            const uint32_t w[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
            auto afrag = [&](int s, uint32_t &a0, uint32_t &a2) {
                if (xr) {
                    a0 = *reinterpret_cast<const uint32_t *>(xr + kb + 16 * s + 2 * t);
                    a2 = *reinterpret_cast<const uint32_t *>(xr + kb + 16 * s + 2 * t + 8);
                } else {
                    a0 = 0u;
                    a2 = 0u;
                }
            };
            if constexpr (FMT == FMT_Q8) {
                const uint32_t sc2[2] = {sc[u].x, sc[u].y};
#pragma unroll
                for (int blk = 0; blk < 2; ++blk) {
                    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int ss = 0; ss < 2; ++ss) {
                        const int s = 2 * blk + ss;
                        uint32_t a0, a2;
                        afrag(s, a0, a2);
                        const uint32_t ub = w[s] ^ 0x80808080u;
                        mma_f16(d, a0, a2, q8_pair(ub, 0x4140u), q8_pair(ub, 0x4342u));
                    }
                    const float2 ds = h2f2(sc2[blk]);
                    acc0 = fmaf(ds.x, d[0], acc0);
                    acc1 = fmaf(ds.y, d[1], acc1);
                }
            } else if constexpr (FMT == FMT_Q4) {
                const uint32_t sc4[4] = {sc[u].x, sc[u].y, sc[u].z, sc[u].w};
#pragma unroll
                for (int blk = 0; blk < 4; ++blk) {
                    float d[4] = {0.f, 0.f, 0.f, 0.f};
                    uint32_t a0, a2;
                    afrag(2 * blk, a0, a2);
                    mma_f16(d, a0, a2, q4_pair(w[blk], 0), q4_pair(w[blk], 4));
                    afrag(2 * blk + 1, a0, a2);
                    mma_f16(d, a0, a2, q4_pair(w[blk], 8), q4_pair(w[blk], 12));
                    const float2 ds = h2f2(sc4[blk]);
                    acc0 = fmaf(ds.x, d[0], acc0);
                    acc1 = fmaf(ds.y, d[1], acc1);
                }
            } else {
                float d[4] = {acc0, acc1, 0.f, 0.f};
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                    uint32_t a0, a2;
                    afrag(s, a0, a2);
                    if constexpr (FMT == FMT_F16) {
                        mma_f16(d, a0, a2, w[2 * s], w[2 * s + 1]);
                    } else {
                        mma_bf16(d, a0, a2, w[2 * s], w[2 * s + 1]);
                        if constexpr (FMT == FMT_F32) {
                            const uint32_t m[4] = {sc[u].x, sc[u].y, sc[u].z, sc[u].w};
                            const uint32_t l[4] = {lo[u].x, lo[u].y, lo[u].z, lo[u].w};
                            mma_bf16(d, a0, a2, m[2 * s], m[2 * s + 1]);
                            mma_bf16(d, a0, a2, l[2 * s], l[2 * s + 1]);
                        }
                    }
                }
                acc0 = d[0];
                acc1 = d[1];
            }
        }
    }
}

// Convert the pass's activation rows to 16-bit in shared memory; returns per-row output scale in s_scale[b].
__device__ inline void gemv_prologue(const GemvArgs &a, uint16_t *xs, float *s_scale, float *s_red) {
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int b = 0; b < a.B; ++b) {
        const float *xr = a.x + (size_t)(a.b0 + b) * a.x_ld;
        float ss = 0.f, mx = 0.f;
        for (int k = tid; k < a.K; k += nt) {
            const float v = xr[k];
            ss = fmaf(v, v, ss);
            mx = fmaxf(mx, fabsf(a.prologue == PRO_RMSNORM ? v * a.norm_w[k] : v));
        }
        ss = warp_sum(ss);
        mx = warp_max(mx);
        if ((tid & 31) == 0) {
            s_red[tid >> 5] = ss;
            s_red[32 + (tid >> 5)] = mx;
        }
        __syncthreads();
        if (tid == 0) {
            float S = 0.f, Mx = 0.f;
            for (int w = 0; w < nt / 32; ++w) {
                S += s_red[w];
                Mx = fmaxf(Mx, s_red[32 + w]);
            }
            const float inv = (a.prologue == PRO_RMSNORM) ? 1.0f / sqrtf(S / (float)a.K + a.eps) : 1.0f;
            float e = 0.f;
            if (!a.xbf16 && Mx * inv > 0.f) {
                int ex;
                frexpf(Mx * inv, &ex);
                e = (float)(ex - 14);   // largest |x| scaled into (2^13, 2^14]
            }
            s_red[64] = inv;
            s_scale[b] = exp2f(e);
            s_red[65] = exp2f(-e);
        }
        __syncthreads();
        const float inv = s_red[64], sdown = s_red[65];
        uint16_t *xo = xs + b * a.kpx;
        for (int k = tid; k < a.kpx; k += nt) {
            float v = 0.f;
            if (k < a.K) {
                v = xr[k] * inv;
                if (a.prologue == PRO_RMSNORM) v *= a.norm_w[k];
            }
            if (a.xbf16) {
                __nv_bfloat16 h = __float2bfloat16_rn(v);
                xo[k] = *reinterpret_cast<uint16_t *>(&h);
            } else {
                __half h = __float2half_rn(v * sdown);
                xo[k] = *reinterpret_cast<uint16_t *>(&h);
            }
        }
        __syncthreads();
    }
}

template <class Epi>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(GemvArgs a, Epi epi) {
    extern __shared__ __align__(16) uint8_t smem[];
    float *s_red = reinterpret_cast<float *>(smem);                  // 96 floats
    float *s_scale = s_red + 96;                                     // GEMV_MB
    float *s_part = s_scale + GEMV_MB;                               // [8 warps][32 lanes][2]
    uint16_t *xs = reinterpret_cast<uint16_t *>(s_part + 8 * 32 * 2);
    gemv_prologue(a, xs, s_scale, s_red);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rtc = 8 / a.wk;
    const int rs = warp / a.wk, kw = warp % a.wk;
    const int gr = blockIdx.x * rtc + rs;
    float acc0 = 0.f, acc1 = 0.f;
    int si = 0, rt = gr;
    const bool active = gr < a.total_rtiles;
    if (active) {
        while (si < a.n_seg - 1 && rt >= a.seg[si].n_rtiles) {
            rt -= a.seg[si].n_rtiles;
            ++si;
        }
        const GemvSeg &sg = a.seg[si];
        const int KT = sg.n_ktiles;
        const int k0 = (kw * KT) / a.wk, k1 = ((kw + 1) * KT) / a.wk;
        const int g = lane >> 2;
        const uint16_t *xr = g < a.B ? xs + g * a.kpx : nullptr;
        const uint8_t *tp = sg.tiles + ((size_t)rt * KT + k0) * tile_bytes(sg.fmt);
        switch (sg.fmt) {
            case FMT_Q8: gemv_tiles<FMT_Q8, 4>(tp, k0, k1 - k0, xr, lane, acc0, acc1); break;
            case FMT_Q4: gemv_tiles<FMT_Q4, 4>(tp, k0, k1 - k0, xr, lane, acc0, acc1); break;
            case FMT_BF16: gemv_tiles<FMT_BF16, 4>(tp, k0, k1 - k0, xr, lane, acc0, acc1); break;
            case FMT_F16: gemv_tiles<FMT_F16, 4>(tp, k0, k1 - k0, xr, lane, acc0, acc1); break;
            default: gemv_tiles<FMT_F32, 2>(tp, k0, k1 - k0, xr, lane, acc0, acc1); break;
        }
    }
    if (a.wk > 1) {
        s_part[(warp * 32 + lane) * 2 + 0] = acc0;
        s_part[(warp * 32 + lane) * 2 + 1] = acc1;
        __syncthreads();
        if (kw == 0) {
            acc0 = 0.f;
            acc1 = 0.f;
            for (int w = 0; w < a.wk; ++w) {
                acc0 += s_part[((warp + w) * 32 + lane) * 2 + 0];
                acc1 += s_part[((warp + w) * 32 + lane) * 2 + 1];
            }
        }
    }
    if (active && kw == 0) {
        const int g = lane >> 2, t = lane & 3;
        if (g < a.B) epi(si, rt, t, a.b0 + g, acc0 * s_scale[g], acc1 * s_scale[g]);
    }
}

inline size_t gemv_smem_bytes(int B, int kpx) {
    return (96 + GEMV_MB + 8 * 32 * 2) * sizeof(float) + (size_t)B * kpx * sizeof(uint16_t);
}

// Host helper: choose the k split so the launch covers the GPU, fill the launch parameters.
void gemv_plan(GemvArgs &a, int n_sm, int &grid, size_t &smem);

}  // namespace v3g
