// Load-time weight re-tiling (VLT3 payload -> fragment-ordered 16-row tiles, layout in v3g.cuh), the inverse
// dequantizer used by the bit-exact tests, and the GEMV launch planner.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "v3g_gemv.cuh"
#include "v3g_internal.h"

namespace v3g {

struct RepackArgs {
    const uint8_t *src0, *src1;  // file payloads (src1: up_proj when interleaving gate/up)
    int fmt;                     // file dtype (= tile format)
    int src_rows, cols;          // rows of each source matrix, K
    int rowmap, head_dim;
    int n_rtiles, n_ktiles;
    float up;                    // BF16 / F32: 2^s applied before the fp16 conversion (1 otherwise)
    uint8_t *dst;
};

__device__ __forceinline__ bool map_row(const RepackArgs &a, int p, int &src, int &row) {
    return map_tile_row(a.rowmap, a.head_dim, a.src_rows, p, src, row);
}

// raw element access into VLT3 payloads (tools/vlt3.py block layouts)
__device__ __forceinline__ uint16_t raw_scale_bits(const RepackArgs &a, const uint8_t *s, int row, int blk) {
    const uint8_t *p = s + ((size_t)row * (a.cols / 32) + blk) * (a.fmt == FMT_Q8 ? 34 : 18);
    return (uint16_t)(p[0] | (p[1] << 8));
}
__device__ __forceinline__ int raw_q8(const RepackArgs &a, const uint8_t *s, int row, int k) {
    return (int)(int8_t)s[((size_t)row * (a.cols / 32) + k / 32) * 34 + 2 + (k & 31)];
}
__device__ __forceinline__ int raw_q4(const RepackArgs &a, const uint8_t *s, int row, int k) {
    const int i = k & 31;
    const uint8_t byte = s[((size_t)row * (a.cols / 32) + k / 32) * 18 + 2 + (i & 15)];
    return i < 16 ? (byte & 15) : (byte >> 4);
}
__device__ __forceinline__ uint16_t raw_u16(const RepackArgs &a, const uint8_t *s, int row, int k) {
    const uint8_t *p = s + ((size_t)row * a.cols + k) * 2;
    return (uint16_t)(p[0] | (p[1] << 8));
}
__device__ __forceinline__ float raw_f32(const RepackArgs &a, const uint8_t *s, int row, int k) {
    float v;
    memcpy(&v, s + ((size_t)row * a.cols + k) * 4, 4);
    return v;
}
__device__ __forceinline__ uint32_t f16_bits_rn(float v) { return __half_as_ushort(__float2half_rn(v)); }
__device__ __forceinline__ float f16_bits_to_f(uint32_t b) { return __half2float(__ushort_as_half((uint16_t)b)); }
__device__ __forceinline__ float bf16_bits_to_f(uint32_t b) { return __uint_as_float(b << 16); }

// largest |w| of a BF16 / F32 payload (n values), or largest |d| of a Q8_0 / Q4_0 payload's fp16 block scales (n
// blocks), as order-preserving bits (non-negative floats compare as integers)
__global__ void absmax_kernel(const uint8_t *src, int fmt, int64_t n, unsigned int *out) {
    float mx = 0.f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float v;
        if (fmt == FMT_BF16) v = bf16_bits_to_f((uint32_t)(src[2 * i] | (src[2 * i + 1] << 8)));
        else if (fmt == FMT_Q8 || fmt == FMT_Q4) {
            const uint8_t *b = src + i * (fmt == FMT_Q8 ? 34 : 18);
            v = f16_bits_to_f((uint32_t)(b[0] | (b[1] << 8)));
        } else memcpy(&v, src + 4 * i, 4);
        mx = fmaxf(mx, fabsf(v));
    }
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(mx));
}

// A-fragment position of the element with index e (0..7) in a lane's 8 halves of one k step:
//   e = 2 * reg + half, reg 0 (row g, k 2t+half), 1 (row g+8, k 2t+half), 2 (row g, k 2t+8+half), 3 (row g+8, ..)
__device__ __forceinline__ void frag_pos(int g, int t, int e, int &r, int &k) {
    const int reg = e >> 1, half = e & 1;
    r = g + ((reg & 1) ? 8 : 0);
    k = 2 * t + half + ((reg & 2) ? 8 : 0);
}

__global__ void repack_kernel(RepackArgs a) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t n = (int64_t)a.n_rtiles * a.n_ktiles * 32;
    if (gid >= n) return;
    const int lane = (int)(gid & 31);
    const int64_t tile = gid >> 5;
    const int rt = (int)(tile / a.n_ktiles), kt = (int)(tile % a.n_ktiles);
    const int g = lane >> 2, t = lane & 3;
    const int TK = tile_k(a.fmt);
    uint8_t *out = a.dst + tile * tile_bytes(a.fmt);
    // the two source rows this lane carries (tile rows g and g+8)
    int src_lo, row_lo, src_hi, row_hi;
    const bool ok_lo = map_row(a, rt * TILE_ROWS + g, src_lo, row_lo);
    const bool ok_hi = map_row(a, rt * TILE_ROWS + g + 8, src_hi, row_hi);
    auto rowinfo = [&](int r, const uint8_t *&s, int &row) {
        s = (r < 8 ? src_lo : src_hi) ? a.src1 : a.src0;
        row = r < 8 ? row_lo : row_hi;
        return r < 8 ? ok_lo : ok_hi;
    };
    uint32_t words[4] = {0, 0, 0, 0};
    if (a.fmt == FMT_Q8) {   // 2 k steps x 8 biased bytes
        for (int s = 0; s < 2; ++s)
            for (int e = 0; e < 8; ++e) {
                int r, k;
                frag_pos(g, t, e, r, k);
                k += kt * TK + 16 * s;
                const uint8_t *sp;
                int row;
                const bool ok = rowinfo(r, sp, row);
                const uint32_t u = (ok && k < a.cols) ? (uint32_t)(raw_q8(a, sp, row, k) + 128) : 128u;
                const int byte = 8 * s + e;   // reg order a0 a1 | a2 a3 per word pair
                words[byte >> 2] |= u << (8 * (byte & 3));
            }
    } else if (a.fmt == FMT_Q4) {   // 4 k steps x 8 nibbles: nibble 4h + reg (bits 4h+4reg .. ) of word s
        for (int s = 0; s < 4; ++s)
            for (int e = 0; e < 8; ++e) {
                int r, k;
                frag_pos(g, t, e, r, k);
                k += kt * TK + 16 * s;
                const uint8_t *sp;
                int row;
                const bool ok = rowinfo(r, sp, row);
                const uint32_t v = (ok && k < a.cols) ? (uint32_t)raw_q4(a, sp, row, k) : 8u;
                const int reg = e >> 1, half = e & 1;
                words[s] |= v << (4 * reg + 16 * half);
            }
    } else if (a.fmt == FMT_BF16 || a.fmt == FMT_F16) {   // 1 k step x 8 halves (BF16 -> fp16 of w 2^s, exact)
        for (int e = 0; e < 8; ++e) {
            int r, k;
            frag_pos(g, t, e, r, k);
            k += kt * TK;
            const uint8_t *sp;
            int row;
            const bool ok = rowinfo(r, sp, row);
            uint32_t v = (ok && k < a.cols) ? raw_u16(a, sp, row, k) : 0u;
            if (a.fmt == FMT_BF16) v = f16_bits_rn(__fmul_rn(bf16_bits_to_f(v), a.up));
            words[e >> 1] |= v << (16 * (e & 1));
        }
    } else {   // F32 -> fp16 planes with w 2^s == hi + 2^-11 mid + 2^-22 lo exactly (11 + 11 + 11 >= 24 bits)
        uint32_t mw[4] = {0, 0, 0, 0}, lw[4] = {0, 0, 0, 0};
        for (int e = 0; e < 8; ++e) {
            int r, k;
            frag_pos(g, t, e, r, k);
            k += kt * TK;
            const uint8_t *sp;
            int row;
            const bool ok = rowinfo(r, sp, row);
            const float w = (ok && k < a.cols) ? __fmul_rn(raw_f32(a, sp, row, k), a.up) : 0.f;
            const uint32_t h = f16_bits_rn(w);
            const float r1 = __fsub_rn(w, f16_bits_to_f(h));
            const uint32_t m = f16_bits_rn(__fmul_rn(r1, 2048.f));
            const uint32_t l = f16_bits_rn(__fmul_rn(__fsub_rn(r1, __fmul_rn(f16_bits_to_f(m), F32_MID)), 4194304.f));
            const int sh = 16 * (e & 1);
            words[e >> 1] |= h << sh;
            mw[e >> 1] |= m << sh;
            lw[e >> 1] |= l << sh;
        }
        *reinterpret_cast<uint4 *>(out + 512 + lane * 16) = make_uint4(mw[0], mw[1], mw[2], mw[3]);
        *reinterpret_cast<uint4 *>(out + 1024 + lane * 16) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    *reinterpret_cast<uint4 *>(out + lane * 16) = make_uint4(words[0], words[1], words[2], words[3]);
    // block scales, per g: Q8 half2(d[g], d[g+8]); Q4 {half2(d[g][b0], d[g+8][b0]), half2(d[g][b1], d[g+8][b1])}
    if ((a.fmt == FMT_Q8 || a.fmt == FMT_Q4) && t == 0) {
        const int nblk = TK / 32;
        uint32_t sc[2] = {0, 0};
        for (int b = 0; b < nblk; ++b) {
            const int blk = kt * nblk + b;
            const uint32_t lo = (ok_lo && blk * 32 < a.cols) ? raw_scale_bits(a, src_lo ? a.src1 : a.src0, row_lo, blk) : 0;
            const uint32_t hi = (ok_hi && blk * 32 < a.cols) ? raw_scale_bits(a, src_hi ? a.src1 : a.src0, row_hi, blk) : 0;
            sc[b] = lo | (hi << 16);
        }
        if (nblk == 1) *reinterpret_cast<uint32_t *>(out + 512 + g * 4) = sc[0];
        else *reinterpret_cast<uint2 *>(out + 512 + g * 8) = make_uint2(sc[0], sc[1]);
    }
}

// out[source row][k] for every element, undoing the row map ([gate; up] for gate/up tiles)
__global__ void dequant_tiles_kernel(const uint8_t *tiles, int fmt, int n_ktiles, int rows, int cols, RepackArgs map,
                                     float *out) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)rows * cols) return;
    const int p = (int)(gid / cols), k = (int)(gid % cols);
    int src, srow;
    if (!map_row(map, p, src, srow)) return;
    out[(size_t)(src * map.src_rows + srow) * cols + k] = tile_value(tiles, fmt, n_ktiles, map.up, p, k);
}

int repack_matrix(MatW &w, const uint8_t *dev_src0, const uint8_t *dev_src1, int fmt, int src_rows, int cols,
                  int rowmap, int head_dim, uint8_t *dst, cudaStream_t st) {
    RepackArgs a;
    a.src0 = dev_src0;
    a.src1 = dev_src1;
    a.fmt = fmt;
    a.src_rows = src_rows;
    a.cols = cols;
    a.rowmap = rowmap;
    a.head_dim = head_dim;
    const int rows = rowmap == ROWS_GATE_UP ? 2 * src_rows : src_rows;
    a.n_rtiles = (rows + TILE_ROWS - 1) / TILE_ROWS;
    a.n_ktiles = (cols + tile_k(fmt) - 1) / tile_k(fmt);
    a.dst = dst;
    a.up = 1.f;
    w.wscale = 1.f;
    if (fmt == FMT_BF16 || fmt == FMT_F32) {   // per-matrix power of two: max|w| 2^s in [2^14, 2^15)
        unsigned int *d_mx = nullptr, mx = 0;
        if (cudaMallocAsync(&d_mx, 4, st) != cudaSuccess) return -1;
        cudaMemsetAsync(d_mx, 0, 4, st);
        const int64_t ne = (int64_t)src_rows * cols;
        absmax_kernel<<<256, 256, 0, st>>>(dev_src0, fmt, ne, d_mx);
        if (dev_src1) absmax_kernel<<<256, 256, 0, st>>>(dev_src1, fmt, ne, d_mx);
        cudaMemcpyAsync(&mx, d_mx, 4, cudaMemcpyDeviceToHost, st);
        cudaFreeAsync(d_mx, st);
        if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
        float fm;
        memcpy(&fm, &mx, 4);
        if (fm > 0.f && std::isfinite(fm)) {
            int ex;
            std::frexp(fm, &ex);                 // fm in [2^(ex-1), 2^ex)
            const int sh = 15 - ex;
            a.up = std::ldexp(1.f, sh);
            w.wscale = std::ldexp(1.f, -sh);
        }
    }
    w.dexp = 0;
    if (fmt == FMT_Q8 || fmt == FMT_Q4) {   // tensor-core path: block scales times 2^dexp, max |q d| 2^dexp ~ 2^13
        unsigned int *d_mx = nullptr, mx = 0;
        if (cudaMallocAsync(&d_mx, 4, st) != cudaSuccess) return -1;
        cudaMemsetAsync(d_mx, 0, 4, st);
        const int64_t nb = (int64_t)src_rows * cols / 32;
        absmax_kernel<<<256, 256, 0, st>>>(dev_src0, fmt, nb, d_mx);
        if (dev_src1) absmax_kernel<<<256, 256, 0, st>>>(dev_src1, fmt, nb, d_mx);
        cudaMemcpyAsync(&mx, d_mx, 4, cudaMemcpyDeviceToHost, st);
        cudaFreeAsync(d_mx, st);
        if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
        float fm;
        memcpy(&fm, &mx, 4);
        fm *= fmt == FMT_Q8 ? 127.f : 8.f;
        if (fm > 0.f && std::isfinite(fm)) {
            int ex;
            std::frexp(fm, &ex);                 // largest |value| in [2^(ex-1), 2^ex)
            // 2^dexp is applied to fp16 block scales by an fp16 multiply: keep it inside fp16's normal range
            w.dexp = std::max(-14, std::min(15, 14 - ex));
        }
    }
    const int64_t n = (int64_t)a.n_rtiles * a.n_ktiles * 32;
    repack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a);
    w.tiles = dst;
    w.fmt = fmt;
    w.rows = rows;
    w.cols = cols;
    w.n_rtiles = a.n_rtiles;
    w.n_ktiles = a.n_ktiles;
    w.rowmap = rowmap;
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

size_t matrix_tile_bytes(int fmt, int rows, int cols) {
    return (size_t)((rows + TILE_ROWS - 1) / TILE_ROWS) * ((cols + tile_k(fmt) - 1) / tile_k(fmt)) * tile_bytes(fmt);
}

int dequant_matrix(const MatW &w, int head_dim, float *out, cudaStream_t st) {
    RepackArgs map{};
    map.rowmap = w.rowmap;
    map.head_dim = head_dim;
    map.src_rows = w.rowmap == ROWS_GATE_UP ? w.rows / 2 : w.rows;
    map.up = w.wscale;
    const int64_t n = (int64_t)w.rows * w.cols;
    dequant_tiles_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w.tiles, w.fmt, w.n_ktiles, w.rows, w.cols, map,
                                                                        out);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

void gemv_plan(GemvArgs &a, const int *fmts, int n_sm, int &grid, size_t &smem) {
    if (a.lo < 0) a.lo = gemv_lo(a.B);   // default: two fp16 parts per activation when the batch leaves columns free
    int maxk = 0, kpad = 0;
    bool bsum = false;
    a.total_rtiles = 0;
    for (int i = 0; i < a.n_seg; ++i) {
        a.total_rtiles += a.seg[i].n_rtiles;
        maxk = a.seg[i].n_ktiles > maxk ? a.seg[i].n_ktiles : maxk;
        const int kp = a.seg[i].n_ktiles * tile_k(fmts[i]);
        kpad = kp > kpad ? kp : kpad;
        bsum = bsum || fmt_int(fmts[i]);
    }
    kpad = (kpad + 31) / 32 * 32;
    a.kpx = kpad + 8;   // +8 halves: conflict-free fragment loads
    a.nblk = kpad / 32;
    // smallest k split that still puts >= 2 CTAs on every SM, keeping >= 2 k tiles per warp
    int wk = 1;
    while (wk < 8) {
        const int ctas = (a.total_rtiles + (8 / wk) - 1) / (8 / wk);
        if (ctas >= 2 * n_sm) break;
        if (maxk / (wk * 2) < 2) break;
        wk *= 2;
    }
    a.wk = wk;
    grid = (a.total_rtiles + (8 / wk) - 1) / (8 / wk);
    smem = gemv_smem_bytes(a, bsum);
}

}  // namespace v3g
