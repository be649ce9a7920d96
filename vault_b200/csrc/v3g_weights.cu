// Load-time weight re-tiling (VLT3 payload -> fragment-ordered tiles), the inverse dequantizer used by the
// bit-exact tests, and the GEMV launch planner.
#include "v3g_gemv.cuh"
#include "v3g_internal.h"

namespace v3g {

struct RepackArgs {
    const uint8_t *src0, *src1;  // file payloads (src1: up_proj when interleaving gate/up)
    int fmt;                     // file dtype (= tile format)
    int src_rows, cols;          // rows of each source matrix, K
    int rowmap, head_dim;
    int n_rtiles, n_ktiles;
    uint8_t *dst;
};

// logical tile row p -> (source, source row); false when p is padding
__device__ __forceinline__ bool map_row(const RepackArgs &a, int p, int &src, int &row) {
    return map_tile_row(a.rowmap, a.head_dim, a.src_rows, p, src, row);
}

__device__ __forceinline__ uint16_t raw_scale_bits(const RepackArgs &a, const uint8_t *s, int row, int blk) {
    const int bpr = a.cols / 32;
    const int bb = a.fmt == FMT_Q8 ? 34 : 18;
    const uint8_t *p = s + ((size_t)row * bpr + blk) * bb;
    return (uint16_t)(p[0] | (p[1] << 8));
}
__device__ __forceinline__ int raw_q8(const RepackArgs &a, const uint8_t *s, int row, int k) {
    const int bpr = a.cols / 32;
    return (int)(int8_t)s[((size_t)row * bpr + k / 32) * 34 + 2 + (k & 31)];
}
__device__ __forceinline__ int raw_q4(const RepackArgs &a, const uint8_t *s, int row, int k) {
    const int bpr = a.cols / 32, i = k & 31;
    const uint8_t byte = s[((size_t)row * bpr + k / 32) * 18 + 2 + (i & 15)];
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
__device__ __forceinline__ uint16_t bf16_bits_rn(float v) {
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    return *reinterpret_cast<uint16_t *>(&h);
}
__device__ __forceinline__ float bf16_bits_to_f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// k offset of element e (0..3) of lane-quad t inside a 16-wide k step
__device__ __forceinline__ int koff(int t, int e) { return 2 * t + (e & 1) + ((e & 2) ? 8 : 0); }

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
    int src, row;
    const bool ok = map_row(a, rt * 8 + g, src, row);
    const uint8_t *s = src ? a.src1 : a.src0;
    uint8_t bytes[16];
    if (a.fmt == FMT_Q8) {
        for (int st = 0; st < 4; ++st)
            for (int e = 0; e < 4; ++e) {
                const int k = kt * TK + 16 * st + koff(t, e);
                bytes[4 * st + e] = (ok && k < a.cols) ? (uint8_t)raw_q8(a, s, row, k) : 0;
            }
    } else if (a.fmt == FMT_Q4) {
        // word j covers k steps 2j (bits 0-3,16-19 / 4-7,20-23) and 2j+1 (bits 8-11,24-27 / 12-15,28-31)
        for (int j = 0; j < 4; ++j) {
            uint32_t w = 0;
            for (int nib = 0; nib < 8; ++nib) {
                const int st = 2 * j + ((nib >> 1) & 1);
                const int e = ((nib & 1) ? 2 : 0) + ((nib >> 2) & 1);
                const int k = kt * TK + 16 * st + koff(t, e);
                const int v = (ok && k < a.cols) ? raw_q4(a, s, row, k) : 8;
                w |= (uint32_t)v << (4 * nib);
            }
            memcpy(bytes + 4 * j, &w, 4);
        }
    } else if (a.fmt == FMT_BF16 || a.fmt == FMT_F16) {
        for (int st = 0; st < 2; ++st)
            for (int e = 0; e < 4; ++e) {
                const int k = kt * TK + 16 * st + koff(t, e);
                const uint16_t v = (ok && k < a.cols) ? raw_u16(a, s, row, k) : 0;
                memcpy(bytes + 2 * (4 * st + e), &v, 2);
            }
    } else {  // F32 -> three bf16 planes
        uint8_t mid[16], lo[16];
        for (int st = 0; st < 2; ++st)
            for (int e = 0; e < 4; ++e) {
                const int k = kt * TK + 16 * st + koff(t, e);
                const float w = (ok && k < a.cols) ? raw_f32(a, s, row, k) : 0.f;
                const uint16_t h = bf16_bits_rn(w);
                const float r1 = w - bf16_bits_to_f(h);
                const uint16_t m = bf16_bits_rn(r1);
                const uint16_t l = bf16_bits_rn(r1 - bf16_bits_to_f(m));
                memcpy(bytes + 2 * (4 * st + e), &h, 2);
                memcpy(mid + 2 * (4 * st + e), &m, 2);
                memcpy(lo + 2 * (4 * st + e), &l, 2);
            }
        memcpy(out + 512 + lane * 16, mid, 16);
        memcpy(out + 1024 + lane * 16, lo, 16);
    }
    memcpy(out + lane * 16, bytes, 16);
    // block scales: lane (g == 0, t) writes the scales of tile rows 2t and 2t+1
    if ((a.fmt == FMT_Q8 || a.fmt == FMT_Q4) && g == 0) {
        const int nblk = TK / 32;
        uint16_t sc[8];
        for (int b = 0; b < nblk; ++b)
            for (int h = 0; h < 2; ++h) {
                int s2, r2;
                const bool ok2 = map_row(a, rt * 8 + 2 * t + h, s2, r2);
                const int blk = kt * nblk + b;
                sc[2 * b + h] = (ok2 && blk * 32 < a.cols) ? raw_scale_bits(a, s2 ? a.src1 : a.src0, r2, blk) : 0;
            }
        memcpy(out + 512 + t * (2 * nblk * 2), sc, 2 * nblk * 2);
    }
}

// fp32 values of logical row `p` (tile order) columns [0, cols) -> out[p * cols + k]; exact inverse of the repack
__global__ void dequant_tiles_kernel(const uint8_t *tiles, int fmt, int n_rtiles, int n_ktiles, int rows, int cols,
                                     RepackArgs map, float *out) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t n = (int64_t)n_rtiles * n_ktiles * 32;
    if (gid >= n) return;
    const int lane = (int)(gid & 31);
    const int64_t tile = gid >> 5;
    const int rt = (int)(tile / n_ktiles), kt = (int)(tile % n_ktiles);
    const int g = lane >> 2, t = lane & 3, TK = tile_k(fmt);
    int src, srow;
    if (rt * 8 + g >= rows || !map_row(map, rt * 8 + g, src, srow)) return;
    const int p = src * map.src_rows + srow;   // output row in source order ([gate; up] for gate/up tiles)
    const uint8_t *tb = tiles + tile * tile_bytes(fmt);
    const uint8_t *q = tb + lane * 16;
    if (fmt == FMT_Q8 || fmt == FMT_Q4) {
        // scales of row g live with lane-quad t' = g / 2, half g % 2
        const int t2 = g >> 1, h = g & 1, nblk = TK / 32;
        const uint16_t *sc = reinterpret_cast<const uint16_t *>(tb + 512 + t2 * (2 * nblk * 2));
        if (fmt == FMT_Q8) {
            for (int st = 0; st < 4; ++st)
                for (int e = 0; e < 4; ++e) {
                    const int k = kt * TK + 16 * st + koff(t, e);
                    if (k >= cols) continue;
                    const float d = __half2float(__ushort_as_half(sc[2 * (k % TK / 32) + h]));
                    out[(size_t)p * cols + k] = (float)(int8_t)q[4 * st + e] * d;
                }
        } else {
            for (int j = 0; j < 4; ++j) {
                uint32_t w;
                memcpy(&w, q + 4 * j, 4);
                for (int nib = 0; nib < 8; ++nib) {
                    const int st = 2 * j + ((nib >> 1) & 1);
                    const int e = ((nib & 1) ? 2 : 0) + ((nib >> 2) & 1);
                    const int k = kt * TK + 16 * st + koff(t, e);
                    if (k >= cols) continue;
                    const float d = __half2float(__ushort_as_half(sc[2 * (k % TK / 32) + h]));
                    out[(size_t)p * cols + k] = (float)((int)((w >> (4 * nib)) & 15u) - 8) * d;
                }
            }
        }
    } else {
        for (int st = 0; st < 2; ++st)
            for (int e = 0; e < 4; ++e) {
                const int k = kt * TK + 16 * st + koff(t, e);
                if (k >= cols) continue;
                uint16_t v;
                memcpy(&v, q + 2 * (4 * st + e), 2);
                float f;
                if (fmt == FMT_F16) {
                    f = __half2float(__ushort_as_half(v));
                } else if (fmt == FMT_BF16) {
                    f = bf16_bits_to_f(v);
                } else {
                    uint16_t m, l;
                    memcpy(&m, tb + 512 + lane * 16 + 2 * (4 * st + e), 2);
                    memcpy(&l, tb + 1024 + lane * 16 + 2 * (4 * st + e), 2);
                    f = (bf16_bits_to_f(v) + bf16_bits_to_f(m)) + bf16_bits_to_f(l);
                }
                out[(size_t)p * cols + k] = f;
            }
    }
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
    a.n_rtiles = (rows + 7) / 8;
    a.n_ktiles = (cols + tile_k(fmt) - 1) / tile_k(fmt);
    a.dst = dst;
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
    return (size_t)((rows + 7) / 8) * ((cols + tile_k(fmt) - 1) / tile_k(fmt)) * tile_bytes(fmt);
}

int dequant_matrix(const MatW &w, int head_dim, float *out, cudaStream_t st) {
    const int64_t n = (int64_t)w.n_rtiles * w.n_ktiles * 32;
    RepackArgs map{};
    map.rowmap = w.rowmap;
    map.head_dim = head_dim;
    map.src_rows = w.rowmap == ROWS_GATE_UP ? w.rows / 2 : w.rows;
    dequant_tiles_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w.tiles, w.fmt, w.n_rtiles, w.n_ktiles,
                                                                        w.rows, w.cols, map, out);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

void gemv_plan(GemvArgs &a, int n_sm, int &grid, size_t &smem) {
    int maxk = 0, kpad = 0;
    a.total_rtiles = 0;
    for (int i = 0; i < a.n_seg; ++i) {
        a.total_rtiles += a.seg[i].n_rtiles;
        maxk = a.seg[i].n_ktiles > maxk ? a.seg[i].n_ktiles : maxk;
        const int kp = a.seg[i].n_ktiles * tile_k(a.seg[i].fmt);
        kpad = kp > kpad ? kp : kpad;
    }
    a.kpx = kpad + 8;   // +8 halves: conflict-free fragment loads
    // smallest k split that still puts >= 2 CTAs on every SM, with >= 2 k tiles per warp
    int wk = 1;
    while (wk < 8) {
        const int ctas = (a.total_rtiles + (8 / wk) - 1) / (8 / wk);
        if (ctas >= 2 * n_sm) break;
        if (maxk / (wk * 2) < 2) break;
        wk *= 2;
    }
    a.wk = wk;
    grid = (a.total_rtiles + (8 / wk) - 1) / (8 / wk);
    smem = gemv_smem_bytes(a.B, a.kpx);
}

}  // namespace v3g
