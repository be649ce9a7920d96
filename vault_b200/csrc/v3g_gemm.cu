// Host side of the tensor-core GEMM (launch planning, activation tensor maps), the activation operand kernel, and
// the kernel-level entry point v3g_gemm used by the tests and the kernel sweep.
#include <string.h>

#include <algorithm>
#include <cmath>

#include <mutex>

#include "../../include/vault_b200.h"
#include "v3g_gemm.cuh"
#include "v3g_internal.h"

namespace v3g {

// ------------------------------------------------------------------------------------------ activation operand
__global__ void __launch_bounds__(256) k_tc_prep(const float *x, int64_t ld_x, int K, const float *norm_w, float eps,
                                                 __half *out, int ldo, float *xscale) {
    const int r = blockIdx.x, tid = threadIdx.x;
    const float *xr = x + (int64_t)r * ld_x;
    __shared__ float red[2][8];
    float ss = 0.f, mx = 0.f;
    for (int k = tid; k < K; k += blockDim.x) {
        const float v = xr[k];
        ss = fmaf(v, v, ss);
        mx = fmaxf(mx, fabsf(norm_w ? v * norm_w[k] : v));
    }
    ss = warp_sum(ss);
    mx = warp_max(mx);
    if ((tid & 31) == 0) {
        red[0][tid >> 5] = ss;
        red[1][tid >> 5] = mx;
    }
    __syncthreads();
    float S = 0.f, M = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) {
        S += red[0][w];
        M = fmaxf(M, red[1][w]);
    }
    const float inv = norm_w ? rsqrtf(S / (float)K + eps) : 1.f;
    // largest |value| into (2^13, 2^14]: exponent from the float bits (zero / subnormal maxima keep e = 0)
    const int be = (__float_as_int(M * inv) >> 23) & 0xff;
    int e = be > 0 ? be - 140 : 0;
    e = e < -126 ? -126 : (e > 126 ? 126 : e);
    const float mul = inv * __int_as_float((127 - e) << 23);
    __half *o = out + (int64_t)r * ldo;
    for (int k = tid; k < ldo; k += blockDim.x) {
        const float v = k < K ? xr[k] * (norm_w ? norm_w[k] : 1.f) * mul : 0.f;
        o[k] = __float2half_rn(v);
    }
    if (tid == 0) xscale[r] = __int_as_float((127 + e) << 23);
}

// The same operand for K a multiple of 4 and at most 1024 NV: the row is read once with 16-byte loads and held in
// registers (NV float4 per thread) for both the statistics and the conversion; 8-byte fp16 stores.
template <int NV>
__global__ void __launch_bounds__(256) k_tc_prep_v(const float *x, int64_t ld_x, int K, const float *norm_w,
                                                   float eps, __half *out, int ldo, float *xscale) {
    const int r = blockIdx.x, tid = threadIdx.x, K4 = K >> 2;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (int64_t)r * ld_x);
    const float4 *wr = reinterpret_cast<const float4 *>(norm_w);
    __shared__ float red[2][8];
    float4 v[NV];
    float ss = 0.f, mx = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int q = tid + 256 * i;
        v[i] = q < K4 ? xr[q] : make_float4(0.f, 0.f, 0.f, 0.f);
        if (norm_w && q < K4) {
            const float4 w = __ldg(wr + q);
            ss = fmaf(v[i].x, v[i].x, ss);
            ss = fmaf(v[i].y, v[i].y, ss);
            ss = fmaf(v[i].z, v[i].z, ss);
            ss = fmaf(v[i].w, v[i].w, ss);
            v[i].x *= w.x;
            v[i].y *= w.y;
            v[i].z *= w.z;
            v[i].w *= w.w;
        }
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
    ss = warp_sum(ss);
    mx = warp_max(mx);
    if ((tid & 31) == 0) {
        red[0][tid >> 5] = ss;
        red[1][tid >> 5] = mx;
    }
    __syncthreads();
    float S = 0.f, M = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        S += red[0][w];
        M = fmaxf(M, red[1][w]);
    }
    const float inv = norm_w ? rsqrtf(S / (float)K + eps) : 1.f;
    const int be = (__float_as_int(M * inv) >> 23) & 0xff;
    int e = be > 0 ? be - 140 : 0;
    e = e < -126 ? -126 : (e > 126 ? 126 : e);
    const float mul = inv * __int_as_float((127 - e) << 23);
    uint2 *o = reinterpret_cast<uint2 *>(out + (int64_t)r * ldo);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int q = tid + 256 * i;
        if (q < K4) {
            const __half2 lo = __floats2half2_rn(v[i].x * mul, v[i].y * mul);
            const __half2 hi = __floats2half2_rn(v[i].z * mul, v[i].w * mul);
            o[q] = make_uint2(*reinterpret_cast<const uint32_t *>(&lo), *reinterpret_cast<const uint32_t *>(&hi));
        }
    }
    for (int q = K4 + tid; q < (ldo >> 2); q += 256) o[q] = make_uint2(0u, 0u);   // zero padding up to ldo
    if (tid == 0) xscale[r] = __int_as_float((127 + e) << 23);
}

cudaError_t tc_prep(const float *x, int64_t ld_x, int n, int K, const float *norm_w, float eps, __half *out, int ldo,
                    float *xscale, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const bool vec = K % 4 == 0 && ld_x % 4 == 0 && ldo % 4 == 0 && ((uintptr_t)x & 15) == 0 &&
                     ((uintptr_t)norm_w & 15) == 0 && ((uintptr_t)out & 7) == 0;
    const int nv = (K / 4 + 255) / 256;
    if (vec && nv <= 2)
        k_tc_prep_v<2><<<n, 256, 0, st>>>(x, ld_x, K, norm_w, eps, out, ldo, xscale);
    else if (vec && nv <= 4)
        k_tc_prep_v<4><<<n, 256, 0, st>>>(x, ld_x, K, norm_w, eps, out, ldo, xscale);
    else if (vec && nv <= 9)
        k_tc_prep_v<9><<<n, 256, 0, st>>>(x, ld_x, K, norm_w, eps, out, ldo, xscale);
    else
        k_tc_prep<<<n, 256, 0, st>>>(x, ld_x, K, norm_w, eps, out, ldo, xscale);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------------------ tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// fp16 matrix [rows, K] with row stride ld elements, loaded as (64 k) x (box_rows rows) boxes with the 128-byte
// swizzle; reads past K or past the last row return zeros
static cudaError_t make_xmap(CUtensorMap *map, const __half *x, int rows, int K, int ld, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (ld * 2) % 16) return cudaErrorInvalidValue;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(x), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// weight tensor map of one matrix: its row-tile buffer as [n_rtiles rows] x [stored bytes of a row tile / 8] elements
// of 8 bytes (rows contiguous), boxes of 8 rows x one 64-k stage; reads past the row (the last stage of a K that is
// not a multiple of 64) or past the last row tile return zeros
static cudaError_t make_wmap(CUtensorMap *map, const MatW &w) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const int tb = tile_bytes(w.fmt), row = w.n_ktiles * tb, box_bytes = tc_stage_raw_bytes(w.fmt);
    if ((reinterpret_cast<uintptr_t>(w.tiles) & 15) || row % 16 || box_bytes % 16 || box_bytes / 8 > 256)
        return cudaErrorInvalidValue;
    const cuuint64_t dims[2] = {(cuuint64_t)(row / 8), (cuuint64_t)w.n_rtiles};
    const cuuint64_t strides[1] = {(cuuint64_t)row};
    const cuuint32_t box[2] = {(cuuint32_t)(box_bytes / 8), 8u};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t *>(w.tiles), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// ------------------------------------------------------------------------------------------------ launch plan
cudaError_t tc_setup(TcLaunch &L, const MatW *const *mats, int n, const __half *x16, int ldx, const float *xscale,
                     int n_tok, int *status, int n_sm, const TcSplitWs *sk) {
    memset(&L, 0, sizeof(L));
    TcArgs &a = L.a;
    if (n < 1 || n > 3 || n_tok < 1) return cudaErrorInvalidValue;
    bool has[16] = {};
    int rb = 0;
    for (int i = 0; i < n; ++i) {
        const MatW &w = *mats[i];
        if (!(w.fmt == FMT_Q8 || w.fmt == FMT_Q4 || w.fmt == FMT_BF16 || w.fmt == FMT_F16)) return cudaErrorNotSupported;
        if (i > 0 && w.cols != mats[0]->cols) return cudaErrorInvalidValue;
        has[w.fmt] = true;
        a.seg[i].tiles = w.tiles;
        a.seg[i].n_rtiles = w.n_rtiles;
        a.seg[i].n_ktiles = w.n_ktiles;
        a.seg[i].fmt = w.fmt;
        a.seg[i].dexp = (w.fmt == FMT_Q8 || w.fmt == FMT_Q4) ? w.dexp : 0;
        a.seg[i].wscale = (w.fmt == FMT_Q8 || w.fmt == FMT_Q4) ? std::ldexp(1.f, -w.dexp) : w.wscale;
        a.rbase[i] = rb;
        rb += w.n_rtiles;
    }
    a.n_seg = n;
    a.rbase[n] = rb;
    int nf = 0;
    for (bool h : has) nf += h ? 1 : 0;
    if (nf == 1) {
        L.fa = L.fb = mats[0]->fmt;
    } else if (nf == 2 && has[FMT_Q4] && has[FMT_Q8]) {
        L.fa = FMT_Q4;
        L.fb = FMT_Q8;
    } else {
        return cudaErrorNotSupported;
    }
    a.K = mats[0]->cols;
    if (ldx < a.K) return cudaErrorInvalidValue;
    a.kstages = (a.K + TC_BK - 1) / TC_BK;
    a.m_tiles = (rb + 7) / 8;
    a.n_tok = n_tok;
    // token tile: the smallest multiple of 16 covering n_tok, at most 256 (the MMA's N range for M = 128)
    a.bn = n_tok >= 256 ? 256 : (n_tok + 15) / 16 * 16;
    a.n_tiles = (n_tok + a.bn - 1) / a.bn;
    a.xscale = xscale;
    a.status = status;
    a.seg_base = 0;
    a.stage_a = TC_BM * TC_BK * 2;
    a.stage_x = a.bn * TC_BK * 2;
    a.raw_row = std::max(tc_stage_raw_bytes(L.fa), tc_stage_raw_bytes(L.fb));   // multiples of 16 bytes
    a.stage_raw = 8 * a.raw_row;
    const int per_stage = a.stage_a + a.stage_x + a.stage_raw;
    const int budget = 227 * 1024 - 1024 - 256;
    a.stages = budget / per_stage < TC_MAX_STAGES ? budget / per_stage : TC_MAX_STAGES;
    if (a.stages < 2) return cudaErrorInvalidValue;
    a.a_off = 0;
    a.x_off = a.stages * a.stage_a;
    a.raw_off = a.x_off + a.stages * a.stage_x;
    a.bar_off = a.raw_off + a.stages * a.stage_raw;
    L.smem = (size_t)a.bar_off + 8 * (3 * a.stages + 4) + 16 + 1024;   // + TMEM address, flag, alignment slack
    // split K when the output tiles cannot cover the GPU (small batches): up to 16 splits of >= 4 stages each,
    // bounded by the workspace
    const int tiles = a.m_tiles * a.n_tiles;
    a.splits = 1;
    if (sk && sk->ws && tiles < n_sm) {
        int sp = n_sm / tiles;
        sp = std::min(sp, std::min(16, a.kstages / 4));
        while (sp > 1 && (size_t)tiles * sp * a.bn * TC_BM * 4 > sk->ws_bytes) --sp;
        if (sp > 1) {
            a.splits = sp;
            a.ws = sk->ws;
        }
    }
    const int work = tiles * a.splits;
    L.grid = work < n_sm ? work : n_sm;
    // weights by one TMA box per stage when no CTA tile straddles two matrices (segments start at multiples of 8
    // row tiles); otherwise one bulk copy per row tile
    a.w_tma = 1;
    for (int i = 0; i < n; ++i)
        if (a.rbase[i] % 8 != 0 || make_wmap(&L.wm.w[i], *mats[i]) != cudaSuccess) a.w_tma = 0;
    return make_xmap(&L.xmap, x16, n_tok, a.K, ldx, a.bn);
}

// ------------------------------------------------------------------------------------------- test epilogue
// y[token, source row] = value: undoes the RoPE-pair / gate-up row order of the tiles (seg = matrix index)
struct TcEpiStore {
    float *y;
    int64_t ld;
    int rowmap, head_dim, src_rows;
    __device__ void operator()(int, int rt, int g, int tok, float y0, float y1) const {
        int src, row;
        if (map_tile_row(rowmap, head_dim, src_rows, TILE_ROWS * rt + g, src, row))
            y[tok * ld + src * src_rows + row] = y0;
        if (map_tile_row(rowmap, head_dim, src_rows, TILE_ROWS * rt + g + 8, src, row))
            y[tok * ld + src * src_rows + row] = y1;
    }
    template <int N>
    __device__ void chunk(int seg, int rt, int g, int tok0, int nv, const float (&y0)[N], const float (&y1)[N]) const {
#pragma unroll
        for (int j = 0; j < N; ++j)
            if (j < nv) (*this)(seg, rt, g, tok0 + j, y0[j], y1[j]);
    }
};

}  // namespace v3g

using namespace v3g;

static const MatW *tc_find_mat(const v3g_model *m, uint32_t id) {
    for (auto &p : m->tensor_index)
        if (p.first == id) return p.second;
    return nullptr;
}

extern "C" size_t v3g_gemm_work_size(const v3g_model *m, uint32_t tensor_id, uint32_t n_tok) {
    const MatW *w = m ? tc_find_mat(m, tensor_id) : nullptr;
    if (!w || n_tok == 0) return 0;
    const size_t ldx = (size_t)(w->cols + 63) / 64 * 64;
    return ((size_t)n_tok * ldx * 2 + 255) / 256 * 256 + ((size_t)n_tok * 4 + 255) / 256 * 256 + 256 +
           TC_SPLITK_WS_BYTES;
}

extern "C" int v3g_gemm(const v3g_model *m, uint32_t tensor_id, const float *dev_x, uint32_t n_tok, float *dev_y,
                        void *dev_work, size_t work_bytes, void *stream) {
    if (!m || !dev_x || !dev_y || !dev_work || n_tok == 0) return v3g_fail(V3G_E_ARG, "null argument or zero tokens");
    const MatW *w = tc_find_mat(m, tensor_id);
    if (!w) return v3g_fail(V3G_E_MISSING, "no device matrix for this tensor id");
    if (work_bytes < v3g_gemm_work_size(m, tensor_id, n_tok) || (reinterpret_cast<uintptr_t>(dev_work) & 255))
        return v3g_fail(V3G_E_ARG, "workspace too small or not 256-byte aligned (v3g_gemm_work_size)");
    cudaStream_t st = (cudaStream_t)stream;
    const int ldx = (w->cols + 63) / 64 * 64;
    uint8_t *wp = static_cast<uint8_t *>(dev_work);
    __half *x16 = reinterpret_cast<__half *>(wp);
    float *xs = reinterpret_cast<float *>(wp + ((size_t)n_tok * ldx * 2 + 255) / 256 * 256);
    int *status = reinterpret_cast<int *>(reinterpret_cast<uint8_t *>(xs) + ((size_t)n_tok * 4 + 255) / 256 * 256);
    TcSplitWs sk;
    sk.ws = reinterpret_cast<float *>(status + 64);
    sk.ws_bytes = TC_SPLITK_WS_BYTES;
    cudaError_t e = cudaMemsetAsync(status, 0, 4, st);
    if (e == cudaSuccess) e = tc_prep(dev_x, w->cols, (int)n_tok, w->cols, nullptr, 0.f, x16, ldx, xs, st);
    const MatW *mats[1] = {w};
    const int src_rows = w->rowmap == ROWS_GATE_UP ? w->rows / 2 : w->rows;
    TcEpiStore epi{dev_y, (int64_t)w->rows, w->rowmap, m->host.D, src_rows};
    if (e == cudaSuccess) e = tc_gemm(mats, 1, x16, ldx, xs, (int)n_tok, status, m->n_sm, epi, st, &sk);
    if (e == cudaErrorNotSupported) return v3g_fail(V3G_E_UNSUPPORTED, "matrix format has no tensor-core path (F32)");
    if (e != cudaSuccess) return v3g_fail(V3G_E_CUDA, std::string("v3g_gemm: ") + cudaGetErrorString(e));
    return V3G_OK;
}
