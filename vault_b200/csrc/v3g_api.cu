// C ABI of the engine: VLT3 validation and upload, state arena layout, step / prefill / greedy generation.
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <vector>

#include "../../include/vault_b200.h"
#include "v3g_internal.h"

using namespace v3g;

static thread_local std::string g_err;

static int fail(int code, const std::string &msg) {
    g_err = msg;
    return code;
}
#define CUDA_TRY(expr)                                                                          \
    do {                                                                                        \
        cudaError_t e_ = (expr);                                                                \
        if (e_ != cudaSuccess) return fail(V3G_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
    } while (0)

// ------------------------------------------------------------------------------------------ file validation
namespace {

constexpr uint64_t HDR = 4096, ENTRY = 128, FALIGN = 64;
enum { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2, DT_Q8 = 8, DT_Q4 = 9 };

uint32_t rd32(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }
uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
uint64_t rd64(const uint8_t *p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }
float rdf(const uint8_t *p) {
    uint32_t u = rd32(p);
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// CRC-32 (IEEE 802.3 / zlib polynomial, reflected), table built on first use
uint32_t crc32_of(const uint8_t *p, uint64_t n) {
    static uint32_t table[256];
    static bool ready = false;
    if (!ready) {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
            table[i] = c;
        }
        ready = true;
    }
    uint32_t c = 0xFFFFFFFFu;
    for (uint64_t i = 0; i < n; ++i) c = table[(c ^ p[i]) & 0xFF] ^ (c >> 8);
    return c ^ 0xFFFFFFFFu;
}

bool finite_f32_bits(uint32_t u) { return (u & 0x7F800000u) != 0x7F800000u; }
bool finite_f16_bits(uint16_t u) { return (u & 0x7C00u) != 0x7C00u; }
bool finite_bf16_bits(uint16_t u) { return (u & 0x7F80u) != 0x7F80u; }

struct Tensor {
    const uint8_t *data = nullptr;
    uint32_t dtype = 0, ndim = 0, dims[4] = {0, 0, 0, 0};
    uint64_t nbytes = 0;
};

struct Parsed {
    uint32_t vocab, d, L, H, G, D, F, W, n_sink, seg_budget, seg_hidden, seg_min, seg_max, n_feat, seg_layers[4];
    float eps, theta;
    uint32_t bos, eos, im_start, im_end, pad, wfmt, flags;
    Tensor embed, norm, sc[6];
    Tensor lay[MAX_LAYERS][12];
    const uint8_t *tok = nullptr;
    uint64_t tok_size = 0;
};

bool dtype_bytes(uint32_t dt, uint64_t n, uint64_t &out) {
    switch (dt) {
        case DT_F32: if (n > (~0ull) / 4) return false; out = 4 * n; return true;
        case DT_F16:
        case DT_BF16: if (n > (~0ull) / 2) return false; out = 2 * n; return true;
        case DT_Q8: if (n % 32) return false; out = n / 32 * 34; return true;
        case DT_Q4: if (n % 32) return false; out = n / 32 * 18; return true;
        default: return false;
    }
}

bool tensor_finite(const uint8_t *p, uint32_t dt, uint64_t n) {
    switch (dt) {
        case DT_F32: for (uint64_t i = 0; i < n; ++i) if (!finite_f32_bits(rd32(p + 4 * i))) return false; return true;
        case DT_F16: for (uint64_t i = 0; i < n; ++i) if (!finite_f16_bits(rd16(p + 2 * i))) return false; return true;
        case DT_BF16: for (uint64_t i = 0; i < n; ++i) if (!finite_bf16_bits(rd16(p + 2 * i))) return false; return true;
        case DT_Q8: for (uint64_t b = 0; b < n / 32; ++b) if (!finite_f16_bits(rd16(p + 34 * b))) return false; return true;
        case DT_Q4: for (uint64_t b = 0; b < n / 32; ++b) if (!finite_f16_bits(rd16(p + 18 * b))) return false; return true;
        default: return false;
    }
}

bool shape_is(const Tensor &t, uint32_t ndim, uint64_t d0, uint64_t d1) {
    if (!t.data || t.ndim != ndim || t.dims[0] != d0) return false;
    return ndim < 2 || t.dims[1] == d1;
}
bool mm_dtype(const Tensor &t) { return t.dtype == DT_F32 || t.dtype == DT_F16 || t.dtype == DT_BF16 || t.dtype == DT_Q8 || t.dtype == DT_Q4; }

// Validation rules of runtime/vault3.c:273-455 (v3_load), restated.
int parse_vlt3(const uint8_t *buf, uint64_t size, int verify_crc, Parsed &P) {
    memset(&P, 0, sizeof(P));
    if (!buf || size < HDR) return fail(V3G_E_SIZE, "buffer smaller than the VLT3 header");
    if ((uintptr_t)buf % FALIGN) return fail(V3G_E_ALIGN, "model buffer not 64-byte aligned");
    if (memcmp(buf, "VLT3", 4) || rd32(buf + 4) != 1 || rd32(buf + 8) != HDR || rd32(buf + 12) != 0x01020304u)
        return fail(V3G_E_MAGIC, "bad magic/version/header size/endianness");
    if (crc32_of(buf, HDR - 4) != rd32(buf + HDR - 4)) return fail(V3G_E_CRC, "header CRC mismatch");
    if (rd64(buf + 16) != size) return fail(V3G_E_SIZE, "file_size field != buffer size");
    if (rd32(buf + 24) != FALIGN) return fail(V3G_E_MAGIC, "alignment field != 64");
    const uint32_t n_t = rd32(buf + 28);
    const uint64_t dir = rd64(buf + 32), dir_n = rd64(buf + 40), tok = rd64(buf + 48), tok_n = rd64(buf + 56);
    const uint64_t dat = rd64(buf + 64), dat_n = rd64(buf + 72);
    auto region = [&](uint64_t o, uint64_t n) { return o >= HDR && o <= size && n <= size - o; };
    if (!region(dir, dir_n) || !region(tok, tok_n) || !region(dat, dat_n)) return fail(V3G_E_BOUNDS, "region out of bounds");
    if (n_t > 8192 || dir_n != (uint64_t)n_t * ENTRY) return fail(V3G_E_BOUNDS, "bad tensor directory size");
    P.vocab = rd32(buf + 80); P.d = rd32(buf + 84); P.L = rd32(buf + 88); P.H = rd32(buf + 92);
    P.G = rd32(buf + 96); P.D = rd32(buf + 100); P.F = rd32(buf + 104); P.W = rd32(buf + 108);
    if (rd32(buf + 112) || rd32(buf + 148)) return fail(V3G_E_LIMIT, "non-zero legacy bank fields");
    for (int i = 0; i < 8; ++i)
        if (rd32(buf + 116 + 4 * i)) return fail(V3G_E_LIMIT, "non-zero legacy prime fields");
    P.eps = rdf(buf + 152); P.theta = rdf(buf + 156);
    if (!finite_f32_bits(rd32(buf + 160))) return fail(V3G_E_NAN, "non-finite vault_eps");
    P.bos = rd32(buf + 164); P.eos = rd32(buf + 168); P.im_start = rd32(buf + 172); P.im_end = rd32(buf + 176);
    P.pad = rd32(buf + 180); P.wfmt = rd32(buf + 184); P.flags = rd32(buf + 188);
    P.n_sink = rd32(buf + 256); P.seg_budget = rd32(buf + 260); P.seg_hidden = rd32(buf + 264);
    P.seg_min = rd32(buf + 268); P.seg_max = rd32(buf + 272); P.n_feat = rd32(buf + 276);
    for (int i = 0; i < 4; ++i) P.seg_layers[i] = rd32(buf + 280 + 4 * i);
    if (P.vocab == 0 || P.vocab > 524288 || P.d == 0 || P.d > 16384 || P.L == 0 || P.L > MAX_LAYERS || P.H == 0 ||
        P.H > 256 || P.D == 0 || P.D > 256 || (P.D & 1) || P.G == 0 || P.G > P.H || P.H % P.G || P.F == 0 ||
        P.F > 65536 || P.W == 0 || P.W > 65536 || P.n_sink > 512 || P.n_sink > P.W)
        return fail(V3G_E_LIMIT, "hyper-parameter out of range");
    if ((uint64_t)P.H * P.D != P.d) return fail(V3G_E_SHAPE, "n_heads * head_dim != d_model");
    if (!finite_f32_bits(rd32(buf + 152)) || !finite_f32_bits(rd32(buf + 156))) return fail(V3G_E_NAN, "non-finite eps/theta");
    if (!(P.theta > 1.0f) || !(P.eps > 0.0f)) return fail(V3G_E_LIMIT, "invalid eps/theta");
    if (P.bos >= P.vocab || P.eos >= P.vocab || P.im_start >= P.vocab || P.im_end >= P.vocab || P.pad >= P.vocab)
        return fail(V3G_E_LIMIT, "special token id >= vocab");
    if (P.n_feat > 4) return fail(V3G_E_LIMIT, "seg_n_feat > 4");
    if (P.n_feat == 0) {
        if (P.seg_budget || P.seg_hidden || P.seg_min || P.seg_max) return fail(V3G_E_LIMIT, "segment fields without scorer");
    } else {
        if (P.seg_budget > MAX_SEG_BUDGET || P.seg_hidden == 0 || P.seg_hidden > 1024 || P.seg_min == 0 ||
            P.seg_min > P.seg_max || P.seg_max > P.W)
            return fail(V3G_E_LIMIT, "invalid segment scorer hyper-parameters");
        for (uint32_t i = 0; i < P.n_feat; ++i)
            if (P.seg_layers[i] >= P.L) return fail(V3G_E_LIMIT, "scorer feature layer out of range");
    }
    uint64_t prev_end = 0;
    for (uint32_t i = 0; i < n_t; ++i) {
        const uint8_t *e = buf + dir + (uint64_t)i * ENTRY;
        const uint32_t id = rd32(e), dt = rd32(e + 4), ndim = rd32(e + 8);
        uint32_t dims[4] = {rd32(e + 12), rd32(e + 16), rd32(e + 20), rd32(e + 24)};
        const uint64_t off = rd64(e + 32), nb = rd64(e + 40);
        if (rd32(e + 28)) return fail(V3G_E_BOUNDS, "reserved directory field not zero");
        if (ndim < 1 || ndim > 4) return fail(V3G_E_SHAPE, "bad ndim");
        uint64_t n = 1;
        for (uint32_t k = 0; k < ndim; ++k) {
            if (dims[k] == 0 || n > (~0ull) / dims[k]) return fail(V3G_E_SHAPE, "zero or overflowing dims");
            n *= dims[k];
        }
        uint64_t want;
        if (!dtype_bytes(dt, n, want)) return fail(V3G_E_DTYPE, "unsupported dtype");
        if ((dt == DT_Q8 || dt == DT_Q4) && dims[ndim - 1] % 32) return fail(V3G_E_SHAPE, "quantized row not a multiple of 32");
        if (want != nb) return fail(V3G_E_SHAPE, "nbytes inconsistent with dtype/dims");
        if (off % FALIGN || off < dat || nb > dat + dat_n - off) return fail(V3G_E_BOUNDS, "tensor outside data region");
        if (off < prev_end) return fail(V3G_E_BOUNDS, "overlapping or unordered tensors");
        prev_end = off + nb;
        if (verify_crc && crc32_of(buf + off, nb) != rd32(e + 48)) return fail(V3G_E_CRC, "tensor CRC mismatch");
        if (!tensor_finite(buf + off, dt, n)) return fail(V3G_E_NAN, "non-finite weight or scale");
        Tensor *dst = nullptr;
        if (id < 256) {
            if (id == 1) dst = &P.embed;
            else if (id == 2) dst = &P.norm;
            else if (P.n_feat > 0 && id >= 4 && id <= 9) dst = &P.sc[id - 4];
        } else {
            const uint32_t l = (id >> 8) - 1, kind = id & 0xFF;
            if (l >= P.L) return fail(V3G_E_MISSING, "tensor for a layer out of range");
            if (kind >= 1 && kind <= 12) dst = &P.lay[l][kind - 1];
        }
        if (!dst || dst->data) return fail(V3G_E_MISSING, "unknown or duplicate tensor id");
        dst->data = buf + off;
        dst->dtype = dt;
        dst->ndim = ndim;
        dst->nbytes = nb;
        memcpy(dst->dims, dims, sizeof(dims));
    }
    const uint64_t d = P.d, H = P.H, G = P.G, D = P.D, F = P.F;
    if (!shape_is(P.embed, 2, P.vocab, d) || !mm_dtype(P.embed)) return fail(V3G_E_SHAPE, "embed_tokens shape/dtype");
    if (!shape_is(P.norm, 1, d, 0) || P.norm.dtype != DT_F32) return fail(V3G_E_SHAPE, "norm shape/dtype");
    if (P.n_feat > 0) {
        const uint64_t fd = (uint64_t)P.n_feat * d, hd = P.seg_hidden;
        const Tensor *s = P.sc;
        if (!shape_is(s[0], 1, fd, 0) || s[0].dtype != DT_F32 || !shape_is(s[1], 1, fd, 0) || s[1].dtype != DT_F32 ||
            !shape_is(s[2], 2, hd, fd) || !mm_dtype(s[2]) || !shape_is(s[3], 1, hd, 0) || s[3].dtype != DT_F32 ||
            !shape_is(s[4], 2, 1, hd) || !mm_dtype(s[4]) || !shape_is(s[5], 1, 1, 0) || s[5].dtype != DT_F32)
            return fail(V3G_E_SHAPE, "segment scorer shape/dtype");
    }
    for (uint32_t l = 0; l < P.L; ++l) {
        const Tensor *t = P.lay[l];
        const bool ok = shape_is(t[0], 1, d, 0) && t[0].dtype == DT_F32 && shape_is(t[8], 1, d, 0) && t[8].dtype == DT_F32 &&
                        shape_is(t[1], 2, H * D, d) && mm_dtype(t[1]) && shape_is(t[3], 2, G * D, d) && mm_dtype(t[3]) &&
                        shape_is(t[5], 2, G * D, d) && mm_dtype(t[5]) && shape_is(t[7], 2, d, H * D) && mm_dtype(t[7]) &&
                        shape_is(t[9], 2, F, d) && mm_dtype(t[9]) && shape_is(t[10], 2, F, d) && mm_dtype(t[10]) &&
                        shape_is(t[11], 2, d, F) && mm_dtype(t[11]) && shape_is(t[2], 1, H * D, 0) && t[2].dtype == DT_F32 &&
                        shape_is(t[4], 1, G * D, 0) && t[4].dtype == DT_F32 && shape_is(t[6], 1, G * D, 0) && t[6].dtype == DT_F32;
        if (!ok) return fail(V3G_E_SHAPE, "layer " + std::to_string(l) + " tensor shape/dtype");
    }
    // tokenizer blob (runtime/vault3.c:410-452)
    const uint8_t *tb = buf + tok;
    if (tok_n < 128 || memcmp(tb, "VTOK", 4) || rd32(tb + 4) != 1) return fail(V3G_E_TOKENIZER, "bad tokenizer header");
    const uint32_t nv = rd32(tb + 8), nm = rd32(tb + 12), ns = rd32(tb + 16), nr = rd32(tb + 20);
    if (nv == 0 || nv > P.vocab || nm > 2097152u || ns > nv || nr > 65536u) return fail(V3G_E_TOKENIZER, "bad tokenizer counts");
    const uint64_t o_tab = rd64(tb + 28), o_pool = rd64(tb + 36), o_mer = rd64(tb + 44), o_spc = rd64(tb + 52),
                   o_rng = rd64(tb + 60), o_byt = rd64(tb + 68);
    auto treg = [&](uint64_t o, uint64_t n) { return o % 4 == 0 && o <= tok_n && n <= tok_n - o; };
    if (!treg(o_tab, (uint64_t)nv * 8) || !treg(o_mer, (uint64_t)nm * 12) || !treg(o_spc, (uint64_t)ns * 4) ||
        !treg(o_rng, (uint64_t)nr * 12) || !treg(o_byt, 1024) || o_pool > o_mer || o_pool < o_tab + (uint64_t)nv * 8)
        return fail(V3G_E_TOKENIZER, "tokenizer section out of range");
    const uint64_t pool_n = o_mer - o_pool;
    for (uint32_t i = 0; i < nv; ++i) {
        const uint64_t so = rd32(tb + o_tab + 8ull * i), sl = rd32(tb + o_tab + 8ull * i + 4);
        if (so > pool_n || sl > pool_n - so) return fail(V3G_E_TOKENIZER, "token string out of pool");
    }
    for (uint32_t i = 0; i < nm; ++i)
        for (int k = 0; k < 3; ++k)
            if (rd32(tb + o_mer + 12ull * i + 4 * k) >= nv) return fail(V3G_E_TOKENIZER, "merge id out of range");
    for (uint32_t i = 0; i < ns; ++i)
        if (rd32(tb + o_spc + 4ull * i) >= nv) return fail(V3G_E_TOKENIZER, "special id out of range");
    for (uint32_t i = 0; i < 256; ++i)
        if (rd32(tb + o_byt + 4ull * i) >= nv) return fail(V3G_E_TOKENIZER, "byte token id out of range");
    P.tok = tb;
    P.tok_size = tok_n;
    return V3G_OK;
}

// 3-tier segment-break class of a token's bytes (src/vault_v3_model.py:116-142, runtime/vault3.c:937-959)
int break_tier(const uint8_t *b, uint32_t n) {
    if (n == 0) return 0;
    bool t2 = false, t3 = false;
    for (uint32_t i = 0; i < n; ++i) {
        const uint8_t ch = b[i];
        if (ch == '\n') return 1;
        if (ch == '}' || ch == ']' || ch == '|' || ch == '\t') t2 = true;
        else if (ch == '"' && i + 1 < n && b[i + 1] == ',') t2 = true;
        else if (ch == ',' || ch == '&') t3 = true;
    }
    uint32_t end = n;
    while (end > 0 && (b[end - 1] == ' ' || b[end - 1] == '\t' || b[end - 1] == '\r' || b[end - 1] == 0x0B || b[end - 1] == 0x0C)) --end;
    const uint8_t last = end ? b[end - 1] : 0;
    if (last == '.' || last == '!' || last == '?' || last == ';') return 1;
    return t2 ? 2 : (t3 ? 3 : 0);
}

}  // namespace

// ------------------------------------------------------------------------------------------ model load
extern "C" int v3g_validate(const uint8_t *buf, uint64_t size, int verify_crc) {
    Parsed *P = new Parsed();   // large (per-layer tensor table): keep it off the caller's stack
    const int rc = parse_vlt3(buf, size, verify_crc, *P);
    delete P;
    return rc;
}

// A VLT3 file mapped read-only for the length of one call (page-aligned, so the format's alignment rule holds
// without a host copy); the loader reads the mapping directly.
struct MappedFile {
    const uint8_t *data = nullptr;
    uint64_t size = 0;
    int open_file(const char *path) {
        if (!path) return fail(V3G_E_ARG, "null path");
        const int fd = open(path, O_RDONLY | O_CLOEXEC);
        if (fd < 0) return fail(V3G_E_ARG, std::string("cannot open ") + path);
        struct stat sb;
        if (fstat(fd, &sb) != 0 || sb.st_size <= 0) {
            close(fd);
            return fail(V3G_E_SIZE, std::string("empty or unreadable file ") + path);
        }
        void *p = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
        close(fd);
        if (p == MAP_FAILED) return fail(V3G_E_ARG, std::string("cannot map ") + path);
        madvise(p, (size_t)sb.st_size, MADV_SEQUENTIAL);
        data = static_cast<const uint8_t *>(p);
        size = (uint64_t)sb.st_size;
        return V3G_OK;
    }
    ~MappedFile() {
        if (data) munmap(const_cast<uint8_t *>(data), (size_t)size);
    }
};

extern "C" int v3g_validate_file(const char *path, int verify_crc) {
    MappedFile f;
    const int rc = f.open_file(path);
    return rc != V3G_OK ? rc : v3g_validate(f.data, f.size, verify_crc);
}

extern "C" int v3g_load_file(v3g_model **out, const char *path, int verify_crc, int device, uint32_t max_sink) {
    MappedFile f;
    const int rc = f.open_file(path);
    return rc != V3G_OK ? rc : v3g_load(out, f.data, f.size, verify_crc, device, max_sink);
}

// the VTOK tokenizer blob of a validated VLT3 buffer (a pointer into buf)
int vlt3_token_blob(const uint8_t *buf, uint64_t size, const uint8_t **tok, uint64_t *tok_size) {
    Parsed *P = new Parsed();
    const int rc = parse_vlt3(buf, size, 0, *P);
    *tok = P->tok;
    *tok_size = P->tok_size;
    delete P;
    return rc;
}

extern "C" int v3g_load(v3g_model **out, const uint8_t *buf, uint64_t size, int verify_crc, int device,
                        uint32_t max_sink) {
    if (!out) return fail(V3G_E_ARG, "null output pointer");
    *out = nullptr;
    Parsed *Pp = new Parsed();
    Parsed &P = *Pp;
    int rc = parse_vlt3(buf, size, verify_crc, P);
    if (rc != V3G_OK) {
        delete Pp;
        return rc;
    }
    const int grp = (int)(P.H / P.G);
    if (grp > 8 || !(P.D == 16 || P.D == 32 || P.D == 64 || P.D == 128) || P.d % 32 || P.F % 32) {
        delete Pp;
        return fail(V3G_E_UNSUPPORTED, "engine supports head_dim in {16,32,64,128}, <= 8 query heads per KV "
                                       "head, d_model and d_ff multiples of 32");
    }
    for (uint32_t l = 0; l < P.L; ++l)
        if (P.lay[l][9].dtype != P.lay[l][10].dtype) {
            delete Pp;
            return fail(V3G_E_UNSUPPORTED, "gate_proj and up_proj of a layer must share a dtype");
        }
    if (max_sink == 0) max_sink = 512;
    if (cudaSetDevice(device) != cudaSuccess) {
        delete Pp;
        return fail(V3G_E_CUDA, "cudaSetDevice failed");
    }
    if (cudaError_t ea = init_kernel_attrs()) {
        delete Pp;
        return fail(V3G_E_CUDA, std::string("kernel attributes: ") + cudaGetErrorString(ea));
    }
    v3g_model *m = new v3g_model();
    m->device = device;
    cudaDeviceGetAttribute(&m->n_sm, cudaDevAttrMultiProcessorCount, device);
    ModelDev &md = m->host;
    memset(&md, 0, sizeof(md));
    md.vocab = P.vocab; md.d = P.d; md.n_layers = P.L; md.H = P.H; md.G = P.G; md.D = P.D; md.F = P.F; md.W = P.W;
    md.rms_eps = P.eps; md.rope_theta = P.theta; md.pad_id = P.pad; md.im_start_id = P.im_start; md.im_end_id = P.im_end;
    md.n_sink = P.n_sink;
    md.max_sink = (int)std::min<uint32_t>(max_sink, MAX_SINK);
    md.sink_cap = std::max<int>(1, std::max<int>((int)P.n_sink, md.max_sink));
    md.seg_n_feat = P.n_feat; md.seg_hidden = P.seg_hidden; md.seg_min = P.seg_min; md.seg_max = P.seg_max;
    md.seg_budget_default = P.n_feat ? P.seg_budget : 0;
    for (int i = 0; i < 4; ++i) md.seg_layers[i] = P.seg_layers[i];
    m->bos_id = P.bos; m->eos_id = P.eos; m->weight_format = P.wfmt; m->flags = P.flags;
    m->file_seg_budget = P.seg_budget;

    // token tables: bytes, tiers, "\n" / "system" ids (runtime/vault3.c:1920-1928, 2047)
    const uint8_t *tb = P.tok;
    const uint32_t nv = rd32(tb + 8);
    const uint64_t o_tab = rd64(tb + 28), o_pool = rd64(tb + 36), o_mer = rd64(tb + 44), o_byt = rd64(tb + 68);
    std::vector<uint8_t> tier(P.vocab, 0);
    std::vector<uint32_t> toff(P.vocab, 0);
    std::vector<uint16_t> tlen(P.vocab, 0);
    const uint8_t *pool = tb + o_pool;
    const uint64_t pool_n = o_mer - o_pool;
    int system_id = 8948;
    bool system_found = false;
    for (uint32_t i = 0; i < nv; ++i) {
        const uint32_t so = rd32(tb + o_tab + 8ull * i), sl = rd32(tb + o_tab + 8ull * i + 4);
        tier[i] = (uint8_t)break_tier(pool + so, sl);
        toff[i] = so;
        tlen[i] = (uint16_t)std::min<uint32_t>(sl, 65535);
        if (!system_found && (sl == 6 || (sl == 7 && pool[so + 6] == '\n')) && memcmp(pool + so, "system", 6) == 0) {
            system_id = (int)i;
            system_found = true;
        }
    }
    md.system_id = system_id;
    md.newline_id = (int)rd32(tb + o_byt + 4 * '\n');

    // RoPE table, positions [-(sink_cap + MAX_SEG_BUDGET), 2W), fp32 angles as the reference computes them
    const int hd = P.D / 2;
    md.rope_pos0 = -(md.sink_cap + MAX_SEG_BUDGET);
    md.rope_rows = 2 * (int)P.W - md.rope_pos0;
    std::vector<float> rope((size_t)md.rope_rows * P.D);
    {
        std::vector<float> inv(hd);
        for (int i = 0; i < hd; ++i) {
            const float ex = (float)(2 * i) / (float)P.D;
            inv[i] = 1.0f / powf(P.theta, ex);
        }
        for (int r = 0; r < md.rope_rows; ++r) {
            const float p = (float)(md.rope_pos0 + r);
            for (int i = 0; i < hd; ++i) {
                const float ang = p * inv[i];
                rope[(size_t)r * P.D + i] = (float)cos((double)ang);
                rope[(size_t)r * P.D + hd + i] = (float)sin((double)ang);
            }
        }
    }

    // device memory plan
    struct Job { MatW *w; const Tensor *a, *b; int rowmap; uint64_t off; };
    std::vector<Job> jobs;
    uint64_t total = 0;
    auto take = [&](uint64_t n) { uint64_t o = total; total = (total + n + 255) & ~255ull; return o; };
    auto add_mat = [&](MatW *w, const Tensor *a, const Tensor *b, int rowmap) {
        const int rows = (int)a->dims[0] * (b ? 2 : 1), cols = (int)a->dims[1];
        jobs.push_back({w, a, b, rowmap, take(matrix_tile_bytes((int)a->dtype, rows, cols))});
        w->file_bytes = a->nbytes + (b ? b->nbytes : 0);
    };
    for (uint32_t l = 0; l < P.L; ++l) {
        LayerW &L = md.layers[l];
        add_mat(&L.q, &P.lay[l][1], nullptr, ROWS_ROPE_PAIRS);
        add_mat(&L.k, &P.lay[l][3], nullptr, ROWS_ROPE_PAIRS);
        add_mat(&L.v, &P.lay[l][5], nullptr, ROWS_ROPE_PAIRS);
        add_mat(&L.o, &P.lay[l][7], nullptr, ROWS_IDENTITY);
        add_mat(&L.gu, &P.lay[l][9], &P.lay[l][10], ROWS_GATE_UP);
        add_mat(&L.down, &P.lay[l][11], nullptr, ROWS_IDENTITY);
    }
    add_mat(&md.embed, &P.embed, nullptr, ROWS_IDENTITY);
    struct VecJob { const float **dst; const void *src; uint64_t n; uint64_t off; };
    std::vector<VecJob> vecs;
    auto add_vec = [&](const float **dst, const void *src, uint64_t nbytes) { vecs.push_back({dst, src, nbytes, take(nbytes)}); };
    for (uint32_t l = 0; l < P.L; ++l) {
        LayerW &L = md.layers[l];
        add_vec(&L.ln1, P.lay[l][0].data, P.lay[l][0].nbytes);
        add_vec(&L.bq, P.lay[l][2].data, P.lay[l][2].nbytes);
        add_vec(&L.bk, P.lay[l][4].data, P.lay[l][4].nbytes);
        add_vec(&L.bv, P.lay[l][6].data, P.lay[l][6].nbytes);
        add_vec(&L.ln2, P.lay[l][8].data, P.lay[l][8].nbytes);
    }
    add_vec(&md.norm, P.norm.data, P.norm.nbytes);
    // the scorer runs on CUDA cores in fp32: store fc1 / fc2 as fp32 rows whatever their file dtype
    std::vector<float> sc_w1, sc_w2;
    if (P.n_feat) {
        auto widen = [&](const Tensor &t, std::vector<float> &o) {
            const uint64_t n = (uint64_t)t.dims[0] * t.dims[1];
            o.resize(n);
            for (uint64_t i = 0; i < n; ++i) {
                switch (t.dtype) {
                    case DT_F32: o[i] = rdf(t.data + 4 * i); break;
                    case DT_BF16: { uint32_t u = (uint32_t)rd16(t.data + 2 * i) << 16; memcpy(&o[i], &u, 4); break; }
                    case DT_F16: { __half h = __ushort_as_half(rd16(t.data + 2 * i)); o[i] = __half2float(h); break; }
                    case DT_Q8: {
                        const uint8_t *blk = t.data + (i / 32) * 34;
                        o[i] = (float)(int8_t)blk[2 + i % 32] * __half2float(__ushort_as_half(rd16(blk)));
                        break;
                    }
                    default: {
                        const uint8_t *blk = t.data + (i / 32) * 18;
                        const int j = (int)(i % 32);
                        const int nib = j < 16 ? (blk[2 + j] & 15) : (blk[2 + j - 16] >> 4);
                        o[i] = (float)(nib - 8) * __half2float(__ushort_as_half(rd16(blk)));
                    }
                }
            }
        };
        widen(P.sc[2], sc_w1);
        widen(P.sc[4], sc_w2);
        add_vec(&md.sc_ln_w, P.sc[0].data, P.sc[0].nbytes);
        add_vec(&md.sc_ln_b, P.sc[1].data, P.sc[1].nbytes);
        add_vec(&md.sc_w1, sc_w1.data(), sc_w1.size() * 4);
        add_vec(&md.sc_b1, P.sc[3].data, P.sc[3].nbytes);
        add_vec(&md.sc_w2, sc_w2.data(), sc_w2.size() * 4);
        add_vec(&md.sc_b2, P.sc[5].data, P.sc[5].nbytes);
    }
    add_vec(&md.rope, rope.data(), rope.size() * 4);
    const uint64_t off_tier = take(P.vocab), off_toff = take((uint64_t)P.vocab * 4), off_tlen = take((uint64_t)P.vocab * 2);
    const uint64_t off_pool = take(pool_n + 16);
    m->weight_alloc = total;

    uint64_t staging_n = 0;
    for (auto &j : jobs) staging_n = std::max<uint64_t>(staging_n, j.a->nbytes + (j.b ? j.b->nbytes : 0));
    uint8_t *staging = nullptr;
    cudaStream_t st = nullptr;
    auto cleanup_fail = [&](int code, const std::string &msg) {
        if (staging) cudaFree(staging);
        if (st) cudaStreamDestroy(st);
        if (m->weights) cudaFree(m->weights);
        delete m;
        delete Pp;
        return fail(code, msg);
    };
    if (cudaMalloc(&m->weights, total) != cudaSuccess) return cleanup_fail(V3G_E_CUDA, "cudaMalloc(weights) failed");
    if (cudaMalloc(&staging, staging_n) != cudaSuccess) return cleanup_fail(V3G_E_CUDA, "cudaMalloc(staging) failed");
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) return cleanup_fail(V3G_E_CUDA, "stream");
    for (auto &j : jobs) {
        const int rows = (int)j.a->dims[0], cols = (int)j.a->dims[1];
        if (cudaMemcpyAsync(staging, j.a->data, j.a->nbytes, cudaMemcpyHostToDevice, st) != cudaSuccess)
            return cleanup_fail(V3G_E_CUDA, "upload failed");
        if (j.b && cudaMemcpyAsync(staging + j.a->nbytes, j.b->data, j.b->nbytes, cudaMemcpyHostToDevice, st) != cudaSuccess)
            return cleanup_fail(V3G_E_CUDA, "upload failed");
        if (repack_matrix(*j.w, staging, j.b ? staging + j.a->nbytes : nullptr, (int)j.a->dtype, rows, cols, j.rowmap,
                          (int)P.D, m->weights + j.off, st))
            return cleanup_fail(V3G_E_CUDA, "repack launch failed");
        if (cudaStreamSynchronize(st) != cudaSuccess) return cleanup_fail(V3G_E_CUDA, "repack failed");
    }
    for (auto &v : vecs) {
        if (cudaMemcpyAsync(m->weights + v.off, v.src, v.n, cudaMemcpyHostToDevice, st) != cudaSuccess)
            return cleanup_fail(V3G_E_CUDA, "upload failed");
        *v.dst = reinterpret_cast<const float *>(m->weights + v.off);
    }
    cudaMemcpyAsync(m->weights + off_tier, tier.data(), P.vocab, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(m->weights + off_toff, toff.data(), (size_t)P.vocab * 4, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(m->weights + off_tlen, tlen.data(), (size_t)P.vocab * 2, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(m->weights + off_pool, pool, pool_n, cudaMemcpyHostToDevice, st);
    md.tier = m->weights + off_tier;
    md.tok_off = reinterpret_cast<const uint32_t *>(m->weights + off_toff);
    md.tok_len = reinterpret_cast<const uint16_t *>(m->weights + off_tlen);
    md.tok_pool = m->weights + off_pool;
    if (cudaMalloc(&m->dev, sizeof(ModelDev)) != cudaSuccess) return cleanup_fail(V3G_E_CUDA, "cudaMalloc(desc)");
    cudaMemcpyAsync(m->dev, &md, sizeof(ModelDev), cudaMemcpyHostToDevice, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) return cleanup_fail(V3G_E_CUDA, "upload failed");
    cudaFree(staging);
    cudaStreamDestroy(st);

    // bookkeeping: algorithmic bytes per decode step, tensor index for tests
    uint64_t per_step = P.norm.nbytes;
    for (uint32_t l = 0; l < P.L; ++l)
        for (int k = 0; k < 12; ++k) per_step += P.lay[l][k].nbytes;
    m->step_bytes_lm = P.embed.nbytes;
    m->step_bytes = per_step + P.embed.nbytes;
    m->scorer_bytes = 0;
    for (int i = 0; i < 6 && P.n_feat; ++i) m->scorer_bytes += P.sc[i].nbytes;
    for (uint32_t l = 0; l < P.L; ++l) {
        LayerW &L = md.layers[l];
        const uint32_t base = (l + 1) << 8;
        m->tensor_index.push_back({base | 2, &L.q});
        m->tensor_index.push_back({base | 4, &L.k});
        m->tensor_index.push_back({base | 6, &L.v});
        m->tensor_index.push_back({base | 8, &L.o});
        m->tensor_index.push_back({base | 10, &L.gu});
        m->tensor_index.push_back({base | 11, &L.gu});
        m->tensor_index.push_back({base | 12, &L.down});
    }
    m->tensor_index.push_back({1u, &md.embed});
    delete Pp;
    *out = m;
    return V3G_OK;
}

extern "C" int v3g_model_get_info(const v3g_model *m, v3g_model_info *o) {
    if (!m || !o) return fail(V3G_E_ARG, "null argument");
    const ModelDev &md = m->host;
    memset(o, 0, sizeof(*o));
    o->vocab_size = md.vocab; o->d_model = md.d; o->n_layers = md.n_layers; o->n_heads = md.H; o->n_kv_heads = md.G;
    o->head_dim = md.D; o->d_ff = md.F; o->window = md.W; o->rms_eps = md.rms_eps; o->rope_theta = md.rope_theta;
    o->bos_id = m->bos_id; o->eos_id = m->eos_id; o->im_start_id = md.im_start_id; o->im_end_id = md.im_end_id;
    o->pad_id = md.pad_id; o->weight_format = m->weight_format; o->flags = m->flags; o->n_sink = md.n_sink;
    o->seg_budget = md.seg_budget_default; o->seg_hidden = md.seg_hidden; o->seg_min = md.seg_min;
    o->seg_max = md.seg_max; o->seg_n_feat = md.seg_n_feat;
    for (int i = 0; i < 4; ++i) o->seg_layers[i] = md.seg_layers[i];
    o->sink_cap = md.sink_cap;
    o->step_weight_bytes = m->step_bytes;
    o->lm_head_bytes = m->step_bytes_lm;
    o->scorer_bytes = m->scorer_bytes;
    o->device_bytes = m->weight_alloc;
    return V3G_OK;
}

extern "C" void v3g_free(v3g_model *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->weights) cudaFree(m->weights);
    if (m->dev) cudaFree(m->dev);
    delete m;
}

// ------------------------------------------------------------------------------------------ state
namespace {

struct Layout {
    uint64_t lb_stride, off_ring, ring_kind, ring_par, off_sink, off_bank, bank_par, off_bank_rot;
    uint64_t kv_bytes;
    uint64_t off_seq, off_step, off_tok_in, off_tok_ring, off_sc_ring, off_seg_ring, off_mem_pos, off_mem_score,
        off_mem_tok, off_mem_seg, off_mem_src, off_ema, off_feat, off_x, off_attn, off_h, off_qc, off_qf, off_part,
        off_cnt, off_logits, off_amax, off_scz, off_bar;
    // chunked-prefill workspace: pf_cap tokens
    uint64_t off_pf_x, off_pf_qc, off_pf_qf, off_pf_attn, off_pf_h, off_pf_x16, off_pf_xs, off_pf_feat, off_pf_hin,
        off_pf_z, off_pf_stat, off_pf_skws;
    int pf_cap, pf_ldx16;
    uint64_t total;
    int max_splits, seg_cap, feat_dim;
};

Layout make_layout(const ModelDev &md, int B, int seg_cap) {
    Layout L{};
    auto al = [](uint64_t v) { return (v + 255) & ~255ull; };
    const uint64_t row = (uint64_t)md.D * 2, G = md.G;
    L.seg_cap = seg_cap;
    const uint64_t bc = seg_cap > 0 ? seg_cap : 1;
    L.ring_kind = al(G * md.W * row);
    L.ring_par = 3 * L.ring_kind;
    L.off_ring = 0;
    L.off_sink = 2 * L.ring_par;
    const uint64_t sink_b = al(3 * G * md.sink_cap * row);
    L.off_bank = L.off_sink + sink_b;
    L.bank_par = al(2 * G * bc * row);
    L.off_bank_rot = L.off_bank + 2 * L.bank_par;
    L.lb_stride = al(L.off_bank_rot + G * bc * row);
    L.kv_bytes = L.lb_stride * md.n_layers * B;
    const int total_keys = md.sink_cap + seg_cap + 2 * md.W;
    L.max_splits = (total_keys + ATT_KEYS_PER_CTA - 1) / ATT_KEYS_PER_CTA;
    L.feat_dim = md.seg_n_feat > 0 ? md.seg_n_feat * md.d : 1;
    uint64_t cur = al(L.kv_bytes);
    auto take = [&](uint64_t n) { uint64_t o = cur; cur = al(cur + n); return o; };
    const int grp = md.H / md.G;
    L.off_seq = take((uint64_t)B * sizeof(SeqCtl));
    L.off_step = take(sizeof(StepCtl));
    L.off_tok_in = take((uint64_t)B * 4);
    L.off_tok_ring = take((uint64_t)B * 2 * md.W * 4);
    L.off_sc_ring = take((uint64_t)B * 2 * md.W * 4);
    L.off_seg_ring = take((uint64_t)B * 2 * md.W * 4);
    L.off_mem_pos = take((uint64_t)B * 2 * bc * 8);
    L.off_mem_score = take((uint64_t)B * 2 * bc * 4);
    L.off_mem_tok = take((uint64_t)B * 2 * bc * 4);
    L.off_mem_seg = take((uint64_t)B * 2 * bc * 4);
    L.off_mem_src = take((uint64_t)B * bc * 4);
    L.off_ema = take((uint64_t)B * L.feat_dim * 4);
    L.off_feat = take((uint64_t)B * L.feat_dim * 4);
    L.off_x = take((uint64_t)B * md.d * 4);
    L.off_attn = take((uint64_t)B * md.H * md.D * 4);
    L.off_h = take((uint64_t)B * md.F * 4);
    L.off_qc = take((uint64_t)B * md.H * md.D * 4);
    L.off_qf = take((uint64_t)B * md.H * md.D * 4);
    L.off_part = take((uint64_t)B * md.G * L.max_splits * grp * att_part_stride(md.D) * 4);
    L.off_cnt = take((uint64_t)B * md.G * 4);
    L.off_logits = take((uint64_t)B * md.vocab * 4);
    L.off_amax = take((uint64_t)B * 8);
    L.off_scz = take((uint64_t)B * 2 * std::max(1, md.seg_hidden) * 4);
    L.off_bar = take(64);
    // chunked prefill: a piece holds at most min(2048, batch x W) tokens (all sequences together)
    L.pf_cap = (int)std::min<int64_t>(2048, (int64_t)B * md.W);
    const uint64_t T = (uint64_t)L.pf_cap, HD = (uint64_t)md.H * md.D;
    L.pf_ldx16 = (int)((std::max<uint64_t>(std::max<uint64_t>(md.d, HD), md.F) + 63) / 64 * 64);
    L.off_pf_x = take(T * md.d * 4);
    L.off_pf_qc = take(T * HD * 4);
    L.off_pf_qf = take(T * HD * 4);
    L.off_pf_attn = take(T * HD * 4);
    L.off_pf_h = take(T * md.F * 4);
    L.off_pf_x16 = take(T * L.pf_ldx16 * 2);
    L.off_pf_xs = take(T * 4);
    const uint64_t fdim = seg_cap > 0 ? (uint64_t)L.feat_dim : 1;   // scorer buffers only with segment memory
    L.off_pf_feat = take(T * fdim * 4);
    L.off_pf_hin = take(T * fdim * 4);
    L.off_pf_z = take(T * 2 * std::max(1, md.seg_hidden) * 4);
    L.off_pf_stat = take(T * 16);
    L.off_pf_skws = take(TC_SPLITK_WS_BYTES);
    L.total = cur;
    return L;
}

}  // namespace

extern "C" size_t v3g_state_arena_size(const v3g_model *m, uint32_t batch, uint32_t max_seg_budget) {
    if (!m || batch == 0 || batch > 4096 || max_seg_budget > MAX_SEG_BUDGET) return 0;
    const int cap = m->host.seg_n_feat > 0 ? (int)max_seg_budget : 0;
    return (size_t)make_layout(m->host, (int)batch, cap).total;
}

extern "C" int v3g_state_init(v3g_state **out, const v3g_model *m, void *dev_arena, size_t arena_size, uint32_t batch,
                              uint32_t max_seg_budget, uint32_t flags) {
    if (!out || !m || !dev_arena) return fail(V3G_E_ARG, "null argument");
    *out = nullptr;
    if ((uintptr_t)dev_arena % 256) return fail(V3G_E_ARENA, "arena not 256-byte aligned");
    if (batch == 0 || batch > 4096) return fail(V3G_E_ARG, "batch out of range");
    if (max_seg_budget > MAX_SEG_BUDGET) return fail(V3G_E_LIMIT, "segment budget above 16384");
    const ModelDev &md = m->host;
    const int cap = md.seg_n_feat > 0 ? (int)max_seg_budget : 0;
    const Layout L = make_layout(md, (int)batch, cap);
    if (arena_size < L.total) return fail(V3G_E_ARENA, "arena too small");
    v3g_state *s = new v3g_state();
    s->m = m;
    s->arena = static_cast<uint8_t *>(dev_arena);
    s->arena_size = L.total;
    s->B = (int)batch;
    s->seg_cap = cap;
    s->per_seq_memory = (flags & V3G_STATE_PER_SEQ_MEMORY) ? 1 : 0;
    const bool batch_mode_ref = batch > 1 && !s->per_seq_memory;
    s->auto_pin = (flags & V3G_STATE_NO_AUTOPIN) || batch_mode_ref ? 0 : 1;
    // active budget: the file's default clamped to the reserved capacity (runtime/vault3.c:833-834)
    int budget = md.seg_budget_default <= cap ? md.seg_budget_default : cap;
    if (md.seg_n_feat > 0 && md.seg_budget_default == 0 && cap > 0) budget = cap;
    s->seg_budget = batch_mode_ref ? 0 : budget;
    s->use_graphs = (flags & V3G_STATE_NO_GRAPHS) ? 0 : 1;
    s->chunked_prefill = (flags & V3G_STATE_TOKEN_PREFILL) ? 0 : 1;
    s->act_single = (flags & V3G_STATE_FP16_ACTIVATIONS) ? 1 : 0;
    StateDev &sd = s->host;
    memset(&sd, 0, sizeof(sd));
    uint8_t *A = s->arena;
    sd.B = (int)batch; sd.W = md.W; sd.G = md.G; sd.D = md.D; sd.H = md.H; sd.sink_cap = md.sink_cap;
    sd.seg_cap = cap > 0 ? cap : 1;
    sd.feat_dim = L.feat_dim;
    sd.max_splits = L.max_splits;
    sd.lb_stride = L.lb_stride;
    sd.kv = A;
    sd.off_ring = L.off_ring; sd.ring_kind_stride = L.ring_kind; sd.ring_par_stride = L.ring_par;
    sd.off_sink = L.off_sink; sd.off_bank = L.off_bank; sd.bank_par_stride = L.bank_par; sd.off_bank_rot = L.off_bank_rot;
    sd.seq = reinterpret_cast<SeqCtl *>(A + L.off_seq);
    sd.step = reinterpret_cast<StepCtl *>(A + L.off_step);
    sd.tok_in = reinterpret_cast<int32_t *>(A + L.off_tok_in);
    sd.tok_ring = reinterpret_cast<int32_t *>(A + L.off_tok_ring);
    sd.sc_ring = reinterpret_cast<float *>(A + L.off_sc_ring);
    sd.seg_ring = reinterpret_cast<int32_t *>(A + L.off_seg_ring);
    sd.mem_pos = reinterpret_cast<int64_t *>(A + L.off_mem_pos);
    sd.mem_score = reinterpret_cast<float *>(A + L.off_mem_score);
    sd.mem_tok = reinterpret_cast<int32_t *>(A + L.off_mem_tok);
    sd.mem_seg = reinterpret_cast<int32_t *>(A + L.off_mem_seg);
    sd.mem_src = reinterpret_cast<int32_t *>(A + L.off_mem_src);
    sd.ema = reinterpret_cast<float *>(A + L.off_ema);
    sd.feat = reinterpret_cast<float *>(A + L.off_feat);
    sd.x = reinterpret_cast<float *>(A + L.off_x);
    sd.attn = reinterpret_cast<float *>(A + L.off_attn);
    sd.hbuf = reinterpret_cast<float *>(A + L.off_h);
    sd.q_cur = reinterpret_cast<float *>(A + L.off_qc);
    sd.q_far = reinterpret_cast<float *>(A + L.off_qf);
    sd.att_part = reinterpret_cast<float *>(A + L.off_part);
    sd.att_cnt = reinterpret_cast<uint32_t *>(A + L.off_cnt);
    sd.logits = reinterpret_cast<float *>(A + L.off_logits);
    sd.amax = reinterpret_cast<unsigned long long *>(A + L.off_amax);
    sd.sc_z = reinterpret_cast<float *>(A + L.off_scz);
    sd.bar = reinterpret_cast<unsigned int *>(A + L.off_bar);
    s->pf.cap = L.pf_cap;
    s->pf.x = reinterpret_cast<float *>(A + L.off_pf_x);
    s->pf.qc = reinterpret_cast<float *>(A + L.off_pf_qc);
    s->pf.qf = reinterpret_cast<float *>(A + L.off_pf_qf);
    s->pf.attn = reinterpret_cast<float *>(A + L.off_pf_attn);
    s->pf.h = reinterpret_cast<float *>(A + L.off_pf_h);
    s->pf.x16 = reinterpret_cast<__half *>(A + L.off_pf_x16);
    s->pf.ldx16 = L.pf_ldx16;
    s->pf.xscale = reinterpret_cast<float *>(A + L.off_pf_xs);
    s->pf.feat = reinterpret_cast<float *>(A + L.off_pf_feat);
    s->pf.hin = reinterpret_cast<float *>(A + L.off_pf_hin);
    s->pf.z = reinterpret_cast<float *>(A + L.off_pf_z);
    s->pf.stat = reinterpret_cast<float4 *>(A + L.off_pf_stat);
    s->pf.sk.ws = reinterpret_cast<float *>(A + L.off_pf_skws);
    s->pf.sk.ws_bytes = TC_SPLITK_WS_BYTES;
    if (cudaSetDevice(m->device) != cudaSuccess || cudaMalloc(&s->dev, sizeof(StateDev)) != cudaSuccess ||
        cudaMemcpy(s->dev, &sd, sizeof(StateDev), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaStreamCreateWithFlags(&s->cap_stream, cudaStreamNonBlocking) != cudaSuccess) {
        if (s->dev) cudaFree(s->dev);
        delete s;
        return fail(V3G_E_CUDA, "state descriptor setup failed");
    }
    if (const cudaError_t ea = tc_init_attrs()) {
        v3g_state_free(s);
        return fail(V3G_E_CUDA, std::string("tensor-core kernel attributes: ") + cudaGetErrorString(ea));
    }
    if (!(flags & V3G_STATE_NO_PERSISTENT)) {
        const cudaError_t em = build_mega(m, s);
        if (em != cudaSuccess) {
            v3g_state_free(s);
            return fail(V3G_E_CUDA, std::string("persistent kernel setup: ") + cudaGetErrorString(em));
        }
        s->use_tc_step = !s->use_mega && (int)batch > GEMV_MB && step_tc_supported(m, s) ? 1 : 0;
    }
    int rc = v3g_state_reset(s, nullptr);
    if (rc != V3G_OK) {
        v3g_state_free(s);
        return rc;
    }
    if (cudaDeviceSynchronize() != cudaSuccess) {
        v3g_state_free(s);
        return fail(V3G_E_CUDA, "state reset failed");
    }
    *out = s;
    return V3G_OK;
}

static void drop_graphs(v3g_state *s) {
    for (auto &g : s->graphs)
        if (g) {
            cudaGraphExecDestroy(g);
            g = nullptr;
        }
}

extern "C" void v3g_state_free(v3g_state *s) {
    if (!s) return;
    cudaSetDevice(s->m->device);
    drop_graphs(s);
    if (s->cap_stream) cudaStreamDestroy(s->cap_stream);
    if (s->dev) cudaFree(s->dev);
    if (s->mk_phases) cudaFree(s->mk_phases);
    if (s->mk_lite) cudaFree(s->mk_lite);
    delete s;
}

extern "C" int v3g_state_reset(v3g_state *s, void *stream) {
    if (!s) return fail(V3G_E_ARG, "null state");
    CUDA_TRY(launch_state_reset(s->m, s, (cudaStream_t)stream));
    s->pos = 0;
    return V3G_OK;
}

extern "C" uint64_t v3g_state_pos(const v3g_state *s) { return s ? s->pos : 0; }

// device SeqCtl field update for every sequence (rare host knobs)
static int set_seq_field(v3g_state *s, size_t field_off, int32_t value, cudaStream_t st) {
    for (int b = 0; b < s->B; ++b) {
        // value must outlive the async copy: use a blocking copy on the stream
        CUDA_TRY(cudaStreamSynchronize(st));
        CUDA_TRY(cudaMemcpy(reinterpret_cast<uint8_t *>(s->host.seq + b) + field_off, &value, 4, cudaMemcpyHostToDevice));
    }
    return V3G_OK;
}

extern "C" int v3g_set_pinned(v3g_state *s, uint32_t n_pin, void *stream) {
    if (!s) return fail(V3G_E_ARG, "null state");
    const ModelDev &md = s->m->host;
    if (n_pin > (uint32_t)md.sink_cap || n_pin > (uint32_t)md.W) return fail(V3G_E_LIMIT, "n_pin above sink capacity");
    cudaStream_t st = (cudaStream_t)stream;
    int rc;
    if ((rc = set_seq_field(s, offsetof(SeqCtl, n_pin), (int32_t)n_pin, st)) != V3G_OK) return rc;
    if ((rc = set_seq_field(s, offsetof(SeqCtl, pin_locked), 1, st)) != V3G_OK) return rc;
    if ((rc = set_seq_field(s, offsetof(SeqCtl, auto_pin), 0, st)) != V3G_OK) return rc;
    s->auto_pin = 0;
    if (s->pos >= 2ull * md.W) CUDA_TRY(launch_prefix_refresh(s->m, s, st));
    return V3G_OK;
}

extern "C" int v3g_set_seg_budget(v3g_state *s, uint32_t budget, void *stream) {
    if (!s) return fail(V3G_E_ARG, "null state");
    if ((int)budget > s->seg_cap) return fail(V3G_E_LIMIT, "budget above the arena's segment capacity");
    if (s->B > 1 && !s->per_seq_memory && budget > 0)
        return fail(V3G_E_UNSUPPORTED, "segment memory at batch > 1 needs V3G_STATE_PER_SEQ_MEMORY");
    cudaStream_t st = (cudaStream_t)stream;
    if (s->pos > 0 && (int)budget < s->seg_budget)
        return fail(V3G_E_UNSUPPORTED, "shrinking the budget of a running stream is not supported");
    int rc;
    if ((rc = set_seq_field(s, offsetof(SeqCtl, seg_budget), (int32_t)budget, st)) != V3G_OK) return rc;
    const int on = (s->m->host.seg_n_feat > 0 && budget > 0) ? 1 : 0;
    if ((rc = set_seq_field(s, offsetof(SeqCtl, seg_on), on, st)) != V3G_OK) return rc;
    s->seg_budget = (int)budget;
    drop_graphs(s);
    if (s->pos >= 2ull * s->m->host.W) CUDA_TRY(launch_prefix_refresh(s->m, s, st));
    return V3G_OK;
}

// ------------------------------------------------------------------------------------------ stepping
// one step through a cached CUDA graph (or direct launches); variant = boundary * 2 + want_lm
static int run_step(v3g_state *s, bool want_lm, cudaStream_t st) {
    const ModelDev &md = s->m->host;
    const bool boundary = (s->pos % md.W) == 0 && s->pos > 0;
    const int variant = (boundary ? 2 : 0) + (want_lm ? 1 : 0);
    if (!s->use_graphs) {
        CUDA_TRY(launch_step(s->m, s, boundary, want_lm, st));
    } else {
        if (!s->graphs[variant]) {
            cudaGraph_t g;
            CUDA_TRY(cudaStreamBeginCapture(s->cap_stream, cudaStreamCaptureModeThreadLocal));
            cudaError_t e = launch_step(s->m, s, boundary, want_lm, s->cap_stream);
            cudaError_t e2 = cudaStreamEndCapture(s->cap_stream, &g);
            if (e != cudaSuccess) return fail(V3G_E_CUDA, std::string("step capture: ") + cudaGetErrorString(e));
            if (e2 != cudaSuccess) return fail(V3G_E_CUDA, std::string("end capture: ") + cudaGetErrorString(e2));
            cudaError_t e3 = cudaGraphInstantiate(&s->graphs[variant], g, 0);
            cudaGraphDestroy(g);
            if (e3 != cudaSuccess) return fail(V3G_E_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e3));
        }
        CUDA_TRY(cudaGraphLaunch(s->graphs[variant], st));
    }
    s->pos += 1;
    return V3G_OK;
}

static int set_step_io(v3g_state *s, const int32_t *ids, int64_t ld, int32_t *out, int64_t out_ld, cudaStream_t st) {
    // StepCtl: ids, ids_ld, ids_idx, out_tokens, out_ld, out_idx  (pos / status untouched)
    struct { const int32_t *ids; int64_t ids_ld, ids_idx; int32_t *out; int64_t out_ld, out_idx; } io{ids, ld, 0, out, out_ld, 0};
    static_assert(sizeof(io) == offsetof(StepCtl, status) - offsetof(StepCtl, ids), "StepCtl io block layout");
    CUDA_TRY(cudaStreamSynchronize(st));
    CUDA_TRY(cudaMemcpy(reinterpret_cast<uint8_t *>(s->host.step) + offsetof(StepCtl, ids), &io, sizeof(io),
                        cudaMemcpyHostToDevice));
    return V3G_OK;
}

extern "C" int v3g_step(v3g_state *s, const int32_t *dev_tokens, float *dev_logits, int32_t *dev_next, void *stream) {
    if (!s || !dev_tokens) return fail(V3G_E_ARG, "null argument");
    cudaStream_t st = (cudaStream_t)stream;
    CUDA_TRY(cudaMemcpyAsync(s->host.tok_in, dev_tokens, (size_t)s->B * 4, cudaMemcpyDeviceToDevice, st));
    int rc = run_step(s, true, st);
    if (rc != V3G_OK) return rc;
    const ModelDev &md = s->m->host;
    if (dev_logits)
        CUDA_TRY(cudaMemcpyAsync(dev_logits, s->host.logits, (size_t)s->B * md.vocab * 4, cudaMemcpyDeviceToDevice, st));
    if (dev_next) CUDA_TRY(cudaMemcpyAsync(dev_next, s->host.tok_in, (size_t)s->B * 4, cudaMemcpyDeviceToDevice, st));
    return V3G_OK;
}

extern "C" int v3g_step_host(v3g_state *s, const uint32_t *tokens, float *logits, uint32_t *next, void *stream) {
    if (!s || !tokens) return fail(V3G_E_ARG, "null argument");
    cudaStream_t st = (cudaStream_t)stream;
    CUDA_TRY(cudaMemcpyAsync(s->host.tok_in, tokens, (size_t)s->B * 4, cudaMemcpyHostToDevice, st));
    int rc = run_step(s, true, st);
    if (rc != V3G_OK) return rc;
    const ModelDev &md = s->m->host;
    if (logits) CUDA_TRY(cudaMemcpyAsync(logits, s->host.logits, (size_t)s->B * md.vocab * 4, cudaMemcpyDeviceToHost, st));
    if (next) CUDA_TRY(cudaMemcpyAsync(next, s->host.tok_in, (size_t)s->B * 4, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    return V3G_OK;
}

extern "C" int v3g_prefill(v3g_state *s, const int32_t *dev_ids, uint32_t n, uint64_t ld, float *dev_logits,
                           int32_t *dev_next, void *stream) {
    if (!s || !dev_ids || n == 0) return fail(V3G_E_ARG, "invalid prefill arguments");
    cudaStream_t st = (cudaStream_t)stream;
    const ModelDev &md = s->m->host;
    if (s->chunked_prefill && piece_supported(s->m, s)) {
        // window-aligned pieces of at most pf_cap tokens over all sequences
        const int per_piece = std::max(1, s->pf.cap / s->B);
        uint32_t done = 0;
        while (done < n) {
            const uint64_t c = s->pos % md.W;
            const uint32_t take = (uint32_t)std::min<uint64_t>(std::min<uint64_t>(n - done, md.W - c), per_piece);
            CUDA_TRY(launch_piece(s->m, s, dev_ids, (int64_t)ld, done, (int)take, (int64_t)s->pos, done + take == n, st));
            s->pos += take;
            done += take;
        }
        if (dev_logits)
            CUDA_TRY(cudaMemcpyAsync(dev_logits, s->host.logits, (size_t)s->B * md.vocab * 4, cudaMemcpyDeviceToDevice, st));
        if (dev_next) CUDA_TRY(cudaMemcpyAsync(dev_next, s->host.tok_in, (size_t)s->B * 4, cudaMemcpyDeviceToDevice, st));
        return V3G_OK;
    }
    int rc = set_step_io(s, dev_ids, (int64_t)ld, nullptr, 0, st);
    if (rc != V3G_OK) return rc;
    for (uint32_t i = 0; i < n; ++i)
        if ((rc = run_step(s, i + 1 == n, st)) != V3G_OK) break;
    int rc2 = set_step_io(s, nullptr, 0, nullptr, 0, st);
    if (rc != V3G_OK) return rc;
    if (rc2 != V3G_OK) return rc2;
    if (dev_logits)
        CUDA_TRY(cudaMemcpyAsync(dev_logits, s->host.logits, (size_t)s->B * md.vocab * 4, cudaMemcpyDeviceToDevice, st));
    if (dev_next) CUDA_TRY(cudaMemcpyAsync(dev_next, s->host.tok_in, (size_t)s->B * 4, cudaMemcpyDeviceToDevice, st));
    return V3G_OK;
}

extern "C" int v3g_generate(v3g_state *s, const int32_t *dev_first, uint32_t n_steps, int32_t *dev_out, uint64_t ld,
                            void *stream) {
    if (!s || !dev_first || !dev_out) return fail(V3G_E_ARG, "null argument");
    cudaStream_t st = (cudaStream_t)stream;
    CUDA_TRY(cudaMemcpyAsync(s->host.tok_in, dev_first, (size_t)s->B * 4, cudaMemcpyDeviceToDevice, st));
    int rc = set_step_io(s, nullptr, 0, dev_out, (int64_t)ld, st);
    if (rc != V3G_OK) return rc;
    for (uint32_t i = 0; i < n_steps; ++i)
        if ((rc = run_step(s, true, st)) != V3G_OK) break;
    int rc2 = set_step_io(s, nullptr, 0, nullptr, 0, st);
    return rc != V3G_OK ? rc : rc2;
}

extern "C" int v3g_generate_sampled(v3g_state *s, const int32_t *dev_first, uint32_t n_steps, int32_t *dev_out,
                                    uint64_t ld, uint32_t k, float temp, uint64_t *dev_rng, const v3g_gov_rules_t *gov,
                                    v3g_gov_stream_t *dev_gov, void *stream) {
    if (!s || !dev_first || !dev_out || !dev_rng) return fail(V3G_E_ARG, "null argument");
    const bool governed = gov && gov->n_rules > 0;
    if (governed && !dev_gov) return fail(V3G_E_ARG, "v3g_generate_sampled: governor rules without stream states");
    // the loop's guard (runtime/vault3_host.c:588): 16 candidates for greedy or small k, else k up to 64
    const uint32_t guard = (temp <= 0.0f || k < 16u) ? 16u : (k > 64u ? 64u : k);
    if (n_steps > ld && s->B > 1) return fail(V3G_E_ARG, "v3g_generate_sampled: ld below n_steps");
    cudaStream_t st = (cudaStream_t)stream;
    const ModelDev &md = s->m->host;
    CUDA_TRY(cudaMemcpyAsync(s->host.tok_in, dev_first, (size_t)s->B * 4, cudaMemcpyDeviceToDevice, st));
    int rc = set_step_io(s, nullptr, 0, nullptr, 0, st);
    if (rc != V3G_OK) return rc;
    // each step's greedy token in tok_in is replaced by the draw from that step's logits before the next step reads it
    for (uint32_t i = 0; i < n_steps; ++i) {
        if ((rc = run_step(s, true, st)) != V3G_OK) return rc;
        if (governed)
            CUDA_TRY(launch_govern(s->m, *gov, dev_gov, s->host.logits, (uint32_t)s->B, (uint64_t)md.vocab, guard, st));
        CUDA_TRY(launch_sample_topk(s->host.logits, (uint32_t)s->B, (uint32_t)md.vocab, (uint64_t)md.vocab, k, temp,
                                    dev_rng, s->host.tok_in, dev_out + i, (int64_t)ld, st));
        if (governed) CUDA_TRY(launch_gov_commit(s->m, *gov, dev_gov, s->host.tok_in, (uint32_t)s->B, st));
    }
    return V3G_OK;
}

extern "C" int v3g_status(v3g_state *s, uint32_t *bits, int clear, void *stream) {
    if (!s || !bits) return fail(V3G_E_ARG, "null argument");
    CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
    int32_t v = 0;
    CUDA_TRY(cudaMemcpy(&v, reinterpret_cast<uint8_t *>(s->host.step) + offsetof(StepCtl, status), 4, cudaMemcpyDeviceToHost));
    *bits = (uint32_t)v;
    if (clear) {
        int32_t z = 0;
        CUDA_TRY(cudaMemcpy(reinterpret_cast<uint8_t *>(s->host.step) + offsetof(StepCtl, status), &z, 4, cudaMemcpyHostToDevice));
    }
    return V3G_OK;
}

extern "C" int v3g_status_copy(v3g_state *s, uint32_t *dst, void *stream) {
    if (!s || !dst) return fail(V3G_E_ARG, "null argument");
    CUDA_TRY(cudaMemcpyAsync(dst, reinterpret_cast<uint8_t *>(s->host.step) + offsetof(StepCtl, status), 4,
                             cudaMemcpyDefault, (cudaStream_t)stream));
    return V3G_OK;
}

extern "C" int v3g_seq_info(v3g_state *s, uint32_t b, v3g_seq_info_t *info, int64_t *mem_pos, float *mem_score,
                            uint32_t cap, void *stream) {
    if (!s || !info || b >= (uint32_t)s->B) return fail(V3G_E_ARG, "invalid argument");
    CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
    SeqCtl q;
    CUDA_TRY(cudaMemcpy(&q, s->host.seq + b, sizeof(q), cudaMemcpyDeviceToHost));
    info->n_pin = q.n_pin;
    info->pin_locked = q.pin_locked;
    info->mem_cnt = q.mem_cnt;
    info->n_uniq_segs = q.n_uniq_segs;
    info->seg_id_offset = q.seg_id_offset;
    info->ema_ready = q.ema_ready;
    info->seg_budget = q.seg_budget;
    info->pos = s->pos;
    const uint32_t n = std::min<uint32_t>(cap, (uint32_t)q.mem_cnt);
    const size_t base = ((size_t)b * 2 + q.bank_par) * s->host.seg_cap;
    if (mem_pos && n) CUDA_TRY(cudaMemcpy(mem_pos, s->host.mem_pos + base, n * 8, cudaMemcpyDeviceToHost));
    if (mem_score && n) CUDA_TRY(cudaMemcpy(mem_score, s->host.mem_score + base, n * 4, cudaMemcpyDeviceToHost));
    return V3G_OK;
}

// ------------------------------------------------------------------------------------------ kernel-level entry points
static const MatW *find_mat(const v3g_model *m, uint32_t id) {
    for (auto &p : m->tensor_index)
        if (p.first == id) return p.second;
    return nullptr;
}

extern "C" int v3g_decode_pass(v3g_state *s, int want_lm, void *stream) {
    if (!s) return fail(V3G_E_ARG, "null state");
    if (!s->use_mega) return fail(V3G_E_UNSUPPORTED, "the state does not run the persistent decode kernel");
    cudaStream_t st = (cudaStream_t)stream;
    CUDA_TRY(cudaMemsetAsync(s->host.bar, 0, sizeof(unsigned int), st));   // grid-barrier counter, as k_begin does
    CUDA_TRY(launch_mega(s->m, s, want_lm != 0, st));
    return V3G_OK;
}

extern "C" int v3g_attention(v3g_state *s, uint32_t layer, void *stream) {
    if (!s || layer >= (uint32_t)s->m->host.n_layers) return fail(V3G_E_ARG, "null state or layer out of range");
    CUDA_TRY(launch_step_attention(s->m, s, (int)layer, (cudaStream_t)stream));
    return V3G_OK;
}

extern "C" int v3g_dequant(const v3g_model *m, uint32_t tensor_id, float *dev_out, void *stream) {
    if (!m || !dev_out) return fail(V3G_E_ARG, "null argument");
    const MatW *w = find_mat(m, tensor_id);
    if (!w) return fail(V3G_E_MISSING, "no device matrix for this tensor id");
    // gate (kind 10) and up (kind 11) share one interleaved matrix: the output holds [gate; up]
    if (dequant_matrix(*w, m->host.D, dev_out, (cudaStream_t)stream)) return fail(V3G_E_CUDA, "dequant launch failed");
    return V3G_OK;
}

extern "C" int v3g_gemv(const v3g_model *m, uint32_t tensor_id, const float *dev_x, uint32_t batch, float *dev_y,
                        void *stream) {
    if (!m || !dev_x || !dev_y || batch == 0) return fail(V3G_E_ARG, "invalid argument");
    const MatW *w = find_mat(m, tensor_id);
    if (!w) return fail(V3G_E_MISSING, "no device matrix for this tensor id");
    CUDA_TRY(launch_gemv_mapped(m, *w, dev_x, (int)batch, dev_y, (cudaStream_t)stream));
    return V3G_OK;
}

extern "C" const char *v3g_error_string(int code) {
    switch (code) {
        case V3G_OK: return "ok";
        case V3G_E_SIZE: return "size";
        case V3G_E_MAGIC: return "magic/version";
        case V3G_E_CRC: return "crc";
        case V3G_E_BOUNDS: return "bounds";
        case V3G_E_DTYPE: return "dtype";
        case V3G_E_MISSING: return "missing tensor";
        case V3G_E_SHAPE: return "shape";
        case V3G_E_ARENA: return "arena";
        case V3G_E_TOKENIZER: return "tokenizer";
        case V3G_E_LIMIT: return "limit";
        case V3G_E_ALIGN: return "alignment";
        case V3G_E_NAN: return "non-finite value";
        case V3G_E_CUDA: return "cuda";
        case V3G_E_ARG: return "argument";
        case V3G_E_UNSUPPORTED: return "unsupported";
        case V3G_E_DEVICE: return "device status";
        default: return "unknown";
    }
}

extern "C" const char *v3g_last_error(void) { return g_err.c_str(); }

// failure report for entry points defined in other translation units
int v3g_fail(int code, const std::string &msg) { return fail(code, msg); }
