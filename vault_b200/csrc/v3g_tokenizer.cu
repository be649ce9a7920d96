// Host tokenizer of a VLT3 file's VTOK blob: byte-level BPE behind the Qwen2 pre-tokenizer, with UAX #15 NFC
// applied to spans that can change under it, and ChatML special tokens matched as whole strings.  It produces the
// reference's ids for the same text: v3_encode / v3_encode_ex (runtime/vault3.c:2708-2809), with
//   pretok_match        runtime/vault3.c:2503-2560  (the pre-tokenizer's piece rules)
//   bpe_piece           runtime/vault3.c:2591-2648  (lowest merge rank first, leftmost first among equal ranks)
//   bpe_piece_long      runtime/vault3.c:2650-2686  (pieces above 32 KB in token-aligned windows, 4 KB carried)
//   nfc_normalize_span  runtime/vault3.c:2408-2478  (decompose, canonical order, compose; at most 2048 code points)
// Host code only: the token loop on the device never calls it.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <functional>
#include <unordered_map>
#include <vector>

#include "../../include/vault_b200.h"
#include "v3g_internal.h"
#include "v3g_nfc_tables.h"

namespace {

constexpr size_t MAX_PIECE = 32768;     // bytes of one BPE pass
constexpr size_t NFC_SPAN = 1024;       // bytes of one NFC span
constexpr size_t NFC_MAX_CPS = 2048;    // code points of one NFC span
constexpr uint32_t DEAD = 0xFFFFFFFFu;

inline uint32_t rd32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return v; }
inline uint64_t rd64(const uint8_t *p) { uint64_t v; memcpy(&v, p, 8); return v; }

// one code point; malformed input gives 0x110000 with length 1 (no overlong / surrogate check)
uint32_t cp_at(const uint8_t *s, size_t n, size_t i, size_t &len) {
    const uint8_t c = s[i];
    len = 1;
    if (c < 0x80) return c;
    int extra;
    uint32_t cp;
    if ((c & 0xE0) == 0xC0) { extra = 1; cp = c & 0x1F; }
    else if ((c & 0xF0) == 0xE0) { extra = 2; cp = c & 0x0F; }
    else if ((c & 0xF8) == 0xF0) { extra = 3; cp = c & 0x07; }
    else return 0x110000u;
    if ((size_t)extra > n - 1 - i) return 0x110000u;
    for (int k = 1; k <= extra; ++k) {
        if ((s[i + k] & 0xC0) != 0x80) return 0x110000u;
        cp = (cp << 6) | (s[i + k] & 0x3F);
    }
    len = (size_t)extra + 1;
    return cp;
}

// strict form for NFC: overlong forms, surrogates and values above U+10FFFF are invalid too, and an invalid byte b
// reads as 0x110000 | b so that it survives normalization unchanged
uint32_t cp_at_strict(const uint8_t *s, size_t n, size_t i, size_t &len) {
    const uint8_t c = s[i];
    len = 1;
    if (c < 0x80) return c;
    int extra;
    uint32_t cp, least;
    if ((c & 0xE0) == 0xC0) { extra = 1; cp = c & 0x1F; least = 0x80; }
    else if ((c & 0xF0) == 0xE0) { extra = 2; cp = c & 0x0F; least = 0x800; }
    else if ((c & 0xF8) == 0xF0) { extra = 3; cp = c & 0x07; least = 0x10000; }
    else return 0x110000u | c;
    if ((size_t)extra > n - 1 - i) return 0x110000u | c;
    for (int k = 1; k <= extra; ++k) {
        if ((s[i + k] & 0xC0) != 0x80) return 0x110000u | c;
        cp = (cp << 6) | (s[i + k] & 0x3F);
    }
    if (cp < least || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return 0x110000u | c;
    len = (size_t)extra + 1;
    return cp;
}

bool is_ws(uint32_t cp) {
    return cp == ' ' || (cp >= 0x09 && cp <= 0x0D) || cp == 0x85 || cp == 0xA0 || cp == 0x1680 ||
           (cp >= 0x2000 && cp <= 0x200A) || cp == 0x2028 || cp == 0x2029 || cp == 0x202F || cp == 0x205F ||
           cp == 0x3000;
}
bool is_crlf(uint32_t cp) { return cp == '\r' || cp == '\n'; }
bool has_nfc_byte(const uint8_t *s, size_t n) {   // bytes below 0xCC only start text that NFC leaves alone
    for (size_t i = 0; i < n; ++i)
        if (s[i] >= 0xCC) return true;
    return false;
}

uint32_t ccc_of(uint32_t cp) {
    if (cp < 0x300 || cp >= 0x110000u) return 0;
    const v3g::NfcCcc *end = v3g::NFC_CCC + sizeof(v3g::NFC_CCC) / sizeof(v3g::NFC_CCC[0]);
    const v3g::NfcCcc *it = std::lower_bound(v3g::NFC_CCC, end, cp, [](const v3g::NfcCcc &e, uint32_t c) { return e.cp < c; });
    return (it != end && it->cp == cp) ? it->ccc : 0;
}

void decompose(uint32_t cp, std::vector<uint32_t> &out) {
    auto put = [&](uint32_t c) { if (out.size() < NFC_MAX_CPS) out.push_back(c); };
    if (cp >= 0xAC00 && cp <= 0xD7A3) {   // Hangul syllable: L V (T)
        const uint32_t s = cp - 0xAC00;
        put(0x1100 + s / 588);
        put(0x1161 + (s % 588) / 28);
        if (s % 28) put(0x11A7 + s % 28);
        return;
    }
    if (cp >= 0xC0 && cp < 0x110000u) {
        const v3g::NfcDecomp *end = v3g::NFC_DECOMP + sizeof(v3g::NFC_DECOMP) / sizeof(v3g::NFC_DECOMP[0]);
        const v3g::NfcDecomp *it =
            std::lower_bound(v3g::NFC_DECOMP, end, cp, [](const v3g::NfcDecomp &e, uint32_t c) { return e.cp < c; });
        if (it != end && it->cp == cp) {
            decompose(it->first, out);
            if (it->second) decompose(it->second, out);
            return;
        }
    }
    put(cp);
}

uint32_t compose(uint32_t a, uint32_t b) {
    if (a >= 0x1100 && a <= 0x1112 && b >= 0x1161 && b <= 0x1175) return 0xAC00 + ((a - 0x1100) * 21 + (b - 0x1161)) * 28;
    if (a >= 0xAC00 && a <= 0xD7A3 && (a - 0xAC00) % 28 == 0 && b >= 0x11A8 && b <= 0x11C2) return a + (b - 0x11A7);
    const v3g::NfcCompose *end = v3g::NFC_COMPOSE + sizeof(v3g::NFC_COMPOSE) / sizeof(v3g::NFC_COMPOSE[0]);
    const v3g::NfcCompose *it = std::lower_bound(v3g::NFC_COMPOSE, end, std::make_pair(a, b),
                                                 [](const v3g::NfcCompose &e, const std::pair<uint32_t, uint32_t> &k) {
                                                     return e.first < k.first || (e.first == k.first && e.second < k.second);
                                                 });
    return (it != end && it->first == a && it->second == b) ? it->composite : 0;
}

void put_utf8(std::vector<uint8_t> &o, uint32_t cp) {
    if (cp >= 0x110000u) o.push_back((uint8_t)(cp & 0xFF));   // an invalid input byte, restored
    else if (cp < 0x80) o.push_back((uint8_t)cp);
    else if (cp < 0x800) { o.push_back((uint8_t)(0xC0 | (cp >> 6))); o.push_back((uint8_t)(0x80 | (cp & 0x3F))); }
    else if (cp < 0x10000) {
        o.push_back((uint8_t)(0xE0 | (cp >> 12)));
        o.push_back((uint8_t)(0x80 | ((cp >> 6) & 0x3F)));
        o.push_back((uint8_t)(0x80 | (cp & 0x3F)));
    } else {
        o.push_back((uint8_t)(0xF0 | (cp >> 18)));
        o.push_back((uint8_t)(0x80 | ((cp >> 12) & 0x3F)));
        o.push_back((uint8_t)(0x80 | ((cp >> 6) & 0x3F)));
        o.push_back((uint8_t)(0x80 | (cp & 0x3F)));
    }
}

}  // namespace

struct v3g_tokenizer {
    std::vector<uint8_t> blob;   // copy of the VTOK blob
    uint32_t n_vocab = 0, n_merges = 0, n_special = 0, n_ranges = 0;
    const uint8_t *table = nullptr, *pool = nullptr, *special = nullptr, *ranges = nullptr, *bytemap = nullptr;
    std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>> merges;   // (left << 32 | right) -> (rank, result)
    std::vector<uint32_t> sym, win;
    std::vector<uint64_t> heap;   // merge candidates, a min-heap kept across pieces
    std::vector<int32_t> prv, nxt;
    std::vector<uint32_t> cps;
    std::vector<uint8_t> nfc;

    bool token(uint32_t id, const uint8_t *&b, uint32_t &n) const {
        if (id >= n_vocab) { b = nullptr; n = 0; return false; }
        b = pool + rd32(table + 8ull * id);
        n = rd32(table + 8ull * id + 4);
        return true;
    }

    // 1 letter, 2 digit, 0 other: ASCII directly, the rest from the blob's sorted (lo, hi, class) ranges
    int cls(uint32_t cp) const {
        if (cp < 128) return ((cp | 0x20) >= 'a' && (cp | 0x20) <= 'z') ? 1 : (cp >= '0' && cp <= '9') ? 2 : 0;
        uint32_t lo = 0, hi = n_ranges;
        while (lo < hi) {
            const uint32_t mid = (lo + hi) / 2;
            const uint8_t *r = ranges + 12ull * mid;
            if (cp < rd32(r)) hi = mid;
            else if (cp > rd32(r + 4)) lo = mid + 1;
            else return (int)rd32(r + 8);
        }
        return 0;
    }

    // length of the pre-tokenizer piece starting at i (the Qwen2 pattern's alternatives in order)
    size_t piece_len(const uint8_t *s, size_t n, size_t i) const {
        size_t l0, l;
        const uint32_t c0 = cp_at(s, n, i, l0);
        if (c0 == '\'' && i + 1 < n) {   // contractions 's 't 'm 'd 're 've 'll, any case
            const uint8_t a = s[i + 1] | 0x20, b = i + 2 < n ? (s[i + 2] | 0x20) : 0;
            if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
            if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
        }
        auto letters_from = [&](size_t j) {
            while (j < n && cls(cp_at(s, n, j, l)) == 1) j += l;
            return j;
        };
        const int k0 = cls(c0);
        // an optional non-letter, non-digit, non-newline prefix, then letters
        const size_t j = (k0 != 1 && k0 != 2 && !is_crlf(c0)) ? i + l0 : i;
        if (j < n && cls(cp_at(s, n, j, l)) == 1) return letters_from(j) - i;
        if (k0 == 1) return letters_from(i) - i;
        if (k0 == 2) return l0;   // one digit
        {   // an optional space, then punctuation-like characters, then trailing newlines
            const size_t b = c0 == ' ' ? i + 1 : i;
            size_t e = b;
            while (e < n) {
                const uint32_t cp = cp_at(s, n, e, l);
                if (is_ws(cp) || cls(cp) != 0) break;
                e += l;
            }
            if (e > b) {
                while (e < n && (s[e] == '\r' || s[e] == '\n')) ++e;
                return e - i;
            }
        }
        if (is_ws(c0)) {   // whitespace: through the last newline, or all but the final character before text
            size_t e = i, nl_end = 0;
            while (e < n) {
                const uint32_t cp = cp_at(s, n, e, l);
                if (!is_ws(cp)) break;
                e += l;
                if (is_crlf(cp)) nl_end = e;
            }
            if (nl_end) return nl_end - i;
            if (e >= n) return e - i;
            size_t p = e - 1;
            while (p > i && (s[p] & 0xC0) == 0x80) --p;
            return p > i ? p - i : e - i;
        }
        return l0;
    }

    bool merge_of(uint32_t a, uint32_t b, uint32_t &rank, uint32_t &res) const {
        auto it = merges.find(((uint64_t)a << 32) | b);
        if (it == merges.end()) return false;
        rank = it->second.first;
        res = it->second.second;
        return true;
    }

    // BPE of one piece (<= MAX_PIECE bytes used); appends at most cap ids to out, sets truncated when more remain
    size_t bpe(const uint8_t *p, size_t len, uint32_t *out, size_t cap, bool &truncated) {
        const size_t n = std::min(len, MAX_PIECE);
        if (n == 0) return 0;
        for (size_t i = 0; i < n; ++i) {
            sym[i] = rd32(bytemap + 4u * p[i]);
            prv[i] = (int32_t)i - 1;
            nxt[i] = (int32_t)i + 1;
        }
        nxt[n - 1] = -1;
        // candidates keyed (rank << 32 | left position): the smallest key merges first
        const std::greater<uint64_t> later;
        auto push = [&](uint64_t key) {
            heap.push_back(key);
            std::push_heap(heap.begin(), heap.end(), later);
        };
        heap.clear();
        uint32_t r, res;
        for (size_t i = 0; i + 1 < n; ++i)
            if (merge_of(sym[i], sym[i + 1], r, res)) push(((uint64_t)r << 32) | (uint32_t)i);
        while (!heap.empty()) {
            std::pop_heap(heap.begin(), heap.end(), later);
            const uint64_t top = heap.back();
            heap.pop_back();
            const int32_t i = (int32_t)(uint32_t)top;
            if (sym[i] == DEAD) continue;
            const int32_t j = nxt[i];
            if (j < 0 || sym[j] == DEAD) continue;
            if (!merge_of(sym[i], sym[j], r, res) || r != (uint32_t)(top >> 32)) continue;   // stale entry
            sym[i] = res;
            sym[j] = DEAD;
            const int32_t after = nxt[j];
            nxt[i] = after;
            if (after >= 0) prv[after] = i;
            if (prv[i] >= 0 && merge_of(sym[prv[i]], sym[i], r, res)) push(((uint64_t)r << 32) | (uint32_t)prv[i]);
            if (after >= 0 && merge_of(sym[i], sym[after], r, res)) push(((uint64_t)r << 32) | (uint32_t)i);
        }
        size_t k = 0;
        for (int32_t c = 0; c >= 0; c = nxt[c]) {
            if (k == cap) { truncated = true; break; }
            out[k++] = sym[c];
        }
        return k;
    }

    // a piece of any length: above MAX_PIECE bytes, BPE a MAX_PIECE window, keep its tokens except a tail of about
    // 4 KB, advance by the kept bytes' window share, repeat
    int bpe_any(const uint8_t *src, size_t len, uint32_t *out, size_t max_out, size_t &k) {
        size_t pos = 0;
        while (pos < len) {
            const size_t left = len - pos;
            bool trunc = false;
            if (left <= MAX_PIECE) {
                k += bpe(src + pos, left, out + k, max_out - k, trunc);
                return trunc ? V3G_E_SIZE : V3G_OK;
            }
            const size_t got = bpe(src + pos, MAX_PIECE, win.data(), MAX_PIECE, trunc);
            if (got == 0) break;
            size_t keep = got, tail = 0;
            while (keep > 1 && tail < 4096) {
                const uint8_t *tb;
                uint32_t tl;
                token(win[keep - 1], tb, tl);
                tail += tl;
                --keep;
            }
            size_t advance = MAX_PIECE - tail;
            if (advance == 0) advance = MAX_PIECE;
            if (keep > max_out - k) {
                std::copy(win.begin(), win.begin() + (max_out - k), out + k);
                k = max_out;
                return V3G_E_SIZE;
            }
            std::copy(win.begin(), win.begin() + keep, out + k);
            k += keep;
            pos += advance;
        }
        return V3G_OK;
    }

    // NFC of src[0, len) into nfc (decomposition stops once fewer than 4 code-point slots remain)
    size_t normalize(const uint8_t *src, size_t len) {
        cps.clear();
        size_t i = 0, l;
        while (i < len && cps.size() + 4 <= NFC_MAX_CPS) {
            decompose(cp_at_strict(src, len, i, l), cps);
            i += l;
        }
        for (size_t k = 1; k < cps.size(); ++k) {   // canonical order: stable insertion by class within a run
            const uint32_t c = ccc_of(cps[k]);
            if (c == 0) continue;
            const uint32_t v = cps[k];
            size_t j = k;
            for (; j > 0 && ccc_of(cps[j - 1]) > c; --j) cps[j] = cps[j - 1];
            cps[j] = v;
        }
        int64_t starter = -1;
        uint32_t last = 0;
        for (size_t k = 0; k < cps.size(); ++k) {   // canonical composition
            const uint32_t c = ccc_of(cps[k]);
            if (starter >= 0 && (last == 0 || last < c)) {
                const uint32_t comp = compose(cps[starter], cps[k]);
                if (comp) {
                    cps[starter] = comp;
                    cps[k] = DEAD;
                    continue;
                }
            }
            if (c == 0) {
                starter = (int64_t)k;
                last = 0;
            } else {
                last = c;
            }
        }
        nfc.clear();
        for (uint32_t cp : cps)
            if (cp != DEAD) put_utf8(nfc, cp);
        return nfc.size();
    }

    bool special_at(const uint8_t *s, size_t n, size_t i, uint32_t &id, size_t &len) const {
        if (s[i] != '<') return false;
        for (uint32_t k = 0; k < n_special; ++k) {   // the first listed special token that matches
            const uint32_t tid = rd32(special + 4ull * k);
            const uint8_t *b;
            uint32_t bl;
            token(tid, b, bl);
            if (bl == 0 || bl > n - i || memcmp(s + i, b, bl) != 0) continue;
            id = tid;
            len = bl;
            return true;
        }
        return false;
    }

    // the end of the NFC span that starts at i (end - i > NFC_SPAN): a clean pre-tokenizer boundary within the
    // first NFC_SPAN bytes, else the last starter before the limit
    size_t span_end(const uint8_t *t, size_t i, size_t end) const {
        size_t lim = i + NFC_SPAN;
        for (size_t p = i + 1; p <= lim; ++p) {
            if ((t[p] & 0xC0) == 0x80) continue;
            if (has_nfc_byte(t + p, std::min<size_t>(end - p, 4))) continue;
            if (t[p - 1] == '\n' && t[p] != '\r' && t[p] != '\n') return p;
            if (t[p - 1] >= 0x80 && t[p] < 0x80 && t[p] != '\'' && cls(t[p]) == 0) return p;
        }
        while (lim > i + 1 && (t[lim] & 0xC0) == 0x80) --lim;
        while (lim > i + 1) {
            size_t l;
            if (ccc_of(cp_at_strict(t, end, lim, l)) == 0) break;
            --lim;
            while (lim > i + 1 && (t[lim] & 0xC0) == 0x80) --lim;
        }
        return lim;
    }

    int encode(const uint8_t *text, size_t len, uint32_t *out, size_t max_out, size_t *n_out, bool specials) {
        size_t i = 0, k = 0;
        auto done = [&](int rc) { *n_out = k; return rc; };
        while (i < len) {
            uint32_t sid;
            size_t sl;
            if (specials && special_at(text, len, i, sid, sl)) {
                if (k >= max_out) return done(V3G_E_SIZE);
                out[k++] = sid;
                i += sl;
                continue;
            }
            size_t end = len;
            if (specials)
                for (end = i; end < len && !(text[end] == '<' && special_at(text, len, end, sid, sl));) ++end;
            while (i < end) {
                if (!has_nfc_byte(text + i, end - i)) {   // nothing NFC could change: pieces straight to BPE
                    while (i < end) {
                        const size_t ml = piece_len(text, end, i);
                        const int rc = bpe_any(text + i, ml, out, max_out, k);
                        if (rc != V3G_OK) return done(rc);
                        i += ml;
                    }
                    break;
                }
                const size_t ml0 = piece_len(text, end, i);
                if (!has_nfc_byte(text + i, i + ml0 + 4 < end ? ml0 + 4 : end - i)) {   // this piece is clean
                    const int rc = bpe_any(text + i, ml0, out, max_out, k);
                    if (rc != V3G_OK) return done(rc);
                    i += ml0;
                    continue;
                }
                size_t sub = end - i <= NFC_SPAN ? end : span_end(text, i, end);
                if (end - i <= NFC_SPAN) {   // split off an ASCII tail that follows non-ASCII text
                    for (size_t p = i + 1; p < sub; ++p) {
                        if (text[p - 1] >= 0x80 && text[p] < 0x80 && text[p] != '\'' && cls(text[p]) == 0 &&
                            !has_nfc_byte(text + p, sub - p)) {
                            sub = p;
                            break;
                        }
                    }
                }
                const size_t nl = normalize(text + i, sub - i);
                for (size_t ni = 0; ni < nl;) {
                    const size_t ml = piece_len(nfc.data(), nl, ni);
                    const int rc = bpe_any(nfc.data() + ni, ml, out, max_out, k);
                    if (rc != V3G_OK) return done(rc);
                    ni += ml;
                }
                i = sub;
            }
        }
        return done(V3G_OK);
    }
};

extern "C" int v3g_tokenizer_create(v3g_tokenizer **out, const uint8_t *buf, uint64_t size) {
    if (!out) return v3g_fail(V3G_E_ARG, "v3g_tokenizer_create: null output");
    *out = nullptr;
    const uint8_t *tb;
    uint64_t tn;
    int rc = vlt3_token_blob(buf, size, &tb, &tn);
    if (rc != V3G_OK) return rc;
    if (!tb || tn < 128) return v3g_fail(V3G_E_TOKENIZER, "no VTOK tokenizer in the file");
    auto *t = new v3g_tokenizer();
    t->blob.assign(tb, tb + tn);
    const uint8_t *b = t->blob.data();
    t->n_vocab = rd32(b + 8);
    t->n_merges = rd32(b + 12);
    t->n_special = rd32(b + 16);
    t->n_ranges = rd32(b + 20);
    t->table = b + rd64(b + 28);
    t->pool = b + rd64(b + 36);
    const uint8_t *mer = b + rd64(b + 44);
    t->special = b + rd64(b + 52);
    t->ranges = b + rd64(b + 60);
    t->bytemap = b + rd64(b + 68);
    t->merges.reserve(t->n_merges * 2 + 16);
    for (uint32_t r = 0; r < t->n_merges; ++r) {   // a repeated pair keeps its first (lowest) rank
        const uint8_t *e = mer + 12ull * r;
        t->merges.emplace(((uint64_t)rd32(e) << 32) | rd32(e + 4), std::make_pair(r, rd32(e + 8)));
    }
    t->sym.resize(MAX_PIECE);
    t->win.resize(MAX_PIECE);
    t->prv.resize(MAX_PIECE);
    t->nxt.resize(MAX_PIECE);
    t->heap.reserve(3 * MAX_PIECE);
    t->cps.reserve(NFC_MAX_CPS);
    t->nfc.reserve(4 * NFC_MAX_CPS);
    *out = t;
    return V3G_OK;
}

extern "C" void v3g_tokenizer_free(v3g_tokenizer *t) { delete t; }

extern "C" int v3g_encode_ex(v3g_tokenizer *t, const uint8_t *text, size_t len, uint32_t *out, size_t max_out,
                             size_t *n_out, int allow_special) {
    if (!t || !n_out) return V3G_E_SIZE;
    *n_out = 0;
    if (len == 0) return V3G_OK;
    if (!text || (max_out > 0 && !out)) return V3G_E_SIZE;
    return t->encode(text, len, out, max_out, n_out, allow_special != 0);
}

extern "C" int v3g_encode(v3g_tokenizer *t, const uint8_t *text, size_t len, uint32_t *out, size_t max_out,
                          size_t *n_out) {
    return v3g_encode_ex(t, text, len, out, max_out, n_out, 1);
}

extern "C" int v3g_token_bytes(const v3g_tokenizer *t, uint32_t id, const uint8_t **bytes, uint32_t *len) {
    const uint8_t *b = nullptr;
    uint32_t n = 0;
    const bool ok = t && t->token(id, b, n);
    if (bytes) *bytes = b;
    if (len) *len = n;
    return ok ? V3G_OK : V3G_E_TOKENIZER;
}
