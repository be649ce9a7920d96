"""CPU oracle for the VAULT v3 streaming decode path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline`
leg of `bench.py` may import it.  The engine in `vault_b200/` never calls it and has no CPU fallback.

It restates, in plain numpy fp32, the reference's per-token step of src/vault_v3_model.py (the same math as
runtime/vault3.c `v3_step`), with its own minimal VLT3 parser and block dequantizers so that it shares no code
with the engine it checks.  Parity pinning: tests/golden/ holds logits produced by the reference Python model
itself (tests/golden/gen_golden.py imports the reference), and tests/test_oracle_golden.py checks this oracle
against them.

Coverage (reference file:line):
  dequant Q8_0 / Q4_0 / BF16 / F16 / F32           tools/vlt3.py:114-116,152-157,189-204
  RMSNorm                                          src/vault_v3_model.py:764-774
  RoPE (rotate-half, fp32 angles)                  src/vault_v3_model.py:777-794
  attention over [sink | segment bank | prev | cur]  src/vault_v3_model.py:1072-1139
  SwiGLU MLP                                       src/vault_v3_model.py:1149-1150
  ChatML system-prompt auto-pin state machine      src/vault_v3_model.py:2224-2252
  segment ids from the 3-tier break rule           src/vault_v3_model.py:116-142,2257-2268
  SegmentScorer + APL habituation EMA              src/vault_v3_model.py:870-883,2294-2305
  authority-spoof quarantine                       src/vault_v3_model.py:1795-1817
  chunk boundary: eviction, top-B bank merge,
    k_prev re-basing, prefix re-rotation           src/vault_v3_model.py:918-949,1842-1935
  tied lm head                                     src/vault_v3_model.py:2150-2151
Not restated: the shingle-resonance bias (src/vault_v3_model.py:1249-1793).  It can only fire within 38 tokens
after a non-pinned <|im_end|> while the bank holds more than two segments; `step` raises NotImplementedError
when that condition is met instead of silently diverging.
"""

from __future__ import annotations

import math
import struct
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np

_F32, _F16, _BF16, _Q8, _Q4 = 0, 1, 2, 8, 9
_KINDS = ("ln1", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "ln2", "wg", "wu", "wd")
_NEWLINE_ID = 198            # hard-coded '\n' id of the reference (src/vault_v3_model.py:1968,2239)


# ---------------------------------------------------------------------------------------------- file parsing

def dequant(raw: bytes, dtype: int, n: int) -> np.ndarray:
    """fp32 values of a tensor payload (tools/vlt3.py:114-116, 152-157, 189-204)."""
    if dtype == _F32:
        return np.frombuffer(raw, "<f4", n).astype(np.float32)
    if dtype == _F16:
        return np.frombuffer(raw, "<f2", n).astype(np.float32)
    if dtype == _BF16:
        return (np.frombuffer(raw, "<u2", n).astype(np.uint32) << 16).view(np.float32)
    nb = n // 32
    if dtype == _Q8:
        blk = np.frombuffer(raw, np.uint8, nb * 34).reshape(nb, 34)
        d = blk[:, :2].copy().view("<f2").astype(np.float32)          # (nb, 1)
        q = blk[:, 2:].view(np.int8).astype(np.float32)
        return (q * d).reshape(-1)
    if dtype == _Q4:
        blk = np.frombuffer(raw, np.uint8, nb * 18).reshape(nb, 18)
        d = blk[:, :2].copy().view("<f2").astype(np.float32)
        qb = blk[:, 2:]
        q = np.concatenate([(qb & 15).astype(np.int32) - 8, (qb >> 4).astype(np.int32) - 8], axis=1)
        return (q.astype(np.float32) * d).reshape(-1)
    raise ValueError(f"dtype {dtype}")


def parse_vlt3(buf: bytes) -> Dict:
    """Header fields and tensor directory of a VLT3 buffer (field offsets of tools/vlt3.py:64-75)."""
    u32 = lambda o: struct.unpack_from("<I", buf, o)[0]
    u64 = lambda o: struct.unpack_from("<Q", buf, o)[0]
    f32 = lambda o: struct.unpack_from("<f", buf, o)[0]
    h = dict(vocab=u32(80), d=u32(84), n_layers=u32(88), n_heads=u32(92), n_kv=u32(96), head_dim=u32(100),
             d_ff=u32(104), window=u32(108), rms_eps=f32(152), rope_theta=f32(156), im_start=u32(172),
             im_end=u32(176), pad=u32(180), n_sink=u32(256), seg_budget=u32(260), seg_hidden=u32(264),
             seg_min=u32(268), seg_max=u32(272), seg_n_feat=u32(276),
             seg_layers=[u32(280 + 4 * i) for i in range(4)], tok_off=u64(48), tok_size=u64(56))
    tensors = {}
    n_t, dir_off = u32(28), u64(32)
    for k in range(n_t):
        e = dir_off + 128 * k
        tid, dt, ndim = struct.unpack_from("<III", buf, e)
        dims = struct.unpack_from("<4I", buf, e + 12)[:ndim]
        off, nb = u64(e + 32), u64(e + 40)
        tensors[tid] = (dt, tuple(int(x) for x in dims), off, nb)
    h["tensors"] = tensors
    return h


def token_bytes_from_blob(buf: bytes, tok_off: int, vocab: int) -> List[bytes]:
    """Per-id raw bytes from the VTOK table (n_vocab x (u32 offset, u32 len) + pool; tools/vlt3.py:283-303)."""
    n_vocab = struct.unpack_from("<I", buf, tok_off + 8)[0]
    o_tab, o_pool = struct.unpack_from("<2Q", buf, tok_off + 28)
    out = [b""] * vocab
    for i in range(min(n_vocab, vocab)):
        so, sl = struct.unpack_from("<II", buf, tok_off + o_tab + 8 * i)
        p = tok_off + o_pool + so
        out[i] = bytes(buf[p:p + sl])
    return out


def seg_break_tier(b: bytes) -> int:
    """3-tier segment-break class of a token's bytes (src/vault_v3_model.py:116-142)."""
    if not b:
        return 0
    t2 = t3 = False
    for i, ch in enumerate(b):
        if ch == 0x0A:
            return 1
        if ch in (0x7D, 0x5D, 0x7C, 0x09):
            t2 = True
        elif ch == 0x22 and i + 1 < len(b) and b[i + 1] == 0x2C:
            t2 = True
        elif ch in (0x2C, 0x26):
            t3 = True
    s = b.rstrip(b" \t\r\x0b\x0c")
    if s and s[-1] in (0x2E, 0x21, 0x3F, 0x3B):
        return 1
    return 2 if t2 else (3 if t3 else 0)


# ---------------------------------------------------------------------------------------------- model

class OracleModel:
    """Dequantized fp32 weights + hyper-parameters of one VLT3 file."""

    def __init__(self, buf: bytes, system_tok_id: Optional[int] = None, max_sink: int = 512,
                 auto_pin_system: bool = True):
        h = parse_vlt3(buf)
        self.h = h
        self.V, self.d, self.L = h["vocab"], h["d"], h["n_layers"]
        self.H, self.G, self.D, self.F, self.W = h["n_heads"], h["n_kv"], h["head_dim"], h["d_ff"], h["window"]
        self.eps = np.float32(h["rms_eps"])
        self.theta = np.float32(h["rope_theta"])
        self.n_sink = h["n_sink"]
        self.max_sink = max_sink
        self.auto_pin_system = auto_pin_system
        self.sink_cap = max(1, self.n_sink, max_sink if auto_pin_system else self.n_sink)
        self.im_start, self.im_end = h["im_start"], h["im_end"]
        self.seg_n_feat = h["seg_n_feat"]
        self.seg_layers = list(h["seg_layers"][: self.seg_n_feat])
        self.seg_budget_default = h["seg_budget"] if self.seg_n_feat else 0
        self.seg_hidden, self.seg_min, self.seg_max = h["seg_hidden"], h["seg_min"], h["seg_max"]

        def get(tid: int) -> np.ndarray:
            dt, dims, off, nb = h["tensors"][tid]
            return dequant(bytes(buf[off:off + nb]), dt, int(np.prod(dims))).reshape(dims)

        self.embed = get(1)
        self.norm = get(2)
        self.layers = []
        for li in range(self.L):
            self.layers.append({k: get(((li + 1) << 8) | (j + 1)) for j, k in enumerate(_KINDS)})
        if self.seg_n_feat:
            self.sc_ln_w, self.sc_ln_b, self.sc_w1, self.sc_b1, self.sc_w2, self.sc_b2 = (get(i) for i in range(4, 10))
        self.raw_bytes = token_bytes_from_blob(buf, h["tok_off"], self.V)
        self.tier = np.array([seg_break_tier(b) for b in self.raw_bytes], dtype=np.uint8)
        if system_tok_id is None:
            system_tok_id = next((i for i, b in enumerate(self.raw_bytes) if b == b"system"), 8948)
        self.system_tok = system_tok_id
        # fp32 RoPE inverse frequencies, as torch computes them (src/vault_v3_model.py:779)
        ex = np.arange(0, self.D, 2, dtype=np.float32) / np.float32(self.D)
        self.inv_freq = (np.float32(1.0) / np.power(self.theta, ex, dtype=np.float32)).astype(np.float32)

    @classmethod
    def from_file(cls, path: str, **kw) -> "OracleModel":
        with open(path, "rb") as f:
            return cls(f.read(), **kw)

    # --- basic ops
    def rmsnorm(self, x: np.ndarray, g: np.ndarray) -> np.ndarray:
        return g * (x * (np.float32(1.0) / np.sqrt(np.mean(x * x, dtype=np.float32) + self.eps))).astype(np.float32)

    def cos_sin(self, positions: np.ndarray):
        ang = positions.astype(np.float32)[:, None] * self.inv_freq[None, :]
        emb = np.concatenate([ang, ang], axis=-1)
        return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)

    @staticmethod
    def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
        h = x.shape[-1] // 2
        rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
        return (x * cos + rot * sin).astype(np.float32)

    def scorer(self, f: np.ndarray) -> np.float32:
        """LayerNorm(eps 1e-5) -> fc1 -> exact-erf GELU -> fc2 (src/vault_v3_model.py:879-883)."""
        mu = np.mean(f, dtype=np.float32)
        var = np.mean((f - mu) ** 2, dtype=np.float32)
        h = (f - mu) / np.sqrt(var + np.float32(1e-5)) * self.sc_ln_w + self.sc_ln_b
        z = self.sc_w1 @ h.astype(np.float32) + self.sc_b1
        gelu = np.array([0.5 * v * (1.0 + math.erf(v / math.sqrt(2.0))) for v in z.astype(np.float64)],
                        dtype=np.float32)
        return np.float32((self.sc_w2 @ gelu + self.sc_b2)[0])


# ---------------------------------------------------------------------------------------------- state

@dataclass
class _LayerKV:
    k_prev: np.ndarray
    k_cur: np.ndarray
    v_prev: np.ndarray
    v_cur: np.ndarray
    kraw_prev: np.ndarray
    kraw_cur: np.ndarray
    k_sink_raw: np.ndarray
    k_sink_rot: np.ndarray
    v_sink: np.ndarray
    k_seg_raw: np.ndarray
    k_seg_rot: np.ndarray
    v_seg: np.ndarray


class OracleState:
    """Per-sequence streaming state (src/vault_v3_model.py:956-1024)."""

    def __init__(self, m: OracleModel, seg_budget: Optional[int] = None, auto_pin: bool = True):
        W, G, D = m.W, m.G, m.D
        self.pos = 0
        self.seg_budget = m.seg_budget_default if seg_budget is None else int(seg_budget)
        self.seg_active = m.seg_n_feat > 0 and self.seg_budget > 0
        self.n_pin = min(m.n_sink, W)
        self.pin_locked = not (auto_pin and m.auto_pin_system)
        self.saw_im_start = False
        self.awaiting_sys_nl = False
        self.ema_ready = False
        self.ema = np.zeros(max(1, m.seg_n_feat * m.d), np.float32)
        self.tok_prev = np.zeros(W, np.int64)
        self.tok_cur = np.zeros(W, np.int64)
        self.sc_prev = np.zeros(W, np.float32)
        self.sc_cur = np.zeros(W, np.float32)
        self.seg_prev = np.zeros(W, np.int64)
        self.seg_cur = np.zeros(W, np.int64)
        self.seg_id_offset = 0
        self.cur_seg_id = 0
        self.seg_len = 0
        self.mem_pos = np.zeros(0, np.int64)
        self.mem_score = np.zeros(0, np.float32)
        self.mem_tok = np.zeros(0, np.int64)
        self.mem_seg = np.zeros(0, np.int64)
        self.n_uniq_segs = 0
        S_cap, B_cap = m.sink_cap, max(1, self.seg_budget)
        z = lambda n: np.zeros((G, n, D), np.float32)
        self.layers = [_LayerKV(z(W), z(W), z(W), z(W), z(W), z(W), z(S_cap), z(S_cap), z(S_cap),
                                z(B_cap), z(B_cap), z(B_cap)) for _ in range(m.L)]

    def set_pinned(self, m: OracleModel, n_pin: int) -> None:
        self.n_pin = max(0, min(int(n_pin), m.W, m.sink_cap))
        self.pin_locked = True


# ---------------------------------------------------------------------------------------------- step

def _auto_pin(m: OracleModel, st: OracleState, tid: int) -> None:
    """Online ChatML system-prompt pinning (src/vault_v3_model.py:2224-2252)."""
    pos = st.pos
    limit = min(m.max_sink, m.W, m.sink_cap)
    if pos == 0:
        if tid == m.im_start and limit >= 2:
            st.saw_im_start = True
        else:
            st.pin_locked = True
    elif pos == 1 and st.saw_im_start:
        if tid != m.system_tok:
            st.saw_im_start = False
            st.pin_locked = True
    elif st.saw_im_start and pos < limit:
        if st.awaiting_sys_nl:
            st.n_pin = max(st.n_pin, pos + 1 if tid == _NEWLINE_ID else pos)
            st.pin_locked = True
            st.awaiting_sys_nl = False
        elif tid == m.im_end:
            st.n_pin = max(st.n_pin, pos + 1)
            if pos + 1 < limit:
                st.awaiting_sys_nl = True
            else:
                st.pin_locked = True
    elif pos >= limit:
        if st.saw_im_start and not st.awaiting_sys_nl:
            st.n_pin = max(st.n_pin, limit)
        st.pin_locked = True
        st.awaiting_sys_nl = False


def merge_bank(mem_pos, mem_score, cand_pos, cand_score, budget: int):
    """Top-`budget` by (score desc, pos asc), returned chronologically (src/vault_v3_model.py:918-949)."""
    M = len(mem_pos)
    all_pos = np.concatenate([mem_pos, cand_pos])
    all_sc = np.concatenate([mem_score, cand_score]).astype(np.float32)
    if budget <= 0 or len(all_pos) == 0:
        e = np.zeros(0, np.int64)
        return e, e, e, np.zeros(0, np.float32)
    if len(all_pos) <= budget:
        return np.arange(M), np.arange(len(all_pos) - M), all_pos, all_sc
    order = np.argsort(-all_sc, kind="stable")[:budget]
    win = np.sort(order)
    keep = win[win < M]
    add = win[win >= M] - M
    return keep, add, all_pos[win], all_sc[win]


def _refresh_prefix(m: OracleModel, st: OracleState) -> None:
    """Re-rotate the bank to positions -M..-1 and the sinks to -(M+S)..-(M+1) (src/vault_v3_model.py:1842-1856)."""
    M = len(st.mem_pos) if st.seg_active else 0
    S = st.n_pin
    if M > 0:
        cs, sn = m.cos_sin(np.arange(-M, 0))
        for lk in st.layers:
            lk.k_seg_rot[:, :M] = m.rope(lk.k_seg_raw[:, :M], cs, sn)
    if S > 0:
        cs, sn = m.cos_sin(np.arange(-(M + S), -M))
        for lk in st.layers:
            lk.k_sink_rot[:, :S] = m.rope(lk.k_sink_raw[:, :S], cs, sn)


def _advance_boundary(m: OracleModel, st: OracleState) -> None:
    """Chunk rollover at pos % W == 0 (src/vault_v3_model.py:1858-1935)."""
    W, pos = m.W, st.pos
    if pos >= 2 * W and st.seg_active and st.seg_budget > 0:
        ev = pos // W - 2
        bad = st.sc_prev <= np.float32(-1.0e29)
        if bad.any():
            bad_seg = np.zeros(int(st.seg_prev.max()) + 1, bool)
            bad_seg[st.seg_prev[bad]] = True
            st.sc_prev[bad_seg[st.seg_prev]] = np.float32(-1.0e30)
        n_loc = int(st.seg_prev.max()) + 1
        mx = np.full(n_loc, -np.inf, np.float32)
        np.maximum.at(mx, st.seg_prev, st.sc_prev)
        full_seg = st.seg_prev + st.seg_id_offset
        cand_all = (mx[st.seg_prev] - np.float32(1e-6) * (full_seg % 16384).astype(np.float32)).astype(np.float32)
        st.seg_id_offset += n_loc
        t0 = st.n_pin if ev == 0 else 0
        if t0 < W:
            t = np.arange(t0, W)
            ok = cand_all[t0:] > np.float32(-1.0e29)
            t = t[ok]
            keep, add, st.mem_pos, st.mem_score = merge_bank(st.mem_pos, st.mem_score, ev * W + t,
                                                             cand_all[t], st.seg_budget)
            st.mem_tok = np.concatenate([st.mem_tok[keep], st.tok_prev[t[add]]])
            st.mem_seg = np.concatenate([st.mem_seg[keep], full_seg[t[add]]])
            nk, na = len(keep), len(add)
            for lk in st.layers:
                kr = lk.k_seg_raw[:, keep].copy()
                vv = lk.v_seg[:, keep].copy()
                lk.k_seg_raw[:, :nk] = kr
                lk.v_seg[:, :nk] = vv
                lk.k_seg_raw[:, nk:nk + na] = lk.kraw_prev[:, t[add]]
                lk.v_seg[:, nk:nk + na] = lk.v_prev[:, t[add]]
            ms = st.mem_seg
            st.n_uniq_segs = 0 if len(ms) == 0 else 1 + int(np.count_nonzero(ms[1:] != ms[:-1]))
    if pos >= 2 * W:
        cs, sn = m.cos_sin(np.array([-W]))
    for lk in st.layers:
        lk.k_prev[...] = lk.k_cur
        lk.v_prev[...] = lk.v_cur
        lk.kraw_prev[...] = lk.kraw_cur
        if pos >= 2 * W:
            lk.k_prev[...] = m.rope(lk.k_prev, cs, sn)
    st.tok_prev[...] = st.tok_cur
    st.sc_prev[...] = st.sc_cur
    st.seg_prev[...] = st.seg_cur
    st.cur_seg_id = 0
    st.seg_len = 0
    if pos >= 2 * W:
        _refresh_prefix(m, st)


def _resonance_could_fire(m: OracleModel, st: OracleState, c: int) -> bool:
    """Necessary condition of the shingle-resonance bias (src/vault_v3_model.py:1643-1716): bank with more than two
    segments and a non-pinned <|im_end|> within the last 38 tokens."""
    if len(st.mem_pos) == 0 or st.n_uniq_segs <= 2:
        return False
    hist = np.concatenate([st.tok_prev, st.tok_cur[: c + 1]])
    hi = m.W + c
    for p in range(hi, max(0, hi - 37) - 1, -1):
        if hist[p] == m.im_end:
            return p > 0 and st.pos - (hi - p) >= st.n_pin
    return False


def _spoof_hit(m: OracleModel, st: OracleState, pos: int, c: int) -> bool:
    """Authority-spoof quarantine test over the last <= 24 tokens (src/vault_v3_model.py:1795-1817)."""
    if st.n_pin <= m.n_sink or pos < st.n_pin:
        return False
    W = m.W
    lb = min(24, pos - st.n_pin + 1)
    avail_cur = c + 1
    lb = min(lb, (W + avail_cur) if pos >= W else avail_cur)
    need_prev = lb - avail_cur if avail_cur < lb else 0
    cur_start = avail_cur - lb if avail_cur > lb else 0
    toks = (list(st.tok_prev[W - need_prev:W]) if need_prev > 0 else []) + list(st.tok_cur[cur_start:c + 1])
    buf = bytearray()
    for tid in toks:
        for ch in (m.raw_bytes[tid] if 0 <= tid < m.V else b""):
            if len(buf) >= 4096:
                break
            buf.append(ch + 32 if 0x41 <= ch <= 0x5A else ch)
    return (b"opi_signed_directive" in buf) or (b"urgent opi delegation" in buf)


def step(m: OracleModel, st: OracleState, token: int) -> np.ndarray:
    """Feed one token, return fp32 logits [V] (src/vault_v3_model.py:2214-2311 for batch 1)."""
    W, D, H, G = m.W, m.D, m.H, m.G
    grp = H // G
    pos = st.pos
    c = pos % W
    tid = int(token)
    if not st.pin_locked:
        _auto_pin(m, st, tid)
    if c == 0 and pos > 0:
        _advance_boundary(m, st)
    st.tok_cur[c] = tid
    if st.seg_active:
        tr = int(m.tier[tid]) if 0 <= tid < m.V else 0
        t2 = max(m.seg_min, (m.seg_max * 2) // 3)
        t3 = max(m.seg_min, m.seg_max - 8 if m.seg_max > 8 else m.seg_min)
        st.seg_cur[c] = st.cur_seg_id
        st.seg_len += 1
        brk = (tr == 1 and st.seg_len >= m.seg_min) or (tr == 2 and st.seg_len >= t2) or \
              (tr == 3 and st.seg_len >= t3)
        if c == W - 1 or brk or st.seg_len >= m.seg_max:
            st.cur_seg_id += 1
            st.seg_len = 0
        if pos >= 2 * W and _resonance_could_fire(m, st, c):
            raise NotImplementedError("shingle-resonance bias would be active (not restated by the oracle)")
    eff = (W + c) if pos >= W else c
    cq, sq = m.cos_sin(np.array([eff]))
    x = m.embed[tid].astype(np.float32).copy()
    feats = []
    S = st.n_pin if pos >= 2 * W else 0
    M = len(st.mem_pos) if (pos >= 2 * W and st.seg_active) else 0
    scale = np.float32(1.0 / math.sqrt(D))
    for li, (Lw, lk) in enumerate(zip(m.layers, st.layers)):
        if st.seg_active and li in m.seg_layers:
            feats.append((li, x.copy()))
        u = m.rmsnorm(x, Lw["ln1"])
        q = (Lw["wq"] @ u + Lw["bq"]).reshape(H, D)
        k = (Lw["wk"] @ u + Lw["bk"]).reshape(G, D)
        v = (Lw["wv"] @ u + Lw["bv"]).reshape(G, D)
        qr = m.rope(q, cq, sq)
        kr = m.rope(k, cq, sq)
        lk.k_cur[:, c] = kr
        lk.v_cur[:, c] = v
        lk.kraw_cur[:, c] = k
        if pos < lk.k_sink_raw.shape[1]:
            lk.k_sink_raw[:, pos] = k
            lk.v_sink[:, pos] = v
        if pos >= W:
            keys = np.concatenate([lk.k_sink_rot[:, :S], lk.k_seg_rot[:, :M], lk.k_prev, lk.k_cur[:, :c + 1]], 1)
            vals = np.concatenate([lk.v_sink[:, :S], lk.v_seg[:, :M], lk.v_prev, lk.v_cur[:, :c + 1]], 1)
        else:
            keys, vals = lk.k_cur[:, :c + 1], lk.v_cur[:, :c + 1]
        out = np.empty((H, D), np.float32)
        for h in range(H):
            g = h // grp
            s = (keys[g] @ qr[h]) * scale
            p = np.exp(s - s.max())
            out[h] = (p / p.sum()) @ vals[g]
        x = x + Lw["wo"] @ out.reshape(-1)
        u2 = m.rmsnorm(x, Lw["ln2"])
        gt = Lw["wg"] @ u2
        x = x + Lw["wd"] @ ((gt / (np.float32(1.0) + np.exp(-gt))) * (Lw["wu"] @ u2))
    if st.seg_active:
        order = {li: i for i, li in enumerate(m.seg_layers)}
        f = np.concatenate([v for _, v in sorted(feats, key=lambda t: order[t[0]])]).astype(np.float32)
        raw = m.scorer(f)
        sc = raw
        if not st.ema_ready:
            st.ema[...] = f
            st.ema_ready = True
        else:
            hab = m.scorer((f - np.float32(0.65) * st.ema).astype(np.float32))
            st.ema[...] = st.ema * np.float32(0.985) + np.float32(0.015) * f
            sc = np.float32(raw + np.float32(0.35) * max(np.float32(0.0), np.float32(hab - raw)))
        st.sc_cur[c] = sc
        if _spoof_hit(m, st, pos, c):
            st.sc_cur[c] = np.float32(-1.0e30)
    st.pos = pos + 1
    return (m.embed @ m.rmsnorm(x, m.norm)).astype(np.float32)


def run(m: OracleModel, ids: Sequence[int], seg_budget: Optional[int] = None, auto_pin: bool = True,
        n_pin: Optional[int] = None, positions: Optional[Sequence[int]] = None):
    """Stream `ids` through a fresh state; return (logits at `positions` (default all) [n, V], state)."""
    st = OracleState(m, seg_budget=seg_budget, auto_pin=auto_pin)
    if n_pin is not None:
        st.set_pinned(m, n_pin)
    want = set(range(len(ids))) if positions is None else set(positions)
    out = []
    for i, t in enumerate(ids):
        lg = step(m, st, int(t))
        if i in want:
            out.append(lg)
    return np.stack(out) if out else np.zeros((0, m.V), np.float32), st
