"""VLT3 checkpoint container: reader, validator, writer and Q8_0/Q4_0 block codecs.

Host-side mirror of the reference's `tools/vlt3.py` (the VLT3 format is an on-disk contract, so the byte layout,
field order, tensor ids, block layouts and validation rules are the same; the code is this project's own).

Layout of a .vlt3 file (all little-endian):
    [ header: 4096 B, fixed fields, CRC32 of the first 4092 B in the last 4 B ]   tools/vlt3.py:64-74
    [ tensor directory: n_tensors x 128 B entries ]                              tools/vlt3.py:75
    [ VTOK tokenizer blob ]                                                      tools/vlt3.py:246-305
    [ tensor payloads, each 64 B aligned ]                                       tools/vlt3.py:355-369

Block codecs (GGML-compatible):
    Q8_0: fp16 scale d + 32 x int8,  value = q * d                          (34 B / 32 weights)  tools/vlt3.py:102-116
    Q4_0: fp16 scale d + 16 B nibbles, byte j holds element j (low nibble)
          and element j+16 (high nibble), value = (n - 8) * d               (18 B / 32 weights)  tools/vlt3.py:119-157
"""

from __future__ import annotations

import json
import os
import struct
import unicodedata
import zlib
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

MAGIC = b"VLT3"
VERSION = 1
HEADER_SIZE = 4096
ENTRY_SIZE = 128
ALIGN = 64
ENDIAN_TAG = 0x01020304
QK = 32

F32, F16, BF16, Q8_0, Q4_0 = 0, 1, 2, 8, 9
DTYPE_NAMES = {F32: "F32", F16: "F16", BF16: "BF16", Q8_0: "Q8_0", Q4_0: "Q4_0"}
FORMAT_CODES = {"f32": F32, "bf16": BF16, "q8_0": Q8_0, "q4_0": Q4_0}

# Global tensor ids (tools/vlt3.py:34-46); per-layer ids are ((layer + 1) << 8) | kind (tools/vlt3.py:48-57,80-91).
GLOBAL_TENSORS = {
    1: "embed_tokens.weight",
    2: "norm.weight",
    4: "seg_scorer.ln.weight",
    5: "seg_scorer.ln.bias",
    6: "seg_scorer.fc1.weight",
    7: "seg_scorer.fc1.bias",
    8: "seg_scorer.fc2.weight",
    9: "seg_scorer.fc2.bias",
}
_GLOBAL_BY_NAME = {v: k for k, v in GLOBAL_TENSORS.items()}
LAYER_KINDS = (
    "input_layernorm.weight",
    "self_attn.q_proj.weight", "self_attn.q_proj.bias",
    "self_attn.k_proj.weight", "self_attn.k_proj.bias",
    "self_attn.v_proj.weight", "self_attn.v_proj.bias",
    "self_attn.o_proj.weight",
    "post_attention_layernorm.weight",
    "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight",
)
_KIND_BY_NAME = {n: i + 1 for i, n in enumerate(LAYER_KINDS)}
MATMUL_KINDS = frozenset(k for k in LAYER_KINDS if k.endswith("_proj.weight"))
SCORER_IDS = (4, 5, 6, 7, 8, 9)

# Header fields in file order with their struct codes (tools/vlt3.py:64-74).  Offsets are part of the format.
_HEADER_FIELDS: Tuple[Tuple[str, str], ...] = (
    ("magic", "4s"), ("version", "I"), ("header_size", "I"), ("endian_tag", "I"),
    ("file_size", "Q"), ("alignment", "I"), ("n_tensors", "I"),
    ("tensor_dir_offset", "Q"), ("tensor_dir_size", "Q"), ("tokenizer_offset", "Q"), ("tokenizer_size", "Q"),
    ("data_offset", "Q"), ("data_size", "Q"),
    ("vocab_size", "I"), ("d_model", "I"), ("n_layers", "I"), ("n_heads", "I"), ("n_kv_heads", "I"),
    ("head_dim", "I"), ("d_ff", "I"), ("window", "I"),
    ("n_banks", "I"), ("primes", "8I"), ("n_cells", "I"),
    ("rms_eps", "f"), ("rope_theta", "f"), ("vault_eps", "f"),
    ("bos_id", "I"), ("eos_id", "I"), ("im_start_id", "I"), ("im_end_id", "I"), ("pad_id", "I"),
    ("weight_format", "I"), ("flags", "I"), ("model_name", "64s"),
    ("n_sink", "I"),
    ("seg_budget", "I"), ("seg_hidden", "I"), ("seg_min", "I"), ("seg_max", "I"), ("seg_n_feat", "I"),
    ("seg_layers", "4I"),
)
_HEADER_STRUCT = struct.Struct("<" + "".join(code for _, code in _HEADER_FIELDS))
# Directory entry: id, dtype, ndim, dims[4], reserved, offset, nbytes, crc32, 12 pad bytes, name[64] (tools/vlt3.py:75).
_ENTRY_STRUCT = struct.Struct("<III4IIQQI12x64s")
assert _ENTRY_STRUCT.size == ENTRY_SIZE and _HEADER_STRUCT.size <= HEADER_SIZE - 4

Q8_BLOCK = np.dtype([("d", "<f2"), ("q", "i1", (QK,))])
Q4_BLOCK = np.dtype([("d", "<f2"), ("q", "u1", (QK // 2,))])
# Candidate scale ratios searched by the clipped-MSE Q4_0 quantizer (tools/vlt3.py:123).
_Q4_RATIOS = np.array([-1.0 / 8.0, -0.98 / 8.0, -0.96 / 8.0, -0.94 / 8.0, -0.92 / 8.0, -0.89 / 8.0,
                       1.0 / 7.5, 0.96 / 7.5], dtype=np.float32)


class VLT3Error(ValueError):
    """Malformed or unsafe VLT3 file (same role as tools/vlt3.py:411 VLT3Error)."""


class PreEncoded:
    """A tensor the writer does not hold as floats: `encode(dtype)` returns its payload bytes for the storage type
    the writer picked (lets large synthetic models be generated and quantized elsewhere, e.g. on a GPU)."""

    def __init__(self, shape, encode):
        self.shape = tuple(shape)
        self.encode = encode


def tensor_id(name: str) -> int:
    if name in _GLOBAL_BY_NAME:
        return _GLOBAL_BY_NAME[name]
    if not name.startswith("layers."):
        raise KeyError(f"unknown tensor name {name!r}")
    _, layer, kind = name.split(".", 2)
    return ((int(layer) + 1) << 8) | _KIND_BY_NAME[kind]


def tensor_name(tid: int) -> str:
    if tid < 256:
        return GLOBAL_TENSORS[tid]
    return f"layers.{(tid >> 8) - 1}.{LAYER_KINDS[(tid & 0xFF) - 1]}"


# ----------------------------------------------------------------------------------------------------------
# Block codecs
# ----------------------------------------------------------------------------------------------------------

def quantize_q8_0(w: np.ndarray) -> bytes:
    """Absmax Q8_0: d = max|x|/127 (rounded to fp16 for storage), q = clip(rint(x/d)) (tools/vlt3.py:102-111)."""
    x = np.ascontiguousarray(w, dtype=np.float32).reshape(-1, QK)
    d = np.abs(x).max(axis=1) / np.float32(127.0)
    safe = np.where(d > 0, d, np.float32(1.0))
    inv = np.where(d > 0, np.float32(1.0) / safe, np.float32(0.0))
    blocks = np.empty(x.shape[0], dtype=Q8_BLOCK)
    blocks["d"] = d.astype(np.float16)
    blocks["q"] = np.clip(np.rint(x * inv[:, None]), -127, 127).astype(np.int8)
    return blocks.tobytes()


def dequantize_q8_0(buf, n: int) -> np.ndarray:
    """q * d in fp32 (exact: int8 x fp16 fits a 24-bit mantissa) (tools/vlt3.py:114-116)."""
    b = np.frombuffer(buf, dtype=Q8_BLOCK, count=n // QK)
    return (b["q"].astype(np.float32) * b["d"].astype(np.float32)[:, None]).reshape(-1)


def quantize_q4_0(w: np.ndarray) -> bytes:
    """Clipped-MSE Q4_0: for each block try 8 signed scale ratios of the absmax element and keep the first one
    with the strictly smallest squared reconstruction error (tools/vlt3.py:119-149)."""
    x = np.ascontiguousarray(w, dtype=np.float32).reshape(-1, QK)
    nb = x.shape[0]
    blocks = np.empty(nb, dtype=Q4_BLOCK)
    for s in range(0, nb, 262144):
        xb = x[s:s + 262144]
        rows = np.arange(xb.shape[0])
        mx = xb[rows, np.abs(xb).argmax(axis=1)]
        best_err = np.full(xb.shape[0], np.inf, dtype=np.float32)
        best_d = np.zeros(xb.shape[0], dtype=np.float16)
        best_q = np.full((xb.shape[0], QK), 8, dtype=np.uint8)
        nonzero = mx != 0.0
        if nonzero.any():
            for ratio in _Q4_RATIOS:
                d16 = (mx * ratio).astype(np.float16)
                d32 = d16.astype(np.float32)
                inv = np.where(d32 != 0.0, np.float32(1.0) / np.where(d32 != 0.0, d32, np.float32(1.0)),
                               np.float32(0.0))
                qi = np.clip(np.rint(xb * inv[:, None] + np.float32(8.0)), 0.0, 15.0).astype(np.uint8)
                err = np.square((qi.astype(np.float32) - np.float32(8.0)) * d32[:, None] - xb).sum(axis=1)
                better = nonzero & (err < best_err)
                if better.any():
                    best_err[better] = err[better]
                    best_d[better] = d16[better]
                    best_q[better] = qi[better]
        blocks["d"][s:s + 262144] = best_d
        blocks["q"][s:s + 262144] = best_q[:, :QK // 2] | (best_q[:, QK // 2:] << 4)
    return blocks.tobytes()


def dequantize_q4_0(buf, n: int) -> np.ndarray:
    b = np.frombuffer(buf, dtype=Q4_BLOCK, count=n // QK)
    lo = (b["q"] & 0x0F).astype(np.int32) - 8
    hi = (b["q"] >> 4).astype(np.int32) - 8
    q = np.concatenate([lo, hi], axis=1).astype(np.float32)
    return (q * b["d"].astype(np.float32)[:, None]).reshape(-1)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit pattern (uint16), identical to torch's .to(bfloat16) for finite x."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def nbytes_for(dtype: int, n: int) -> int:
    if dtype == F32:
        return 4 * n
    if dtype in (F16, BF16):
        return 2 * n
    if dtype in (Q8_0, Q4_0):
        if n % QK:
            raise VLT3Error("quantized tensor size not a multiple of 32")
        return (n // QK) * (34 if dtype == Q8_0 else 18)
    raise VLT3Error(f"unknown dtype {dtype}")


def encode_array(a: np.ndarray, dtype: int) -> bytes:
    a = np.ascontiguousarray(a, dtype=np.float32)
    if dtype == F32:
        return a.astype("<f4").tobytes()
    if dtype == F16:
        return a.astype("<f2").tobytes()
    if dtype == BF16:
        return f32_to_bf16_bits(a).astype("<u2").tobytes()
    if dtype == Q8_0:
        return quantize_q8_0(a)
    if dtype == Q4_0:
        return quantize_q4_0(a)
    raise VLT3Error(f"unknown dtype {dtype}")


def decode_array(buf, dtype: int, shape: Sequence[int]) -> np.ndarray:
    """Dequantize/widen a tensor payload to fp32 (tools/vlt3.py:189-204)."""
    n = int(np.prod(shape))
    if dtype == F32:
        a = np.frombuffer(buf, dtype="<f4", count=n).copy()
    elif dtype == F16:
        a = np.frombuffer(buf, dtype="<f2", count=n).astype(np.float32)
    elif dtype == BF16:
        a = (np.frombuffer(buf, dtype="<u2", count=n).astype(np.uint32) << 16).view(np.float32)
    elif dtype == Q8_0:
        a = dequantize_q8_0(buf, n)
    elif dtype == Q4_0:
        a = dequantize_q4_0(buf, n)
    else:
        raise VLT3Error(f"unknown dtype {dtype}")
    return a.reshape(tuple(shape))


def choose_dtype(name: str, fmt: str, n_layers: int = 0) -> int:
    """Per-tensor storage type for a file format (tools/vlt3.py:312-330).

    Hybrid Q4_0 keeps the tied embedding, every k/v projection, and the q/o projections of the first two and
    last two layers in Q8_0; norms, biases and the segment scorer stay F32."""
    if fmt == "f32":
        return F32
    if name == "embed_tokens.weight":
        return BF16 if fmt == "bf16" else Q8_0
    layer, kind = -1, name
    if name.startswith("layers."):
        _, layer_s, kind = name.split(".", 2)
        layer = int(layer_s)
    if kind not in MATMUL_KINDS:
        return F32
    if fmt == "q4_0":
        if kind in ("self_attn.k_proj.weight", "self_attn.v_proj.weight"):
            return Q8_0
        if n_layers >= 8 and layer in (0, 1, n_layers - 2, n_layers - 1) and \
                kind in ("self_attn.q_proj.weight", "self_attn.o_proj.weight"):
            return Q8_0
    return FORMAT_CODES[fmt]


# ----------------------------------------------------------------------------------------------------------
# VTOK tokenizer blob (byte-level BPE tables; tools/vlt3.py:210-305)
# ----------------------------------------------------------------------------------------------------------

def byte_to_unicode() -> Dict[int, str]:
    """GPT-2 reversible byte -> printable-unicode map used by byte-level BPE vocabularies."""
    keep = list(range(0x21, 0x7F)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    out = {b: chr(b) for b in keep}
    extra = 0
    for b in range(256):
        if b not in out:
            out[b] = chr(256 + extra)
            extra += 1
    # keep the insertion order identical to the classic construction (kept bytes first, then the remapped ones)
    return {b: out[b] for b in keep + [b for b in range(256) if b not in keep]}


def _letter_number_ranges() -> List[Tuple[int, int, int]]:
    """Maximal code-point runs of Unicode letters (cat 1) and numbers (cat 2) for the pre-tokenizer."""
    ranges: List[Tuple[int, int, int]] = []
    lo, cat_run = 0, -1
    for cp in range(0x110000):
        c = unicodedata.category(chr(cp))[0]
        cat = 1 if c == "L" else (2 if c == "N" else 0)
        if cat != cat_run:
            if cat_run > 0:
                ranges.append((lo, cp - 1, cat_run))
            lo, cat_run = cp, cat
    if cat_run > 0:
        ranges.append((lo, 0x10FFFF, cat_run))
    return ranges


def build_tokenizer_blob(tokenizer_dir: str) -> Tuple[bytes, Dict[str, int]]:
    with open(os.path.join(tokenizer_dir, "tokenizer.json"), encoding="utf-8") as f:
        tj = json.load(f)
    u2b = {u: b for b, u in byte_to_unicode().items()}
    vocab: Dict[str, int] = tj["model"]["vocab"]
    added = {a["content"]: a["id"] for a in tj.get("added_tokens", [])}
    n_vocab = max(max(vocab.values()), max(added.values()) if added else 0) + 1
    tok_bytes: List[bytes] = [b""] * n_vocab
    for s, i in vocab.items():
        tok_bytes[i] = bytes(u2b[ch] for ch in s)
    for s, i in added.items():
        tok_bytes[i] = s.encode("utf-8")
    merges = []
    for m in tj["model"]["merges"]:
        a, b = m.split(" ", 1) if isinstance(m, str) else m
        merges.append((vocab[a], vocab[b], vocab[a + b]))
    b2u = byte_to_unicode()
    byte_tok = [vocab[b2u[b]] for b in range(256)]
    specials = sorted(added.values())
    table = np.zeros((n_vocab, 2), dtype="<u4")
    pool = bytearray()
    for i, tb in enumerate(tok_bytes):
        table[i] = (len(pool), len(tb))
        pool += tb
    sections = [
        table.tobytes(), bytes(pool),
        np.asarray(merges, dtype="<u4").tobytes(),
        np.asarray(specials, dtype="<u4").tobytes(),
        np.asarray(_letter_number_ranges(), dtype="<u4").tobytes(),
        np.asarray(byte_tok, dtype="<u4").tobytes(),
    ]
    offsets, cur = [], 128
    for s in sections:
        cur = (cur + 7) & ~7
        offsets.append(cur)
        cur += len(s)
    head = struct.pack("<4sIIIIII", b"VTOK", 1, n_vocab, len(merges), len(specials),
                       len(sections[4]) // 12, 0) + struct.pack("<6Q", *offsets)
    blob = bytearray(head.ljust(128, b"\0"))
    for off, s in zip(offsets, sections):
        blob += b"\0" * (off - len(blob))
        blob += s
    ids = {
        "bos": added.get("<|endoftext|>", 0),
        "eos": added.get("<|im_end|>", 0),
        "im_start": added.get("<|im_start|>", 0),
        "im_end": added.get("<|im_end|>", 0),
        "pad": added.get("<|endoftext|>", 0),
    }
    return bytes(blob), ids


def parse_token_bytes(blob, vocab_size: int) -> List[bytes]:
    """Raw byte string of every token id (< vocab_size) from a VTOK blob; ids beyond the table map to b''."""
    mv = memoryview(blob)
    if len(mv) < 128 or bytes(mv[:4]) != b"VTOK":
        raise VLT3Error("malformed tokenizer blob")
    n_vocab = struct.unpack_from("<I", mv, 8)[0]
    o_tab, o_pool, o_mer = struct.unpack_from("<3Q", mv, 28)
    table = np.frombuffer(mv, dtype="<u4", count=2 * n_vocab, offset=o_tab).reshape(-1, 2)
    pool = bytes(mv[o_pool:o_mer])
    out = [b""] * vocab_size
    for i in range(min(n_vocab, vocab_size)):
        o, n = int(table[i, 0]), int(table[i, 1])
        out[i] = pool[o:o + n]
    return out


# ----------------------------------------------------------------------------------------------------------
# Writer
# ----------------------------------------------------------------------------------------------------------

def write_vlt3(path: str, state: Dict[str, "np.ndarray"], cfg, tokenizer_dir: str, fmt: str,
               model_name: str = "VAULT-v3") -> Dict:
    """Serialize a float state dict to VLT3 (tools/vlt3.py:333-402).  Values may be numpy arrays, torch tensors or
    zero-argument callables returning either (generated one at a time to bound host memory)."""
    names = sorted(state.keys(), key=tensor_id)
    n_layers = int(getattr(cfg, "n_layers", 0))
    entries, payloads = [], []
    for nm in names:
        arr = state[nm]
        if callable(arr):
            arr = arr()
        dt = choose_dtype(nm, fmt, n_layers)
        if isinstance(arr, PreEncoded):
            shape = tuple(arr.shape)
            if dt in (Q8_0, Q4_0) and shape[-1] % QK:
                dt = BF16
            data = arr.encode(dt)
        else:
            arr = arr.detach().float().cpu().numpy() if hasattr(arr, "detach") else np.asarray(arr, dtype=np.float32)
            shape = arr.shape
            if dt in (Q8_0, Q4_0) and arr.shape[-1] % QK:
                dt = BF16
            data = encode_array(arr, dt)
        if len(data) != nbytes_for(dt, int(np.prod(shape))):
            raise VLT3Error(f"{nm}: encoded size mismatch")
        dims = list(shape) + [1] * (4 - len(shape))
        entries.append(dict(id=tensor_id(nm), dtype=dt, ndim=len(shape), dims=dims, nbytes=len(data),
                            crc=zlib.crc32(data), name=nm))
        payloads.append(data)
    tok_blob, ids = build_tokenizer_blob(tokenizer_dir)

    def up(v: int) -> int:
        return (v + ALIGN - 1) // ALIGN * ALIGN

    dir_off = HEADER_SIZE
    tok_off = up(dir_off + ENTRY_SIZE * len(entries))
    data_off = up(tok_off + len(tok_blob))
    cur = data_off
    for e in entries:
        e["offset"] = cur = up(cur)
        cur += e["nbytes"]
    file_size = cur
    seg_layers = list(getattr(cfg, "seg_layers", ()) or ())
    n_feat = len(seg_layers) if (seg_layers and "seg_scorer.ln.weight" in state) else 0
    hv = dict(
        magic=MAGIC, version=VERSION, header_size=HEADER_SIZE, endian_tag=ENDIAN_TAG,
        file_size=file_size, alignment=ALIGN, n_tensors=len(entries),
        tensor_dir_offset=dir_off, tensor_dir_size=ENTRY_SIZE * len(entries),
        tokenizer_offset=tok_off, tokenizer_size=len(tok_blob),
        data_offset=data_off, data_size=file_size - data_off,
        vocab_size=cfg.vocab_size, d_model=cfg.d_model, n_layers=cfg.n_layers, n_heads=cfg.n_heads,
        n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, d_ff=cfg.d_ff, window=cfg.window,
        n_banks=0, primes=[0] * 8, n_cells=0,
        rms_eps=cfg.rms_eps, rope_theta=cfg.rope_theta, vault_eps=0.0,
        bos_id=ids["bos"], eos_id=ids["eos"], im_start_id=ids["im_start"], im_end_id=ids["im_end"],
        pad_id=ids["pad"], weight_format=FORMAT_CODES[fmt],
        flags=(1 if cfg.tie_embeddings else 0) | (4 if n_feat else 0),
        model_name=model_name.encode("utf-8")[:63], n_sink=int(getattr(cfg, "n_sink", 0)),
        seg_budget=int(getattr(cfg, "seg_budget", 0)) if n_feat else 0,
        seg_hidden=int(getattr(cfg, "seg_hidden", 256)) if n_feat else 0,
        seg_min=int(getattr(cfg, "seg_min", 16)) if n_feat else 0,
        seg_max=int(getattr(cfg, "seg_max", 48)) if n_feat else 0,
        seg_n_feat=n_feat, seg_layers=(seg_layers[:4] + [0] * 4)[:4],
    )
    flat: List = []
    for fname, code in _HEADER_FIELDS:
        v = hv[fname]
        flat.extend(v) if code in ("8I", "4I") else flat.append(v)
    head = _HEADER_STRUCT.pack(*flat).ljust(HEADER_SIZE - 4, b"\0")
    head += struct.pack("<I", zlib.crc32(head))
    with open(path, "wb") as f:
        f.write(head)
        for e in entries:
            f.write(_ENTRY_STRUCT.pack(e["id"], e["dtype"], e["ndim"], *e["dims"], 0, e["offset"], e["nbytes"],
                                       e["crc"], e["name"].encode()[:63]))
        f.write(b"\0" * (tok_off - f.tell()))
        f.write(tok_blob)
        for e, data in zip(entries, payloads):
            f.write(b"\0" * (e["offset"] - f.tell()))
            f.write(data)
        if f.tell() != file_size:
            raise VLT3Error("writer size mismatch")
    return {"file_size": file_size, "n_tensors": len(entries), "tokenizer_bytes": len(tok_blob)}


# ----------------------------------------------------------------------------------------------------------
# Reader / validator
# ----------------------------------------------------------------------------------------------------------

@dataclass
class VLT3File:
    header: Dict
    entries: List[Dict]
    buf: memoryview
    by_id: Dict[int, Dict] = field(default_factory=dict)

    def entry(self, name: str) -> Dict:
        return self.by_id[tensor_id(name)]

    def raw(self, name: str) -> memoryview:
        e = self.entry(name)
        return self.buf[e["offset"]: e["offset"] + e["nbytes"]]

    def tensor(self, name: str) -> np.ndarray:
        """fp32 copy of a tensor (dequantized when quantized)."""
        e = self.entry(name)
        return decode_array(self.raw(name), e["dtype"], e["dims"][: e["ndim"]])

    def tokenizer_blob(self) -> memoryview:
        h = self.header
        return self.buf[h["tokenizer_offset"]: h["tokenizer_offset"] + h["tokenizer_size"]]


def _finite_payload(buf, dt: int, n: int) -> bool:
    if dt == F32:
        return bool(np.isfinite(np.frombuffer(buf, dtype="<f4", count=n)).all())
    if dt == F16:
        return bool(np.isfinite(np.frombuffer(buf, dtype="<f2", count=n)).all())
    if dt == BF16:
        return not bool(((np.frombuffer(buf, dtype="<u2", count=n) & 0x7F80) == 0x7F80).any())
    blocks = np.frombuffer(buf, dtype=Q8_BLOCK if dt == Q8_0 else Q4_BLOCK, count=n // QK)
    return bool(np.isfinite(blocks["d"]).all())


def read_vlt3(path_or_bytes, check_crc: bool = True) -> VLT3File:
    """Parse and validate a VLT3 file (tools/vlt3.py:453-545).  Raises VLT3Error on any inconsistency."""
    if isinstance(path_or_bytes, (bytes, bytearray, memoryview)):
        data = bytes(path_or_bytes)
    else:
        with open(path_or_bytes, "rb") as f:
            data = f.read()
    size = len(data)
    if size < HEADER_SIZE:
        raise VLT3Error("file smaller than header")
    if zlib.crc32(data[: HEADER_SIZE - 4]) != struct.unpack_from("<I", data, HEADER_SIZE - 4)[0]:
        raise VLT3Error("header CRC mismatch")
    vals = list(_HEADER_STRUCT.unpack_from(data, 0))
    h: Dict = {}
    for fname, code in _HEADER_FIELDS:
        k = 8 if code == "8I" else (4 if code == "4I" else 1)
        h[fname] = vals[:k] if k > 1 else vals[0]
        del vals[:k]
    if (h["magic"] != MAGIC or h["version"] != VERSION or h["header_size"] != HEADER_SIZE
            or h["endian_tag"] != ENDIAN_TAG):
        raise VLT3Error("bad magic/version/header_size/endianness")
    if h["file_size"] != size:
        raise VLT3Error(f"file_size {h['file_size']} != actual {size}")
    if h["alignment"] != ALIGN:
        raise VLT3Error("unsupported alignment")
    for what, off_k, n_k in (("tensor directory", "tensor_dir_offset", "tensor_dir_size"),
                             ("tokenizer", "tokenizer_offset", "tokenizer_size"),
                             ("data", "data_offset", "data_size")):
        off, n = h[off_k], h[n_k]
        if off < HEADER_SIZE or off > size or n > size - off:
            raise VLT3Error(f"{what} out of bounds")
    if h["tensor_dir_size"] != h["n_tensors"] * ENTRY_SIZE:
        raise VLT3Error("tensor_dir_size != n_tensors * 128")
    if not (0 < h["n_layers"] <= 64) or not (0 < h["n_heads"] <= 256) or not (0 < h["head_dim"] <= 256):
        raise VLT3Error("bad layer/head dimensions")
    if h["n_kv_heads"] == 0 or h["n_heads"] % h["n_kv_heads"] or h["n_heads"] * h["head_dim"] != h["d_model"]:
        raise VLT3Error("inconsistent GQA/d_model dimensions")
    if h["n_sink"] > 512 or h["n_sink"] > h["window"]:
        raise VLT3Error("bad n_sink")
    if h["n_banks"] or h["n_cells"] or any(h["primes"]):
        raise VLT3Error("bad vault bank description (expected 0 in Kenyon-free VLT3)")
    if not (np.isfinite(h["rms_eps"]) and h["rms_eps"] > 0 and np.isfinite(h["rope_theta"])
            and h["rope_theta"] > 1.0 and np.isfinite(h["vault_eps"])):
        raise VLT3Error("non-finite or invalid eps/theta")
    nf = h["seg_n_feat"]
    if nf > 0:
        if nf > 4 or not (0 < h["seg_hidden"] <= 1024) or not (0 < h["seg_min"] <= h["seg_max"] <= h["window"]):
            raise VLT3Error("invalid segment scorer hyperparameters")
        if h["seg_budget"] > 16384 or any(l >= h["n_layers"] for l in h["seg_layers"][:nf]):
            raise VLT3Error("invalid segment budget or feature layers")
    buf = memoryview(data)
    entries: List[Dict] = []
    by_id: Dict[int, Dict] = {}
    spans = []
    for k in range(h["n_tensors"]):
        tid, dt, ndim, d0, d1, d2, d3, rsv, off, nb, crc, nm = _ENTRY_STRUCT.unpack_from(
            data, h["tensor_dir_offset"] + k * ENTRY_SIZE)
        dims = [d0, d1, d2, d3]
        if rsv:
            raise VLT3Error(f"tensor entry {k}: reserved field not zero")
        if tid in by_id:
            raise VLT3Error(f"duplicate tensor id {tid}")
        if dt not in DTYPE_NAMES or not (1 <= ndim <= 4) or any(x == 0 for x in dims[:ndim]):
            raise VLT3Error(f"bad dtype/ndim/zero-dim for tensor {tid}")
        n = int(np.prod([int(x) for x in dims[:ndim]]))
        if dt in (Q8_0, Q4_0) and n % QK:
            raise VLT3Error(f"tensor {tid}: quantized size not a multiple of 32")
        if nb != nbytes_for(dt, n):
            raise VLT3Error(f"tensor {tid}: nbytes {nb} inconsistent with dtype/dims")
        if off % ALIGN or off < h["data_offset"] or nb > h["data_offset"] + h["data_size"] - off:
            raise VLT3Error(f"tensor {tid}: offset out of data region or misaligned")
        if check_crc and zlib.crc32(buf[off: off + nb]) != crc:
            raise VLT3Error(f"tensor {tid}: CRC mismatch")
        if not _finite_payload(buf[off: off + nb], dt, n):
            raise VLT3Error(f"tensor {tid}: non-finite values")
        spans.append((off, off + nb))
        e = dict(id=tid, dtype=dt, ndim=ndim, dims=dims, offset=off, nbytes=nb, crc=crc,
                 name=nm.rstrip(b"\0").decode("utf-8", "replace"))
        entries.append(e)
        by_id[tid] = e
    spans.sort()
    for (_a0, a1), (b0, _b1) in zip(spans, spans[1:]):
        if b0 < a1:
            raise VLT3Error("overlapping tensors")
    need = {1, 2} | {((l + 1) << 8) | (j + 1) for l in range(h["n_layers"]) for j in range(len(LAYER_KINDS))}
    if nf > 0:
        need |= set(SCORER_IDS)
    missing = need - set(by_id)
    if missing:
        raise VLT3Error(f"missing tensors: {sorted(missing)[:5]}")
    return VLT3File(h, entries, buf, by_id)


def vlt3_to_state_dict(vf: VLT3File) -> Dict[str, np.ndarray]:
    return {tensor_name(e["id"]): vf.tensor(tensor_name(e["id"])) for e in vf.entries}


def vlt3_config(vf: VLT3File):
    """Model hyper-parameters stored in a VLT3 header (tools/vlt3.py:552-566)."""
    from .config import VAULTv3Config
    h = vf.header
    nf = h["seg_n_feat"]
    return VAULTv3Config(
        vocab_size=h["vocab_size"], d_model=h["d_model"], n_layers=h["n_layers"], n_heads=h["n_heads"],
        n_kv_heads=h["n_kv_heads"], head_dim=h["head_dim"], d_ff=h["d_ff"], rms_eps=h["rms_eps"],
        rope_theta=h["rope_theta"], tie_embeddings=bool(h["flags"] & 1), window=h["window"], n_sink=h["n_sink"],
        seg_budget=h["seg_budget"] if nf else 0,
        seg_hidden=h["seg_hidden"] if nf else 256,
        seg_min=h["seg_min"] if nf else 16,
        seg_max=h["seg_max"] if nf else 48,
        seg_layers=tuple(h["seg_layers"][:nf]) if nf else (),
    )
