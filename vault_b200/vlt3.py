"""VLT3 checkpoint container: reader, validator, writer and Q8_0/Q4_0 block codecs.

Counterpart of the reference's `tools/vlt3.py`.  The VLT3 format is an on-disk contract, so the byte layout, field
order, tensor ids, block layouts and the codecs' arithmetic are the same (the writer is checked byte-identical
against the reference writer); validation is the engine's own C++ loader check (v3g_validate), shared with the
device loader.

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
_Q4_SLICE = 1 << 15   # blocks per candidate evaluation (8 x 32 x 4 B per block)


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


def _q4_candidates(xb: np.ndarray):
    """Every candidate encoding of a stack of blocks: fp16 scales [n, R] (the block's signed absmax element times
    each ratio of _Q4_RATIOS), their codes [n, R, 32] and squared reconstruction errors [n, R] (fp32 sums)."""
    n = xb.shape[0]
    peak = xb[np.arange(n), np.abs(xb).argmax(axis=1)]                 # signed element of largest magnitude
    d16 = (peak[:, None] * _Q4_RATIOS[None, :]).astype(np.float16)     # [n, R]
    d = d16.astype(np.float32)
    inv = np.divide(np.float32(1.0), d, out=np.zeros_like(d), where=d != 0.0)
    codes = np.clip(np.rint(xb[:, None, :] * inv[:, :, None] + np.float32(8.0)), 0.0, 15.0).astype(np.uint8)
    recon = (codes.astype(np.float32) - np.float32(8.0)) * d[:, :, None]
    err = np.square(recon - xb[:, None, :]).sum(axis=2)
    return peak, d16, codes, err


def quantize_q4_0(w: np.ndarray) -> bytes:
    """Clipped-MSE Q4_0 (tools/vlt3.py:119-149): each block takes the candidate scale of smallest squared error,
    the earliest ratio on ties; all-zero blocks (and blocks where no candidate has a finite error) keep d = 0 and
    every code 8.  Blocks are processed in slices to bound the [n, 8, 32] candidate arrays."""
    x = np.ascontiguousarray(w, dtype=np.float32).reshape(-1, QK)
    blocks = np.zeros(x.shape[0], dtype=Q4_BLOCK)
    blocks["q"] = 0x88
    for lo in range(0, x.shape[0], _Q4_SLICE):
        xb = x[lo:lo + _Q4_SLICE]
        peak, d16, codes, err = _q4_candidates(xb)
        err = np.where(np.isnan(err), np.float32(np.inf), err)
        pick = err.argmin(axis=1)                                         # first minimum = earliest ratio on ties
        rows = np.arange(xb.shape[0])
        ok = (peak != 0.0) & np.isfinite(err[rows, pick])
        q = codes[rows, pick]                                             # [n, 32]: element j, j + 16 share a byte
        sel = blocks[lo:lo + xb.shape[0]]
        sel["d"] = np.where(ok, d16[rows, pick], np.float16(0.0))
        sel["q"] = np.where(ok[:, None], q[:, :QK // 2] | (q[:, QK // 2:] << 4), np.uint8(0x88))
        blocks[lo:lo + xb.shape[0]] = sel
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


# Roles of the ChatML control tokens in the header (tools/vlt3.py:299-305): role -> added-token text
_CONTROL_ROLES = (("bos", "<|endoftext|>"), ("eos", "<|im_end|>"), ("im_start", "<|im_start|>"),
                  ("im_end", "<|im_end|>"), ("pad", "<|endoftext|>"))
_VTOK_HEAD, _VTOK_ALIGN = 128, 8


def _token_strings(tj: dict) -> Dict[int, bytes]:
    """id -> raw bytes of every vocabulary entry (byte-level strings decoded) and added token (UTF-8 text); an
    added token overrides a vocabulary entry of the same id."""
    decode = {ch: b for b, ch in byte_to_unicode().items()}
    strings = {tid: bytes(decode[ch] for ch in text) for text, tid in tj["model"]["vocab"].items()}
    strings.update({a["id"]: a["content"].encode("utf-8") for a in tj.get("added_tokens", [])})
    return strings


def _pack_sections(fixed: bytes, sections: Sequence[bytes]) -> bytes:
    """VTOK container: `fixed` header fields, then the section offsets (u64 each), padded to _VTOK_HEAD bytes; each
    section starts at the next multiple of _VTOK_ALIGN."""
    offsets, end = [], _VTOK_HEAD
    for sec in sections:
        start = -(-end // _VTOK_ALIGN) * _VTOK_ALIGN
        offsets.append(start)
        end = start + len(sec)
    out = bytearray(end)
    head = fixed + struct.pack(f"<{len(offsets)}Q", *offsets)
    out[:len(head)] = head
    for start, sec in zip(offsets, sections):
        out[start:start + len(sec)] = sec
    return bytes(out)


def build_tokenizer_blob(tokenizer_dir: str) -> Tuple[bytes, Dict[str, int]]:
    """The VTOK tokenizer section of a VLT3 file from a byte-level BPE `tokenizer.json` (format of
    tools/vlt3.py:246-305): a string table (offset, length per id) into one byte pool, the merge triples
    (left, right, merged), the sorted control-token ids, the letter/number code-point runs of the pre-tokenizer and
    the id of every single byte.  Returns the blob and the control-token ids of the header."""
    with open(os.path.join(tokenizer_dir, "tokenizer.json"), encoding="utf-8") as f:
        tj = json.load(f)
    vocab: Dict[str, int] = tj["model"]["vocab"]
    strings = _token_strings(tj)
    n_vocab = max(strings) + 1
    ordered = [strings.get(i, b"") for i in range(n_vocab)]
    lengths = np.fromiter((len(t) for t in ordered), dtype=np.int64, count=n_vocab)
    starts = np.cumsum(lengths) - lengths
    table = np.stack([starts, lengths], axis=1).astype("<u4")
    pairs = (m.split(" ", 1) if isinstance(m, str) else m for m in tj["model"]["merges"])
    merges = np.array([(vocab[l], vocab[r], vocab[l + r]) for l, r in pairs], dtype="<u4").reshape(-1, 3)
    added = {a["content"]: a["id"] for a in tj.get("added_tokens", [])}
    controls = np.array(sorted(added.values()), dtype="<u4")
    runs = np.array(_letter_number_ranges(), dtype="<u4").reshape(-1, 3)
    b2u = byte_to_unicode()
    byte_ids = np.array([vocab[b2u[b]] for b in range(256)], dtype="<u4")
    fixed = struct.pack("<4s6I", b"VTOK", 1, n_vocab, merges.shape[0], controls.size, runs.shape[0], 0)
    blob = _pack_sections(fixed, [table.tobytes(), b"".join(ordered), merges.tobytes(), controls.tobytes(),
                                  runs.tobytes(), byte_ids.tobytes()])
    return blob, {role: added.get(text, 0) for role, text in _CONTROL_ROLES}


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


def aligned_buffer(src) -> np.ndarray:
    """Host copy of a VLT3 file (path or bytes) in a 64-byte aligned uint8 buffer: the alignment the format's
    readers require of a model buffer (runtime/vault3.h:8)."""
    if isinstance(src, (bytes, bytearray, memoryview)):
        data = np.frombuffer(src, dtype=np.uint8)
        n = data.size
    else:
        data, n = None, os.path.getsize(src)
    raw = np.empty(n + ALIGN, dtype=np.uint8)
    off = (-raw.ctypes.data) % ALIGN
    buf = raw[off:off + n]
    if data is not None:
        buf[:] = data
    else:
        with open(src, "rb") as f:
            f.readinto(memoryview(buf))
    return buf


def _unpack_header(buf) -> Dict:
    """Header fields by name (the _HEADER_FIELDS table; array fields as lists)."""
    flat = iter(_HEADER_STRUCT.unpack_from(buf, 0))
    out: Dict = {}
    for fname, code in _HEADER_FIELDS:
        count = int(code[:-1]) if code[:-1].isdigit() and code[-1] == "I" else 1
        out[fname] = [next(flat) for _ in range(count)] if count > 1 else next(flat)
    return out


def _unpack_entry(buf, at: int) -> Dict:
    tid, dt, ndim, d0, d1, d2, d3, _reserved, off, nb, crc, nm = _ENTRY_STRUCT.unpack_from(buf, at)
    return dict(id=tid, dtype=dt, ndim=ndim, dims=[d0, d1, d2, d3], offset=off, nbytes=nb, crc=crc,
                name=nm.rstrip(b"\0").decode("utf-8", "replace"))


def read_vlt3(path_or_bytes, check_crc: bool = True) -> VLT3File:
    """Open a VLT3 file (the role of tools/vlt3.py:453-545 read_vlt3).

    The file is validated by the engine's own loader checks (v3g_validate: the rules of the reference C runtime's
    v3_load, runtime/vault3.c:273-455 -- bounds, alignment, dtypes and shapes of every required tensor, finite
    scales and weights, CRCs when check_crc, the tokenizer section), so this reader and the device loader accept
    exactly the same files.  A rejected file raises VLT3Error naming the status code and the failed check."""
    from . import _lib

    buf = aligned_buffer(path_or_bytes)
    L = _lib.lib()
    rc = L.v3g_validate(buf.ctypes.data, buf.size, int(bool(check_crc)))
    if rc != 0:
        raise VLT3Error(f"{L.v3g_error_string(rc).decode()} ({rc}): {_lib.last_error()}")
    mv = memoryview(buf)
    header = _unpack_header(mv)
    entries = [_unpack_entry(mv, header["tensor_dir_offset"] + k * ENTRY_SIZE) for k in range(header["n_tensors"])]
    return VLT3File(header, entries, mv, {e["id"]: e for e in entries})


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
