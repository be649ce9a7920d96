"""CPU: VLT3 validation (Python reader and the engine's C++ loader) on the malformed files of the reference's
loader-fuzz test (tests/test_vlt3_runtime.py:141-218), and the C ABI's exported symbols."""

import ctypes as C
import os
import re
import struct
import subprocess
import zlib

import numpy as np
import pytest

from vault_b200 import _lib, vlt3

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_HOST = os.path.join(REPO, "oracle", "_ref", "vault3_host")


def _fix_header_crc(b: bytearray) -> None:
    struct.pack_into("<I", b, 4092, zlib.crc32(bytes(b[:4092])) & 0xFFFFFFFF)


def _set_entry_crc(b: bytearray, dir_off: int, n: int, tid: int, off: int, nb: int) -> None:
    for k in range(n):
        eo = dir_off + 128 * k
        if struct.unpack_from("<I", b, eo)[0] == tid:
            struct.pack_into("<I", b, eo + 48, zlib.crc32(bytes(b[off:off + nb])) & 0xFFFFFFFF)
            return


def corrupt_cases(good: bytes):
    """(name, bytes, verify_crc, expected engine status) -- same corruptions as the reference's fuzz test."""
    raw = bytearray(good)
    vf = vlt3.read_vlt3(good)
    dir_off = struct.unpack_from("<Q", raw, 32)[0]
    n_t = vf.header["n_tensors"]
    t0_off = struct.unpack_from("<Q", raw, dir_off + 32)[0]
    out = []
    b = bytearray(raw); b[0:4] = b"BAD!"; out.append(("bad_magic", b, True, -2))
    b = bytearray(raw); b[80] ^= 0xFF; out.append(("bad_hdr_crc", b, True, -3))
    out.append(("truncated", bytearray(raw[:-128]), True, -1))
    b = bytearray(raw); struct.pack_into("<Q", b, 32, len(raw) + 4096); _fix_header_crc(b)
    out.append(("oob_dir_off", b, True, -4))
    b = bytearray(raw); struct.pack_into("<Q", b, dir_off + 32, t0_off + 8); out.append(("unaligned_tensor", b, True, -4))
    b = bytearray(raw); struct.pack_into("<Q", b, dir_off + 40, len(raw) * 2); out.append(("oob_tensor_size", b, True, -7))
    b = bytearray(raw); b[t0_off + 4] ^= 0x55; out.append(("corrupt_tensor_crc", b, True, -3))
    b = bytearray(raw)
    for off, val in ((84, 65536), (92, 65536), (100, 65536)):
        struct.pack_into("<I", b, off, val)
    _fix_header_crc(b)
    out.append(("u32_hd_overflow", b, True, -10))
    e = vf.by_id[2]
    b = bytearray(raw); struct.pack_into("<I", b, e["offset"], 0x7FC00000)
    _set_entry_crc(b, dir_off, n_t, 2, e["offset"], e["nbytes"])
    out.append(("nan_norm_weight", b, True, -12))
    e = vf.by_id[1]
    b = bytearray(raw); struct.pack_into("<H", b, e["offset"] + (e["nbytes"] // 34) // 2 * 34, 0x7E00)
    _set_entry_crc(b, dir_off, n_t, 1, e["offset"], e["nbytes"])
    out.append(("nan_q8_midblock_unverified", b, False, -12))
    b = bytearray(raw); struct.pack_into("<I", b, 112, 3); _fix_header_crc(b)
    out.append(("nonzero_legacy_nbanks", b, False, -10))
    return out


@pytest.fixture(scope="module")
def good_q8(case_files):
    with open(case_files("tiny_seg_q8_0"), "rb") as f:
        return f.read()


def _engine_load(data: bytes, verify: bool) -> int:
    buf = np.empty(len(data) + 64, np.uint8)
    off = (-buf.ctypes.data) % 64
    a = buf[off:off + len(data)]
    a[:] = np.frombuffer(data, np.uint8)
    h = C.c_void_p()
    rc = _lib.lib().v3g_load(C.byref(h), C.c_void_p(a.ctypes.data), len(data), int(verify), 0, 0)
    if rc == 0:
        _lib.lib().v3g_free(h)
    return rc


def test_python_reader_rejects_corrupt_files(good_q8):
    vlt3.read_vlt3(good_q8)
    for name, data, verify, _ in corrupt_cases(good_q8):
        with pytest.raises(vlt3.VLT3Error):
            vlt3.read_vlt3(bytes(data), check_crc=verify)
            pytest.fail(name)


def test_engine_loader_rejects_corrupt_files(good_q8):
    # validation runs on the host before any device work, so this needs no GPU
    for name, data, verify, code in corrupt_cases(good_q8):
        assert _engine_load(bytes(data), verify) == code, name
    assert _engine_load(good_q8, True) not in _lib.FILE_ERRORS


def test_engine_loader_rejects_misaligned_buffer(good_q8):
    buf = np.empty(len(good_q8) + 128, np.uint8)
    off = (-buf.ctypes.data) % 64 + 8
    a = buf[off:off + len(good_q8)]
    a[:] = np.frombuffer(good_q8, np.uint8)
    h = C.c_void_p()
    assert _lib.lib().v3g_load(C.byref(h), C.c_void_p(a.ctypes.data), len(good_q8), 1, 0, 0) == -11


def test_file_validation_matches_buffer_validation(good_q8, tmp_path):
    """v3g_validate_file (the file mapped read-only, read in place) gives the codes of v3g_validate on an aligned
    copy, for the good file and every corrupt case; a missing file is an argument error, an empty one a size error."""
    L = _lib.lib()
    cases = [("good", bytearray(good_q8), True, None)] + list(corrupt_cases(good_q8))
    for name, data, verify, _ in cases:
        p = tmp_path / f"{name}.vlt3"
        p.write_bytes(bytes(data))
        buf = vlt3.aligned_buffer(bytes(data))
        want = L.v3g_validate(C.c_void_p(buf.ctypes.data), buf.size, int(verify))
        assert L.v3g_validate_file(str(p).encode(), int(verify)) == want, name
    assert L.v3g_validate_file(str(tmp_path / "good.vlt3").encode(), 1) == 0
    assert L.v3g_validate_file(str(tmp_path / "missing.vlt3").encode(), 0) == -21
    (tmp_path / "empty.vlt3").write_bytes(b"")
    assert L.v3g_validate_file(str(tmp_path / "empty.vlt3").encode(), 0) == -1


@pytest.mark.skipif(not os.path.exists(REF_HOST), reason="reference C runtime not built (oracle/Makefile)")
def test_reference_runtime_agrees_on_rejections(good_q8, tmp_path):
    for name, data, verify, _ in corrupt_cases(good_q8):
        p = tmp_path / f"{name}.vlt3"
        p.write_bytes(bytes(data))
        r = subprocess.run([REF_HOST, str(p), *(["--verify"] if verify else []), "--bench", "1"],
                           capture_output=True, text=True, timeout=120)
        assert r.returncode == 2, name


def test_library_exports_every_declared_symbol():
    with open(os.path.join(REPO, "include", "vault_b200.h")) as f:
        decl = set(re.findall(r"^V3G_API\s+[\w\s\*]*?\b(v3g_\w+)\s*\(", f.read(), re.M))
    assert decl, "no declarations parsed"
    assert decl == set(_lib.exported_symbols())
    L = _lib.lib()
    for name in decl:
        assert getattr(L, name) is not None
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert decl <= exported


def test_round_trip_dequant(good_q8):
    vf = vlt3.read_vlt3(good_q8)
    w = vf.tensor("layers.0.self_attn.q_proj.weight")
    assert w.dtype == np.float32 and w.shape == (64, 64)


def test_config_from_qwen_config_and_dict_round_trip():
    """VAULTv3Config.from_qwen_config maps a Qwen2 config.json the way src/vault_v3_model.py:87-103 does (the
    Qwen2.5-1.5B numbers give the default v3 backbone), overrides apply, and to_dict / from_dict round-trip."""
    from vault_b200 import VAULTv3Config
    qc = {"vocab_size": 151936, "hidden_size": 1536, "num_hidden_layers": 28, "num_attention_heads": 12,
          "num_key_value_heads": 2, "intermediate_size": 8960, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0,
          "tie_word_embeddings": True}
    cfg = VAULTv3Config.from_qwen_config(qc, seg_budget=1024, seg_layers=(8, 16, 24))
    assert cfg == VAULTv3Config(seg_budget=1024, seg_layers=(8, 16, 24))
    assert cfg.head_dim == 128 and cfg.group_size == 6 and cfg.n_cells == 0 and cfg.has_seg_scorer
    assert VAULTv3Config.from_dict(cfg.to_dict()) == cfg
    assert VAULTv3Config.from_qwen_config(dict(qc, tie_word_embeddings=False)).tie_embeddings is False
