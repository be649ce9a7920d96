"""ctypes binding of the reference's own governor (runtime/vault3.h:191-216) in oracle/_ref/libvault3.so, which
oracle/Makefile builds from the reference sources: the checker for the engine's governor.  Test infrastructure."""
import ctypes as C
import os

import numpy as np
import pytest

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libvault3.so")


class RefGov(C.Structure):
    """v3_governor (runtime/vault3.h:198-209)."""
    _fields_ = [("active", C.c_int), ("n_rules", C.c_uint32), ("rules", (C.c_uint8 * 32) * 8),
                ("rule_len", C.c_uint32 * 8), ("hist", C.c_uint8 * 64), ("hist_len", C.c_uint32),
                ("utf8_rem", C.c_uint8 * 4), ("utf8_len", C.c_uint32), ("raw_tail", C.c_uint8 * 96),
                ("raw_len", C.c_uint32)]


def ref_lib() -> C.CDLL:
    if not os.path.exists(LIB):
        pytest.skip("oracle/_ref/libvault3.so is not built (oracle/Makefile needs the reference sources)")
    L = C.CDLL(LIB)
    L.ref_sizeof_model.restype = C.c_size_t
    L.ref_sizeof_governor.restype = C.c_size_t
    gp = C.POINTER(RefGov)
    L.v3_gov_init.argtypes = [gp]
    L.v3_gov_add_rule.argtypes = [gp, C.c_char_p, C.c_size_t]
    L.v3_gov_add_rule.restype = C.c_int
    L.v3_gov_arm_system.argtypes = [gp, C.c_char_p, C.c_size_t]
    L.v3_govern_logits.argtypes = [gp, C.c_void_p, C.c_void_p, C.c_uint32]
    L.v3_gov_commit.argtypes = [gp, C.c_void_p, C.c_uint32]
    L.v3_load.argtypes = [C.c_void_p, C.c_void_p, C.c_uint64, C.c_int]
    L.v3_load.restype = C.c_int
    L.v3_token_bytes.argtypes = [C.c_void_p, C.c_uint32, C.POINTER(C.POINTER(C.c_uint8)), C.POINTER(C.c_uint32)]
    L.v3_token_bytes.restype = C.c_int
    assert L.ref_sizeof_governor() == C.sizeof(RefGov)
    return L


class RefModel:
    """A VLT3 file loaded by the reference's v3_load (from a page-aligned copy, as its alignment rule asks)."""

    def __init__(self, L: C.CDLL, path: str):
        raw = open(path, "rb").read()
        self._arr = np.empty(len(raw) + 4096, np.uint8)
        off = (-self._arr.ctypes.data) % 4096
        self._buf = self._arr[off:off + len(raw)]
        self._buf[:] = np.frombuffer(raw, np.uint8)
        self.handle = C.create_string_buffer(L.ref_sizeof_model())
        rc = L.v3_load(self.handle, self._buf.ctypes.data, len(raw), 1)
        assert rc == 0, rc
        self.L = L

    def token_bytes(self, vocab: int) -> list:
        out = []
        for i in range(vocab):
            p, n = C.POINTER(C.c_uint8)(), C.c_uint32()
            ok = self.L.v3_token_bytes(self.handle, i, C.byref(p), C.byref(n)) == 0
            out.append(bytes(p[:n.value]) if ok and n.value else b"")
        return out


def rules_of(g) -> list:
    """The rule list of a RefGov or an engine GovRules: [(len, bytes)]."""
    return [bytes(g.rules[r][:g.rule_len[r]]) for r in range(g.n_rules)]
