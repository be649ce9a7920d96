"""The sampler oracle (oracle/sample_oracle.py) against the reference's own v3_sample_topk
(runtime/vault3.c:3204-3230), called from oracle/_ref/libvault3.so, which oracle/Makefile builds from the reference
sources.  Same logits, k, temperature and xorshift state: same token and same new state."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import sample_oracle as so

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libvault3.so")


def _ref():
    if not os.path.exists(LIB):
        pytest.skip("oracle/_ref/libvault3.so is not built (oracle/Makefile needs the reference sources)")
    L = C.CDLL(LIB)
    L.v3_sample_topk.restype = C.c_uint32
    L.v3_sample_topk.argtypes = [C.POINTER(C.c_float), C.c_uint32, C.c_uint32, C.c_float, C.POINTER(C.c_uint64)]
    return L


def sample_cases():
    """(logits, k, temp, rng) cases: random rows, rows with many equal values, signed zeros."""
    rng = np.random.default_rng(7)
    cases = []
    for n in (7, 64, 1000, 151936):
        for rep in range(3 if n > 1000 else 8):
            v = (rng.standard_normal(n) * 3).astype(np.float32)
            if rep % 3 == 1:
                v = np.round(v * 2) / 2          # many ties
            if rep % 3 == 2:
                v[rng.integers(0, n, size=min(n, 16))] = 0.0
                v[rng.integers(0, n, size=min(n, 16))] = -0.0
            for k, temp in ((1, 1.0), (2, 0.7), (5, 1.0), (40, 1.3), (64, 0.5), (100, 2.0), (8, 0.0)):
                state = int(rng.integers(0, 2 ** 63)) if rep % 2 else 0
                cases.append((v.astype(np.float32), k, temp, state))
    return cases


def test_sampler_oracle_matches_reference():
    L = _ref()
    for v, k, temp, state in sample_cases():
        st = C.c_uint64(state)
        tok = L.v3_sample_topk(v.ctypes.data_as(C.POINTER(C.c_float)), len(v), k, temp, C.byref(st))
        otok, ost = so.sample_topk(v, k, temp, state)
        assert (tok, st.value) == (otok, ost), (len(v), k, temp, state, tok, otok)


def test_expf_matches_reference_on_the_sampler_range():
    """The restated exponential against the reference's, through one-candidate-pair draws: p[1] = v3_expf(d) decides
    whether the second candidate is chosen, so the draw flips exactly where the two exponentials would differ."""
    L = _ref()
    for d in np.linspace(-30.0, 0.0, 61).astype(np.float32):
        v = np.array([0.0, d], dtype=np.float32)
        for state in (1, 12345, 2 ** 40 + 3):
            st = C.c_uint64(state)
            tok = L.v3_sample_topk(v.ctypes.data_as(C.POINTER(C.c_float)), 2, 2, 1.0, C.byref(st))
            assert (tok, st.value) == so.sample_topk(v, 2, 1.0, state)
