"""Generate tests/golden/tokenizer.npz: the ids the REFERENCE tokenizer (v3_encode_ex, runtime/vault3.c:2708-2809,
called from oracle/_ref/libvault3.so, which oracle/Makefile builds from the reference sources) gives for the seeded
texts of tests/golden/tok_fixture.py on the fixture file it builds.  Run in the build container, where the reference
build exists:  python tests/golden/gen_tokenizer_golden.py"""
import ctypes as C
import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden.tok_fixture import build_tokenizer_file, golden_texts  # noqa: E402
from tests.ref_governor import RefModel, ref_lib  # noqa: E402


def main() -> None:
    L = ref_lib()
    L.ref_sizeof_tokenizer.restype = C.c_size_t
    L.v3_tok_arena_size.argtypes = [C.c_void_p]
    L.v3_tok_arena_size.restype = C.c_size_t
    L.v3_tok_init.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]
    L.v3_encode_ex.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t),
                               C.c_int]
    with tempfile.TemporaryDirectory() as td:
        path = build_tokenizer_file(td)
        sha = hashlib.sha256(open(path, "rb").read()).hexdigest()
        model = RefModel(L, path)
        n = L.v3_tok_arena_size(model.handle)
        raw = np.zeros(n + 64, np.uint8)
        arena = raw[(-raw.ctypes.data) % 64:]
        tok = C.create_string_buffer(L.ref_sizeof_tokenizer())
        assert L.v3_tok_init(tok, model.handle, arena.ctypes.data, n) == 0
        ids, off, special = [], [0], []
        for text, s in golden_texts():
            out = np.zeros(len(text) + 8, np.uint32)
            got = C.c_size_t()
            assert L.v3_encode_ex(tok, text, len(text), out.ctypes.data, out.size, C.byref(got), s) == 0
            ids += out[:got.value].tolist()
            off.append(len(ids))
            special.append(s)
    np.savez_compressed(os.path.join(HERE, "tokenizer.npz"), ids=np.array(ids, np.uint32),
                        id_off=np.array(off, np.int64), special=np.array(special, np.int8), file_sha256=sha)
    print(f"tokenizer.npz: {len(special)} encodings, {len(ids)} ids, fixture sha256 {sha[:16]}")


if __name__ == "__main__":
    main()
