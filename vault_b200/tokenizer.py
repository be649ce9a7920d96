"""Host tokenizer of a VLT3 file's VTOK blob through the engine library (v3g_encode_ex): the counterpart of the
reference's v3_tok_init / v3_encode / v3_encode_ex / v3_token_bytes (runtime/vault3.h:182-189).  No GPU needed."""
from __future__ import annotations

import ctypes as C
from typing import Iterable, List, Union

import numpy as np

from . import _lib
from .vlt3 import _unpack_header, aligned_buffer


class Tokenizer:
    """Byte-level BPE with the Qwen2 pre-tokenizer and NFC, as the reference's C runtime encodes prompts."""

    def __init__(self, vlt3: Union[str, bytes]):
        buf = aligned_buffer(vlt3)
        h = C.c_void_p()
        _lib.check(_lib.lib().v3g_tokenizer_create(C.byref(h), C.c_void_p(buf.ctypes.data), buf.size),
                   "v3g_tokenizer_create")
        self._h = h
        hdr = _unpack_header(buf)
        self.bos_id, self.eos_id = hdr["bos_id"], hdr["eos_id"]
        self.im_start_id, self.im_end_id = hdr["im_start_id"], hdr["im_end_id"]

    def encode(self, text: Union[str, bytes], allow_special: bool = True) -> List[int]:
        """Token ids of text (UTF-8 when str); with allow_special=False, <|im_start|> and the like are plain text."""
        data = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        out = np.zeros(len(data) + 1, np.uint32)   # every id consumes at least one byte
        n = C.c_size_t()
        _lib.check(_lib.lib().v3g_encode_ex(self._h, data, len(data), C.c_void_p(out.ctypes.data), out.size,
                                            C.byref(n), int(allow_special)), "v3g_encode_ex")
        return out[:n.value].tolist()

    def chat_ids(self, system: Union[str, bytes], user: Union[str, bytes]) -> List[int]:
        """The ChatML prompt of the reference's chat mode (runtime/vault3_host.c:552-570): system and user text are
        encoded with special tokens off, so text that spells <|im_start|> or <|im_end|> cannot open or close a
        turn; the control tokens come from the file header's ids."""
        ids = [self.im_start_id] + self.encode(b"system\n", False) + self.encode(system, False)
        ids += [self.im_end_id] + self.encode(b"\n", False)
        ids += [self.im_start_id] + self.encode(b"user\n", False) + self.encode(user, False)
        ids += [self.im_end_id] + self.encode(b"\n", False)
        return ids + [self.im_start_id] + self.encode(b"assistant\n", False)

    def token_bytes(self, token_id: int) -> bytes:
        p, n = C.POINTER(C.c_uint8)(), C.c_uint32()
        if _lib.lib().v3g_token_bytes(self._h, int(token_id), C.byref(p), C.byref(n)) != _lib.V3G_OK:
            raise ValueError(f"token id {token_id} is outside the tokenizer's vocabulary")
        return bytes(p[:n.value])

    def decode(self, ids: Iterable[int]) -> bytes:
        """The raw bytes of the tokens, concatenated (not necessarily valid UTF-8 mid-stream)."""
        return b"".join(self.token_bytes(i) for i in ids)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            _lib.lib().v3g_tokenizer_free(h)
            self._h = None
