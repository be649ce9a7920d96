"""ctypes binding of libvault_b200.so (the C ABI declared in include/vault_b200.h).

The engine has no CPU fallback: importing the binding fails loudly when the library is missing.
"""

from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvault_b200.so")

V3G_OK = 0
V3G_STATE_PER_SEQ_MEMORY, V3G_STATE_NO_AUTOPIN, V3G_STATE_NO_GRAPHS, V3G_STATE_NO_PERSISTENT = 1, 2, 4, 8
V3G_STATE_TOKEN_PREFILL = 16
V3G_STATE_FP16_ACTIVATIONS = 32
V3G_STATUS_RESONANCE, V3G_STATUS_BOUNDS, V3G_STATUS_TIMEOUT = 1, 2, 4
# codes -1..-12 are the file-validation codes of runtime/vault3.h:35-49
FILE_ERRORS = set(range(-12, 0)) - {-8}


class ModelInfo(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("vocab_size", "d_model", "n_layers", "n_heads", "n_kv_heads", "head_dim",
                                           "d_ff", "window")] + \
               [("rms_eps", C.c_float), ("rope_theta", C.c_float)] + \
               [(n, C.c_uint32) for n in ("bos_id", "eos_id", "im_start_id", "im_end_id", "pad_id", "weight_format",
                                           "flags", "n_sink", "seg_budget", "seg_hidden", "seg_min", "seg_max",
                                           "seg_n_feat")] + \
               [("seg_layers", C.c_uint32 * 4), ("sink_cap", C.c_uint32)] + \
               [(n, C.c_uint64) for n in ("step_weight_bytes", "lm_head_bytes", "scorer_bytes", "device_bytes")]


class SeqInfo(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("n_pin", "pin_locked", "mem_cnt", "n_uniq_segs", "seg_id_offset",
                                          "ema_ready", "seg_budget")] + [("pos", C.c_uint64)]


class GovRules(C.Structure):
    """v3g_gov_rules_t: the governor's canonical patterns (the rule part of runtime/vault3.h:198-209 v3_governor)."""
    _fields_ = [("n_rules", C.c_uint32), ("rule_len", C.c_uint32 * 8), ("rules", (C.c_uint8 * 32) * 8)]


GOV_STREAM_BYTES = 192   # sizeof(v3g_gov_stream_t)

_P = C.c_void_p
_SIGS = {
    "v3g_load": (C.c_int, [C.POINTER(_P), _P, C.c_uint64, C.c_int, C.c_int, C.c_uint32]),
    "v3g_validate": (C.c_int, [_P, C.c_uint64, C.c_int]),
    "v3g_load_file": (C.c_int, [C.POINTER(_P), C.c_char_p, C.c_int, C.c_int, C.c_uint32]),
    "v3g_validate_file": (C.c_int, [C.c_char_p, C.c_int]),
    "v3g_model_get_info": (C.c_int, [_P, C.POINTER(ModelInfo)]),
    "v3g_free": (None, [_P]),
    "v3g_state_arena_size": (C.c_size_t, [_P, C.c_uint32, C.c_uint32]),
    "v3g_state_init": (C.c_int, [C.POINTER(_P), _P, _P, C.c_size_t, C.c_uint32, C.c_uint32, C.c_uint32]),
    "v3g_state_free": (None, [_P]),
    "v3g_state_reset": (C.c_int, [_P, _P]),
    "v3g_set_pinned": (C.c_int, [_P, C.c_uint32, _P]),
    "v3g_set_seg_budget": (C.c_int, [_P, C.c_uint32, _P]),
    "v3g_state_pos": (C.c_uint64, [_P]),
    "v3g_step": (C.c_int, [_P, _P, _P, _P, _P]),
    "v3g_step_host": (C.c_int, [_P, _P, _P, _P, _P]),
    "v3g_prefill": (C.c_int, [_P, _P, C.c_uint32, C.c_uint64, _P, _P, _P]),
    "v3g_generate": (C.c_int, [_P, _P, C.c_uint32, _P, C.c_uint64, _P]),
    "v3g_status": (C.c_int, [_P, C.POINTER(C.c_uint32), C.c_int, _P]),
    "v3g_seq_info": (C.c_int, [_P, C.c_uint32, C.POINTER(SeqInfo), _P, _P, C.c_uint32, _P]),
    "v3g_dequant": (C.c_int, [_P, C.c_uint32, _P, _P]),
    "v3g_gemv": (C.c_int, [_P, C.c_uint32, _P, C.c_uint32, _P, _P]),
    "v3g_decode_pass": (C.c_int, [_P, C.c_int, _P]),
    "v3g_attention": (C.c_int, [_P, C.c_uint32, _P]),
    "v3g_status_copy": (C.c_int, [_P, _P, _P]),
    "v3g_sample_topk": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.c_uint64, C.c_uint32, C.c_float, _P, _P, _P]),
    "v3g_generate_sampled": (C.c_int, [_P, _P, C.c_uint32, _P, C.c_uint64, C.c_uint32, C.c_float, _P,
                                       C.POINTER(GovRules), _P, _P]),
    "v3g_gov_init": (None, [C.POINTER(GovRules)]),
    "v3g_tokenizer_create": (C.c_int, [C.POINTER(_P), _P, C.c_uint64]),
    "v3g_tokenizer_free": (None, [_P]),
    "v3g_encode_ex": (C.c_int, [_P, C.c_char_p, C.c_size_t, _P, C.c_size_t, C.POINTER(C.c_size_t), C.c_int]),
    "v3g_encode": (C.c_int, [_P, C.c_char_p, C.c_size_t, _P, C.c_size_t, C.POINTER(C.c_size_t)]),
    "v3g_token_bytes": (C.c_int, [_P, C.c_uint32, C.POINTER(C.POINTER(C.c_uint8)), C.POINTER(C.c_uint32)]),
    "v3g_gov_add_rule": (C.c_int, [C.POINTER(GovRules), C.c_char_p, C.c_size_t]),
    "v3g_gov_arm_system": (None, [C.POINTER(GovRules), C.c_char_p, C.c_size_t]),
    "v3g_govern_logits": (C.c_int, [_P, C.POINTER(GovRules), _P, _P, C.c_uint32, C.c_uint64, C.c_uint32, _P]),
    "v3g_gov_commit": (C.c_int, [_P, C.POINTER(GovRules), _P, _P, C.c_uint32, _P]),
    "v3g_gemm_work_size": (C.c_size_t, [_P, C.c_uint32, C.c_uint32]),
    "v3g_gemm": (C.c_int, [_P, C.c_uint32, _P, C.c_uint32, _P, _P, C.c_size_t, _P]),
    "v3g_argmax_noalloc": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.c_uint64, _P, _P]),
    "v3g_error_string": (C.c_char_p, [C.c_int]),
    "v3g_last_error": (C.c_char_p, []),
}

_lib = None


def lib() -> C.CDLL:
    """Load the engine library (once).  Raises when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m vault_b200.build` "
                               "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS)


def last_error() -> str:
    return lib().v3g_last_error().decode("utf-8", "replace")


class EngineError(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what} failed: {lib().v3g_error_string(code).decode()} ({code}): {last_error()}")


def check(code: int, what: str) -> None:
    if code != V3G_OK:
        if code in FILE_ERRORS:
            from .vlt3 import VLT3Error
            raise VLT3Error(f"{what}: {lib().v3g_error_string(code).decode()} ({code}): {last_error()}")
        raise EngineError(code, what)
