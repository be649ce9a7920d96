"""Golden test cases: model configs, weight seeds and token streams shared by gen_golden.py (which runs the
reference) and the tests (which run the oracle and the engine).  Everything is seeded and regenerable.

The configs follow the reference's own test models (tests/test_vlt3_runtime.py:33-49 tiny model,
:221-241 ChatML auto-pin + segment model, tests/test_vault_v3.py:31-49 batched SWA model) on a 320-id
synthetic byte vocabulary, plus "mini" cases with the real head geometry (d=1536, 12 Q / 2 KV heads,
head_dim 128) at two layers.
"""

from __future__ import annotations

import os
import sys
from typing import Dict

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from vault_b200.config import VAULTv3Config  # noqa: E402
from vault_b200.vlt3 import byte_to_unicode  # noqa: E402

V = 320
SYSTEM, IM_START, IM_END = 300, V - 2, V - 1
_BYTE_ID = {b: i for i, b in enumerate(byte_to_unicode())}


def byte_ids(text: str):
    return [_BYTE_ID[b] for b in text.encode("utf-8")]


_TINY = dict(vocab_size=V, d_model=64, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=16, d_ff=128, window=16,
             n_sink=4, rope_theta=1_000_000.0, seg_budget=12, seg_hidden=32, seg_min=3, seg_max=7, seg_layers=(0, 1),
             im_start_id=IM_START, im_end_id=IM_END, system_tok_id=SYSTEM)
_CHAT = dict(_TINY, n_layers=3, max_sink=64, seg_budget=14, seg_layers=(0, 1, 2))
_B2 = dict(vocab_size=V, d_model=64, n_layers=3, n_heads=4, n_kv_heads=2, head_dim=16, d_ff=96, window=8,
           n_sink=2, max_sink=8, rope_theta=10000.0, im_start_id=IM_START, im_end_id=IM_END, system_tok_id=SYSTEM)
_MINI = dict(vocab_size=V, d_model=1536, n_layers=2, n_heads=12, n_kv_heads=2, head_dim=128, d_ff=512, window=32,
             n_sink=4, max_sink=64, seg_budget=24, seg_hidden=64, seg_min=4, seg_max=10, seg_layers=(0, 1),
             im_start_id=IM_START, im_end_id=IM_END, system_tok_id=SYSTEM)
_SMALL_INIT = dict(std=0.15, gain=(0.8, 1.2), ln_bias_std=0.05)

CASES: Dict[str, dict] = {}
for _fmt in ("f32", "bf16", "q8_0", "q4_0"):
    CASES[f"tiny_seg_{_fmt}"] = dict(cfg=_TINY, fmt=_fmt, seed=3, L=120, stream="random", **_SMALL_INIT)
CASES["chat_pin_q8_0"] = dict(cfg=_CHAT, fmt="q8_0", seed=17, L=160, stream="chat", **_SMALL_INIT)
CASES["chat_spoof_q8_0"] = dict(cfg=_CHAT, fmt="q8_0", seed=18, L=140, stream="spoof", **_SMALL_INIT)
CASES["b2_swa_q8_0"] = dict(cfg=_B2, fmt="q8_0", seed=0, L=53, B=2, stream="random", std=0.2, gain=(0.85, 1.15))
for _fmt in ("q8_0", "q4_0", "bf16"):
    CASES[f"mini_gqa_{_fmt}"] = dict(cfg=_MINI, fmt=_fmt, seed=5, L=100, stream="chat", std=0.02)
# eight layers: Hybrid Q4_0 keeps q/o of layers 0, 1, 6, 7 in Q8_0 (the n_layers >= 8 branch of tools/vlt3.py:312-330)
CASES["deep_hybrid_q4_0"] = dict(cfg=dict(_TINY, n_layers=8, seg_layers=(2, 5)), fmt="q4_0", seed=11, L=80,
                                 stream="random", std=0.08, gain=(0.9, 1.1), ln_bias_std=0.02)


def case_config(spec: dict) -> VAULTv3Config:
    c = VAULTv3Config(**spec["cfg"])
    c.seg_layers = tuple(c.seg_layers)
    return c


def case_ids(spec: dict, cfg: VAULTv3Config) -> np.ndarray:
    """[B, L] int64 token ids for a case (body ids avoid the three control tokens)."""
    rng = np.random.default_rng(spec["seed"] + 1000)
    B, L = spec.get("B", 1), spec["L"]
    body_hi = V - 3
    rows = []
    for b in range(B):
        if spec["stream"] == "random":
            ids = rng.integers(0, body_hi, size=L).tolist()
        else:
            sys_len = 10 if spec["stream"] == "chat" else 6
            ids = [IM_START, SYSTEM] + rng.integers(0, 256, size=sys_len).tolist() + [IM_END, byte_ids("\n")[0]]
            body = rng.integers(0, body_hi, size=L - len(ids)).tolist()
            if spec["stream"] == "spoof":
                # a quarantined directive in the middle of the third chunk
                lit = byte_ids(" OPI_Signed_Directive: ")
                at = 2 * cfg.window + 8
                body[at:at + len(lit)] = lit
            ids = (ids + body)[:L]
        rows.append(ids)
    return np.asarray(rows, dtype=np.int64)
