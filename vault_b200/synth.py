"""Seeded synthetic VAULT v3 models and the synthetic byte-level tokenizer used for them.

No real checkpoint or Qwen tokenizer exists in this environment, so every model this project runs is built here:
weights are drawn from a seeded numpy generator (matrices and biases N(0, std), norm gains 1 or U(lo, hi)) and
exported through `vlt3.write_vlt3`.  The tokenizer is a 256-token byte vocabulary in GPT-2 byte order (so byte
'\\n' is id 198, the id the reference hard-codes at src/vault_v3_model.py:1968,2239), a "system" token, and the
three ChatML control tokens as added tokens.
"""

from __future__ import annotations

import json
import os
from typing import Callable, Dict, Optional, Tuple

import numpy as np

from .config import VAULTv3Config
from .vlt3 import LAYER_KINDS, PreEncoded, byte_to_unicode, write_vlt3


def make_tokenizer_dir(path: str, vocab_size: int, extra_tokens: Optional[Dict[str, int]] = None) -> Dict[str, int]:
    """Write `tokenizer.json` for a byte-level vocabulary that fits in `vocab_size` ids.

    Full-size vocabularies (>= 151646) use the Qwen2 ids (system 8948, <|endoftext|>/<|im_start|>/<|im_end|> =
    151643/151644/151645); small test vocabularies put "system" at 300 and the three control tokens at the top
    three ids.  Returns the id map."""
    os.makedirs(path, exist_ok=True)
    b2u = byte_to_unicode()
    vocab = {b2u[b]: i for i, b in enumerate(b2u)}
    if vocab_size >= 151646:
        ids = dict(system=8948, endoftext=151643, im_start=151644, im_end=151645)
    else:
        if vocab_size < 320:
            raise ValueError("synthetic tokenizer needs vocab_size >= 320")
        ids = dict(system=300, endoftext=vocab_size - 3, im_start=vocab_size - 2, im_end=vocab_size - 1)
    vocab["system"] = ids["system"]
    for text, tid in (extra_tokens or {}).items():
        vocab["".join(b2u[b] for b in text.encode("utf-8"))] = tid
    tj = {
        "model": {"type": "BPE", "vocab": vocab, "merges": []},
        "added_tokens": [
            {"id": ids["endoftext"], "content": "<|endoftext|>", "special": True},
            {"id": ids["im_start"], "content": "<|im_start|>", "special": True},
            {"id": ids["im_end"], "content": "<|im_end|>", "special": True},
        ],
    }
    with open(os.path.join(path, "tokenizer.json"), "w", encoding="utf-8") as f:
        json.dump(tj, f, ensure_ascii=False)
    ids["newline"] = 198
    return ids


# Extra multi-byte tokens of the small test vocabularies: they exercise every segment-break tier rule
# (src/vault_v3_model.py:116-142): '",' is tier 2, '. ' is tier 1 (trailing whitespace ignored), ', ' tier 3.
SMALL_EXTRA_TOKENS = {'",': 256, ". ": 257, ", ": 258, "ab;": 259, "x}y": 260, "&q": 261, "line\n": 262}


def tensor_shapes(cfg: VAULTv3Config) -> Dict[str, Tuple[int, ...]]:
    d, H, G, D, F = cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.d_ff
    shapes: Dict[str, Tuple[int, ...]] = {"embed_tokens.weight": (cfg.vocab_size, d), "norm.weight": (d,)}
    per_layer = {
        "input_layernorm.weight": (d,),
        "self_attn.q_proj.weight": (H * D, d), "self_attn.q_proj.bias": (H * D,),
        "self_attn.k_proj.weight": (G * D, d), "self_attn.k_proj.bias": (G * D,),
        "self_attn.v_proj.weight": (G * D, d), "self_attn.v_proj.bias": (G * D,),
        "self_attn.o_proj.weight": (d, H * D),
        "post_attention_layernorm.weight": (d,),
        "mlp.gate_proj.weight": (F, d), "mlp.up_proj.weight": (F, d), "mlp.down_proj.weight": (d, F),
    }
    for li in range(cfg.n_layers):
        for k in LAYER_KINDS:
            shapes[f"layers.{li}.{k}"] = per_layer[k]
    if cfg.seg_layers:
        fd = len(cfg.seg_layers) * d
        shapes.update({
            "seg_scorer.ln.weight": (fd,), "seg_scorer.ln.bias": (fd,),
            "seg_scorer.fc1.weight": (cfg.seg_hidden, fd), "seg_scorer.fc1.bias": (cfg.seg_hidden,),
            "seg_scorer.fc2.weight": (1, cfg.seg_hidden), "seg_scorer.fc2.bias": (1,),
        })
    return shapes


def _is_gain(name: str) -> bool:
    return "layernorm" in name or name in ("norm.weight", "seg_scorer.ln.weight")


def lazy_state(cfg: VAULTv3Config, seed: int, std: float = 0.02,
               gain: Optional[Tuple[float, float]] = None, ln_bias_std: float = 0.0) -> Dict[str, Callable[[], np.ndarray]]:
    """Per-tensor generators: every tensor gets its own seeded stream (seed, tensor index), so any tensor can be
    regenerated alone and in any order.  Gains are 1 (or U(gain)), the scorer LayerNorm bias 0 (or N(0, ln_bias_std)),
    everything else N(0, std)."""
    shapes = tensor_shapes(cfg)
    out: Dict[str, Callable[[], np.ndarray]] = {}
    for idx, (name, shape) in enumerate(shapes.items()):
        def gen(name=name, shape=shape, idx=idx) -> np.ndarray:
            rng = np.random.default_rng([seed, idx])
            if _is_gain(name):
                if gain is None:
                    return np.ones(shape, dtype=np.float32)
                return rng.uniform(gain[0], gain[1], size=shape).astype(np.float32)
            if name == "seg_scorer.ln.bias":
                if ln_bias_std == 0.0:
                    return np.zeros(shape, dtype=np.float32)
                return (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(ln_bias_std))
            return rng.standard_normal(size=shape, dtype=np.float32) * np.float32(std)
        out[name] = gen
    return out


def build_state(cfg: VAULTv3Config, seed: int, **kw) -> Dict[str, np.ndarray]:
    return {k: g() for k, g in lazy_state(cfg, seed, **kw).items()}


def write_synthetic_vlt3(path: str, cfg: VAULTv3Config, fmt: str, seed: int, tokenizer_dir: Optional[str] = None,
                         model_name: str = "VAULT-v3-synthetic", **kw) -> Dict:
    """Export a seeded synthetic model to VLT3 (tensors are generated one at a time)."""
    if tokenizer_dir is None:
        tokenizer_dir = os.path.join(os.path.dirname(os.path.abspath(path)), "synthetic_tokenizer")
        make_tokenizer_dir(tokenizer_dir, cfg.vocab_size,
                           None if cfg.vocab_size >= 151646 else SMALL_EXTRA_TOKENS)
    return write_vlt3(path, lazy_state(cfg, seed, **kw), cfg, tokenizer_dir, fmt, model_name=model_name)


def _torch_encoder(name: str, shape, seed: int, idx: int, std: float, device: str):
    """PreEncoded tensor generated and quantized with torch on `device` (same block rules as quantize_q8_0 /
    quantize_q4_0 / RNE bf16; the random stream differs from the numpy generator, so files are seed-stable but not
    byte-identical to write_synthetic_vlt3)."""
    import torch

    def encode(dt: int) -> bytes:
        g = torch.Generator(device=device).manual_seed(seed * 1000003 + idx)
        if _is_gain(name):
            x = torch.ones(shape, device=device)
        elif name == "seg_scorer.ln.bias":
            x = torch.zeros(shape, device=device)
        else:
            x = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std
        return encode_torch(x, dt)

    return PreEncoded(shape, encode)


def encode_torch(x, dt: int) -> bytes:
    """Encode an fp32 torch tensor to VLT3 payload bytes (rules of tools/vlt3.py:102-149, 177-186)."""
    import torch
    from .vlt3 import BF16, F16, F32, Q4_0, Q8_0, QK

    if dt == F32:
        return x.float().contiguous().cpu().numpy().astype("<f4").tobytes()
    if dt == F16:
        return x.half().contiguous().cpu().numpy().astype("<f2").tobytes()
    if dt == BF16:
        return x.to(torch.bfloat16).contiguous().view(torch.int16).cpu().numpy().astype("<i2").tobytes()
    xb = x.reshape(-1, QK).float()
    nb = xb.shape[0]
    if dt == Q8_0:
        d = xb.abs().amax(dim=1) / 127.0
        inv = torch.where(d > 0, 1.0 / torch.where(d > 0, d, torch.ones_like(d)), torch.zeros_like(d))
        q = torch.clamp(torch.round(xb * inv[:, None]), -127, 127).to(torch.int8)
        out = torch.empty(nb, 34, dtype=torch.uint8, device=x.device)
        out[:, :2] = d.half().view(torch.uint8).view(nb, 2)
        out[:, 2:] = q.view(torch.uint8)
        return out.cpu().numpy().tobytes()
    if dt == Q4_0:
        ratios = [-1.0 / 8.0, -0.98 / 8.0, -0.96 / 8.0, -0.94 / 8.0, -0.92 / 8.0, -0.89 / 8.0, 1.0 / 7.5, 0.96 / 7.5]
        mx = xb.gather(1, xb.abs().argmax(dim=1, keepdim=True))[:, 0]
        best_err = torch.full((nb,), float("inf"), device=x.device)
        best_d = torch.zeros(nb, dtype=torch.float16, device=x.device)
        best_q = torch.full((nb, QK), 8, dtype=torch.uint8, device=x.device)
        nz = mx != 0
        for r in ratios:
            d16 = (mx * torch.tensor(r, dtype=torch.float32)).half()
            d32 = d16.float()
            inv = torch.where(d32 != 0, 1.0 / torch.where(d32 != 0, d32, torch.ones_like(d32)), torch.zeros_like(d32))
            qi = torch.clamp(torch.round(xb * inv[:, None] + 8.0), 0, 15).to(torch.uint8)
            err = ((qi.float() - 8.0) * d32[:, None] - xb).square().sum(dim=1)
            better = nz & (err < best_err)
            best_err = torch.where(better, err, best_err)
            best_d = torch.where(better, d16, best_d)
            best_q = torch.where(better[:, None], qi, best_q)
        out = torch.empty(nb, 18, dtype=torch.uint8, device=x.device)
        out[:, :2] = best_d.view(torch.uint8).view(nb, 2)
        out[:, 2:] = best_q[:, :QK // 2] | (best_q[:, QK // 2:] << 4)
        return out.cpu().numpy().tobytes()
    raise ValueError(dt)


def write_synthetic_vlt3_fast(path: str, cfg: VAULTv3Config, fmt: str, seed: int, device: str = "cuda",
                              std: float = 0.02, model_name: str = "VAULT-v3-synthetic") -> Dict:
    """Full-size synthetic export with tensors drawn and quantized by torch on `device` (seconds on a GPU).
    Weights N(0, std), norm gains 1, scorer LayerNorm bias 0 (the BASELINE synthetic models)."""
    tokenizer_dir = os.path.join(os.path.dirname(os.path.abspath(path)), "synthetic_tokenizer")
    make_tokenizer_dir(tokenizer_dir, cfg.vocab_size, None if cfg.vocab_size >= 151646 else SMALL_EXTRA_TOKENS)
    state = {name: _torch_encoder(name, shape, seed, idx, std, device)
             for idx, (name, shape) in enumerate(tensor_shapes(cfg).items())}
    return write_vlt3(path, state, cfg, tokenizer_dir, fmt, model_name=model_name)


def full_config(**overrides) -> VAULTv3Config:
    """The 1.54B VAULT v3 architecture: d=1536, 28 layers, 12/2 heads, head_dim 128, FFN 8960."""
    cfg = VAULTv3Config()
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


def full_model_file(fmt: str = "q8_0", seed: int = 0, directory: Optional[str] = None, **cfg_overrides) -> str:
    """Path of a cached full-size synthetic model (the BASELINE architecture, `fmt` weights, seed `seed`), written
    on first use with write_synthetic_vlt3_fast.  The directory is $VAULT_B200_BENCH_DIR (default: a folder in the
    system temp dir); a `.done` marker next to the file says the export finished.  Extra keyword arguments override
    config fields (for example n_sink=4, or the segment scorer fields) and become part of the file name."""
    import tempfile
    import time

    d = directory or os.environ.get("VAULT_B200_BENCH_DIR", os.path.join(tempfile.gettempdir(), "vault_b200_bench"))
    os.makedirs(d, exist_ok=True)
    tag = "".join(f"_{k}{'-'.join(map(str, v)) if isinstance(v, (tuple, list)) else v}"
                  for k, v in sorted(cfg_overrides.items()))
    path = os.path.join(d, f"vault_v3_1p5b_{fmt}_seed{seed}{tag}.vlt3")
    if not os.path.exists(path + ".done"):
        import torch
        cfg = full_config(**({"n_sink": 0} | cfg_overrides))
        t0 = time.time()
        write_synthetic_vlt3_fast(path, cfg, fmt, seed=seed, device="cuda" if torch.cuda.is_available() else "cpu")
        open(path + ".done", "w").close()
        print(f"[synth] wrote {path} ({os.path.getsize(path) / 1e9:.2f} GB) in {time.time() - t0:.1f}s",
              flush=True)
    return path
