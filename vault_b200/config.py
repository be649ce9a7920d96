"""Model hyper-parameters of a VAULT v3 network (same fields and defaults as src/vault_v3_model.py:37-104)."""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Tuple


@dataclass
class VAULTv3Config:
    vocab_size: int = 151936
    d_model: int = 1536
    n_layers: int = 28
    n_heads: int = 12
    n_kv_heads: int = 2
    head_dim: int = 128
    d_ff: int = 8960
    rms_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    tie_embeddings: bool = True
    window: int = 1024           # chunk size W; a query sees the previous chunk and its own chunk causally
    n_sink: int = 4              # base attention-sink tokens
    max_sink: int = 512          # cap of the auto-pinned ChatML system prefix
    auto_pin_system: bool = True
    im_start_id: int = 151644
    im_end_id: int = 151645
    system_tok_id: int = 8948
    seg_budget: int = 0          # segment-memory bank slots (0 = sliding window + sinks only)
    seg_hidden: int = 256
    seg_min: int = 16
    seg_max: int = 48
    seg_layers: Tuple[int, ...] = ()

    @property
    def n_cells(self) -> int:
        """Kenyon memory cells: none in v3 (src/vault_v3_model.py:63-65)."""
        return 0

    @property
    def group_size(self) -> int:
        return self.n_heads // self.n_kv_heads

    @property
    def has_seg_scorer(self) -> bool:
        return len(self.seg_layers) > 0 and self.seg_budget > 0

    @property
    def sink_cap(self) -> int:
        """Rows reserved for sink keys per layer (src/vault_v3_model.py:965)."""
        return max(1, self.n_sink, self.max_sink if self.auto_pin_system else self.n_sink)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["seg_layers"] = list(self.seg_layers)
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "VAULTv3Config":
        d = {k: v for k, v in dict(d).items() if k in cls.__dataclass_fields__}
        if "seg_layers" in d:
            d["seg_layers"] = tuple(int(x) for x in d["seg_layers"])
        return cls(**d)

    @classmethod
    def from_qwen_config(cls, qc: dict, **overrides) -> "VAULTv3Config":
        """Backbone sizes from a Hugging Face Qwen2 config.json dict, then keyword overrides
        (src/vault_v3_model.py:87-103)."""
        cfg = cls(vocab_size=qc["vocab_size"], d_model=qc["hidden_size"], n_layers=qc["num_hidden_layers"],
                  n_heads=qc["num_attention_heads"], n_kv_heads=qc["num_key_value_heads"],
                  head_dim=qc["hidden_size"] // qc["num_attention_heads"], d_ff=qc["intermediate_size"],
                  rms_eps=qc["rms_norm_eps"], rope_theta=qc["rope_theta"],
                  tie_embeddings=qc.get("tie_word_embeddings", True))
        for k, v in overrides.items():
            setattr(cfg, k, v)
        return cfg
