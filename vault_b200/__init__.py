"""vault_b200: B200-native (sm_100a) decode/prefill engine for VAULT v3 models stored as VLT3 files.

The public API mirrors the reference's src/vault_v3_model.py streaming interface (`VAULTv3ForCausalLM.prefill`,
`.step`, `.new_state`, `.forward`) and tools/vlt3.py (`read_vlt3`, `write_vlt3`, ...); the compute path is the
CUDA library `libvault_b200.so` behind the C ABI in include/vault_b200.h.
"""

from .config import VAULTv3Config
from .tokenizer import Tokenizer
from .vlt3 import VLT3Error, read_vlt3, vlt3_config, write_vlt3


def __getattr__(name):
    # torch-dependent classes load lazily so the format tools work without CUDA
    if name in ("Governor", "VAULTv3ForCausalLM", "VAULTv3State", "sample_topk"):
        from . import model
        return getattr(model, name)
    raise AttributeError(name)


__all__ = ["Governor", "VAULTv3Config", "VAULTv3ForCausalLM", "VAULTv3State", "VLT3Error", "read_vlt3", "sample_topk",
           "Tokenizer", "vlt3_config", "write_vlt3"]
