import os
import sys
import tempfile

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(REPO, "tests", "golden")


@pytest.fixture(scope="session")
def case_files():
    """Build every golden case's VLT3 file once per session (seeded, regenerated from tests/golden/cases.py)."""
    from tests.golden.cases import CASES, case_config
    from vault_b200 import synth

    td = tempfile.mkdtemp(prefix="v3g_cases_")
    cache = {}

    def get(name: str) -> str:
        if name not in cache:
            spec = CASES[name]
            cfg = case_config(spec)
            tok = os.path.join(td, f"tok_{cfg.vocab_size}")
            if not os.path.exists(os.path.join(tok, "tokenizer.json")):
                synth.make_tokenizer_dir(tok, cfg.vocab_size, synth.SMALL_EXTRA_TOKENS)
            path = os.path.join(td, f"{name}.vlt3")
            synth.write_synthetic_vlt3(path, cfg, spec["fmt"], spec["seed"], tokenizer_dir=tok, model_name=name,
                                       std=spec["std"], gain=spec.get("gain"), ln_bias_std=spec.get("ln_bias_std", 0.0))
            cache[name] = path
        return cache[name]

    return get
