"""GPU parity at key spans of 1 to 6 attention splits (64 keys each), against the oracle.

The golden cases keep every span under 128 keys.  Here a window of 192 makes the span grow to 384 keys, so
the decode kernels go through all three ways of finishing attention: a single split written directly, 2-4
splits merged by the next phase's activation prologue (persistent kernel), and more splits merged by the last
CTA of the group (both paths).  Tolerances are the golden tests' own.
"""
import os
import tempfile

import numpy as np
import pytest
import torch

from oracle import vault_oracle as vo
from tests.golden.cases import IM_END, IM_START, SYSTEM, V
from vault_b200 import synth
from vault_b200.model import VAULTv3Config

pytestmark = pytest.mark.gpu

_CFG = dict(vocab_size=V, d_model=1536, n_layers=2, n_heads=12, n_kv_heads=2, head_dim=128, d_ff=512, window=192,
            n_sink=4, max_sink=64, seg_budget=24, seg_hidden=64, seg_min=4, seg_max=10, seg_layers=(0, 1),
            im_start_id=IM_START, im_end_id=IM_END, system_tok_id=SYSTEM)
_L = 420


@pytest.fixture(scope="module")
def long_case():
    cfg = VAULTv3Config(**_CFG)
    td = tempfile.mkdtemp(prefix="v3g_long_")
    tok = os.path.join(td, "tok")
    synth.make_tokenizer_dir(tok, cfg.vocab_size, synth.SMALL_EXTRA_TOKENS)
    path = os.path.join(td, "long_q8_0.vlt3")
    synth.write_synthetic_vlt3(path, cfg, "q8_0", 11, tokenizer_dir=tok, model_name="long_q8_0", std=0.02)
    ids = np.random.default_rng(1011).integers(0, V - 3, size=_L).astype(np.int64)
    om = vo.OracleModel.from_file(path, max_sink=cfg.max_sink)
    ref, _ = vo.run(om, ids.tolist())
    return cfg, path, ids, ref


@pytest.mark.parametrize("persistent", [True, False], ids=["persistent", "per_phase"])
def test_long_spans_match_oracle(long_case, persistent):
    from vault_b200.model import VAULTv3ForCausalLM
    cfg, path, ids, ref = long_case
    m = VAULTv3ForCausalLM(path, device=0, max_sink=cfg.max_sink)
    st = m.new_state(1, persistent=persistent)
    t = torch.from_numpy(ids)[None]
    out = np.stack([m.step(t[:, i], st).cpu().numpy()[0] for i in range(_L)])
    st.check()
    tol = 2e-2 * max(1.0, float(np.abs(ref).max()) / 4.0)
    err = np.abs(out - ref).max(axis=1)
    assert err.max() <= tol, (int(err.argmax()), float(err.max()), tol)
    assert (out.argmax(-1) == ref.argmax(-1)).mean() >= 0.99
