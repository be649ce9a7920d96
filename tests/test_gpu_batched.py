"""GPU: batched decode above 8 sequences, where every projection runs on the tensor-core GEMM (one weight stream per
step for the whole batch).

- Per-sequence segment memory (V3G_STATE_PER_SEQ_MEMORY, BASELINE config 3's mode): the reference runs segment
  memory only at batch 1 (src/vault_v3_model.py:1944,2222), so each sequence of the batch is checked against an
  independent batch-1 oracle run of its own stream -- logits within the bar, identical bank positions, same n_pin.
- The reference's batched sliding-window step (no segment memory, n_sink sinks): the tensor-core step against the
  GEMV step of the same engine, and against per-sequence oracle runs.
"""

import numpy as np
import pytest
import torch

from oracle import vault_oracle as vo
from tests.golden.cases import CASES, IM_END, IM_START, SYSTEM, case_config, byte_ids

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _streams(cfg, B, L, seed):
    """B seeded streams: ChatML system prefixes of varied length (auto-pin), then random bodies."""
    rng = np.random.default_rng(seed)
    rows = []
    for b in range(B):
        sys_len = int(rng.integers(2, 12))
        ids = [IM_START, SYSTEM] + rng.integers(0, 256, size=sys_len).tolist() + [IM_END, byte_ids("\n")[0]]
        if b % 3 == 2:
            ids = []   # no system prompt: nothing pinned
        ids += rng.integers(0, cfg.vocab_size - 3, size=L - len(ids)).tolist()
        rows.append(ids[:L])
    return np.asarray(rows, dtype=np.int64)


@pytest.mark.parametrize("name,B", [("tiny_seg_q8_0", 12), ("mini_gqa_q8_0", 10), ("mini_gqa_q4_0", 16)])
def test_per_sequence_memory_matches_batch1_oracle(name, B, case_files):
    from vault_b200.model import VAULTv3ForCausalLM
    spec = CASES[name]
    cfg = case_config(spec)
    m = VAULTv3ForCausalLM(case_files(name), device=0, max_sink=cfg.max_sink)
    L = 4 * cfg.window + 7
    ids = _streams(cfg, B, L, seed=B)
    st = m.new_state(B, per_sequence_memory=True)
    out = np.stack([m.step(torch.from_numpy(ids[:, t]), st).cpu().numpy() for t in range(L)], axis=1)
    st.check()
    om = vo.OracleModel.from_file(case_files(name), max_sink=cfg.max_sink)
    for b in range(B):
        ref, ost = vo.run(om, ids[b])
        err = float(np.abs(out[b] - ref).max())
        assert err <= TOL, (b, err)
        si, mem_pos, _ = st.info(b, with_bank=True)
        assert si.n_pin == ost.n_pin, b
        assert mem_pos.tolist() == ost.mem_pos.tolist(), b


@pytest.mark.parametrize("name", ["mini_gqa_q8_0", "mini_gqa_bf16", "deep_hybrid_q4_0"])
def test_batched_window_step_tensor_core_vs_gemv(name, case_files):
    from vault_b200.model import VAULTv3ForCausalLM
    spec = CASES[name]
    cfg = case_config(spec)
    m = VAULTv3ForCausalLM(case_files(name), device=0, max_sink=cfg.max_sink)
    B, L = 12, 3 * cfg.window + 5
    ids = torch.from_numpy(np.random.default_rng(3).integers(0, cfg.vocab_size - 3, size=(B, L)))
    outs = []
    for persistent in (True, False):   # B > 8: tensor-core step, or GEMV passes with persistent=False
        st = m.new_state(B, persistent=persistent)
        outs.append(np.stack([m.step(ids[:, t], st).cpu().numpy() for t in range(L)], axis=1))
        st.check()
    assert np.abs(outs[0] - outs[1]).max() <= TOL
    om = vo.OracleModel.from_file(case_files(name), max_sink=cfg.max_sink)
    for b in (0, B - 1):
        ref, _ = vo.run(om, ids[b].numpy(), seg_budget=0, auto_pin=False, n_pin=min(cfg.n_sink, cfg.window))
        assert np.abs(outs[0][b] - ref).max() <= TOL, b
