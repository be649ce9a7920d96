"""CPU: pin the oracle and the VLT3 writer to the reference's own outputs (tests/golden/*, made by gen_golden.py)."""

import hashlib
import json
import os

import numpy as np
import pytest

from oracle import vault_oracle as vo
from tests.golden.cases import CASES, case_config, case_ids
from vault_b200 import vlt3

# the oracle restates the reference in fp32; the reference's own C runtime agrees with it to ~1e-5
ORACLE_ATOL = 1e-4


def _manifest(golden_dir):
    with open(os.path.join(golden_dir, "manifest.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("name", sorted(CASES))
def test_writer_byte_identical_to_reference(name, case_files, golden_dir):
    with open(case_files(name), "rb") as f:
        sha = hashlib.sha256(f.read()).hexdigest()
    assert sha == _manifest(golden_dir)[name]["sha256"]


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_logits(name, case_files, golden_dir):
    spec = CASES[name]
    cfg = case_config(spec)
    g = np.load(os.path.join(golden_dir, f"{name}.npz"))
    m = vo.OracleModel.from_file(case_files(name), max_sink=cfg.max_sink)
    ids = case_ids(spec, cfg)
    assert np.array_equal(ids, g["ids"])
    B = ids.shape[0]
    for b in range(B):
        lg, st = vo.run(m, ids[b], seg_budget=None if B == 1 else 0, auto_pin=(B == 1))
        ref = g["step_logits"][b]
        assert np.abs(lg - ref).max() < ORACLE_ATOL
        assert (lg.argmax(-1) == ref.argmax(-1)).all()
        if B == 1:
            assert st.n_pin == int(g["final_n_pin"])
            assert st.mem_pos.tolist() == g["final_mem_pos"].tolist()
            assert np.abs(st.mem_score - g["final_mem_score"]).max() < 1e-4
            assert np.abs(st.sc_prev - g["final_sc_prev"]).max() < 1e-4


def test_golden_cases_exercise_the_mechanisms(golden_dir):
    man = _manifest(golden_dir)
    assert man["chat_pin_q8_0"]["final_n_pin"] > 4            # ChatML auto-pin fired
    assert man["tiny_seg_q8_0"]["final_mem_cnt"] == 12        # segment bank full
    assert man["mini_gqa_q8_0"]["final_mem_cnt"] == 24
    # reference self-consistency: forward(mode="block") == step loop
    for name, e in man.items():
        assert e["forward_vs_step_max_abs"] < 1e-4, name


def test_spoof_case_quarantines(case_files):
    spec = CASES["chat_spoof_q8_0"]
    cfg = case_config(spec)
    m = vo.OracleModel.from_file(case_files("chat_spoof_q8_0"), max_sink=cfg.max_sink)
    st = vo.OracleState(m)
    hits = []
    for i, t in enumerate(case_ids(spec, cfg)[0]):
        vo.step(m, st, int(t))
        if st.sc_cur[i % m.W] < -1e29:
            hits.append(i)
    assert hits, "spoof literal never quarantined"


def test_block_codecs_bit_exact(golden_dir):
    g = np.load(os.path.join(golden_dir, "codec.npz"))
    w = g["w"]
    assert np.frombuffer(vlt3.quantize_q8_0(w), np.uint8).tobytes() == g["q8"].tobytes()
    assert np.frombuffer(vlt3.quantize_q4_0(w), np.uint8).tobytes() == g["q4"].tobytes()
    for deq, key, dt in ((vlt3.dequantize_q8_0, "q8", vo._Q8), (vlt3.dequantize_q4_0, "q4", vo._Q4)):
        ref = g[f"{key}_deq"]
        mine = deq(g[key].tobytes(), w.size)
        orc = vo.dequant(g[key].tobytes(), dt, w.size)
        assert mine.view(np.uint32).tobytes() == ref.view(np.uint32).tobytes()
        assert orc.view(np.uint32).tobytes() == ref.view(np.uint32).tobytes()


def test_hybrid_policy_keeps_boundary_layers_q8(case_files):
    """Hybrid Q4_0 on an 8-layer model: q/o of layers 0, 1, L-2, L-1 and every k/v stay Q8_0, the rest Q4_0
    (tools/vlt3.py:312-330); the file is byte-identical to the reference writer's (manifest sha256)."""
    vf = vlt3.read_vlt3(case_files("deep_hybrid_q4_0"))
    L = vf.header["n_layers"]
    assert L == 8
    for li in range(L):
        for kind, want in (("q_proj", vlt3.Q8_0 if li in (0, 1, L - 2, L - 1) else vlt3.Q4_0),
                           ("o_proj", vlt3.Q8_0 if li in (0, 1, L - 2, L - 1) else vlt3.Q4_0),
                           ("k_proj", vlt3.Q8_0), ("v_proj", vlt3.Q8_0)):
            assert vf.entry(f"layers.{li}.self_attn.{kind}.weight")["dtype"] == want, (li, kind)
        assert vf.entry(f"layers.{li}.mlp.down_proj.weight")["dtype"] == vlt3.Q4_0
