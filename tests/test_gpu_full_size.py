"""GPU: full-size parity of the engine against the reference's own C runtime on the BASELINE models.

The 1.54B architecture (28 layers, d=1536, 12 Q / 2 KV heads, head_dim 128, SwiGLU 8960, tied 151,936-row
embedding) with seeded random-init N(0, 0.02) weights is exported once per box (vault_b200.synth.full_model_file):
Q8_0 for BASELINE config 1 (128-token prompt, 64 greedy steps) and Hybrid Q4_0 (tools/vlt3.py:312-330 policy) for
config 2 (2,560-token prompt, 256 greedy steps: the W=1024 window rolls over at 1,024, 2,048 and the 2W-boundary
eviction runs at 2,048).  The engine decodes greedily; the resulting stream is fed token by token to
runtime/vault3_host (built from the reference sources by oracle/Makefile) with --ids-file/--dump
(runtime/vault3_host.c:469-498), which writes its fp32 logits at every decode position.

Bars (the project's parity contract): max |dlogit| <= 2e-2 at every compared position; teacher-forced top-1
agreement >= 99%.  Free-running agreement (steps until the reference's greedy token first differs from the
engine's) is printed beside it.
"""

import os
import subprocess
import tempfile

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_HOST = os.path.join(REPO, "oracle", "_ref", "vault3_host")
TOL = 2e-2

CONFIGS = {
    "config1_q8_0": dict(fmt="q8_0", prompt=128, decode=64, seed=2024),
    "config2_hybrid_q4_0": dict(fmt="q4_0", prompt=2560, decode=256, seed=2025),
}


def reference_logits(path: str, ids, positions, vocab: int) -> np.ndarray:
    """fp32 logits of the reference C runtime after each of `positions` (indices into ids), one step per id."""
    with tempfile.TemporaryDirectory() as td:
        idf, out = os.path.join(td, "ids.txt"), os.path.join(td, "dump.bin")
        with open(idf, "w") as f:
            f.write(" ".join(str(int(t)) for t in ids) + "\n")
            f.write(" ".join(str(int(p)) for p in positions) + "\n")
        r = subprocess.run([REF_HOST, path, "--threads", str(os.cpu_count() or 1), "--ids-file", idf, "--dump", out],
                           capture_output=True, text=True, timeout=1800)
        assert r.returncode == 0, r.stderr[-2000:]
        return np.fromfile(out, dtype=np.float32).reshape(len(positions), vocab)


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_full_size_logits_match_reference_runtime(name):
    if not os.path.exists(REF_HOST):
        pytest.skip("oracle/_ref/vault3_host is not built (oracle/Makefile needs the reference sources)")
    from vault_b200 import synth
    from vault_b200.model import VAULTv3ForCausalLM

    spec = CONFIGS[name]
    P, N = spec["prompt"], spec["decode"]
    path = synth.full_model_file(spec["fmt"], seed=0, n_sink=0)
    torch.cuda.set_device(0)
    m = VAULTv3ForCausalLM(path, device=0, verify_crc=False)
    V = m.cfg.vocab_size
    prompt = torch.from_numpy(np.random.default_rng(spec["seed"]).integers(0, 151643, size=P).astype(np.int64))

    # free-running greedy decode on the device
    lg, st = m.prefill(prompt[None])
    first = lg.argmax(-1)
    greedy = torch.cat([first.cpu().to(torch.int64), m.generate(st, first, N - 1).cpu()[0].to(torch.int64)])
    stream = torch.cat([prompt, greedy[:-1]])            # position P-1+i predicts greedy[i]
    positions = list(range(P - 1, P - 1 + N))

    # teacher-forced engine logits at the same positions
    _, st2 = m.prefill(stream[None, :P - 1])
    mine = np.stack([m.step(stream[t:t + 1], st2).cpu().numpy()[0] for t in positions])
    st2.check()

    ref = reference_logits(path, stream.tolist(), positions, V)
    err = float(np.abs(mine - ref).max())
    ref_top = ref.argmax(-1)
    tf = float((mine.argmax(-1) == ref_top).mean())
    agree = ref_top == greedy.numpy()
    free = int(np.argmin(agree)) if not agree.all() else N
    srt = np.sort(ref, axis=-1)
    gaps = [f"{float(srt[i, -1] - srt[i, -2]):.1e}" for i in np.nonzero(mine.argmax(-1) != ref_top)[0]]
    print(f"\n[full-size] {name}: {P}-token prompt + {N} greedy steps, max|dlogit| vs vault3_host {err:.3e} "
          f"(bar {TOL}), teacher-forced top-1 {tf * 100:.2f}%, free-running agreement {free}/{N} steps; "
          f"reference top-1/top-2 gap where the top-1 differs: {gaps or 'none'}")
    assert err <= TOL, err
    assert tf >= 0.99, tf
