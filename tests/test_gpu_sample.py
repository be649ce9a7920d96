"""GPU: top-k + temperature sampling on the device (v3g_sample_topk) against the sampler oracle, which
tests/test_oracle_sample.py pins to the reference's own v3_sample_topk.  Tokens and the updated xorshift states
must match bit for bit (the device draw uses the reference's operation order and exponential), over two calls in
a row so the state update is chained."""
import numpy as np
import pytest
import torch

from oracle import sample_oracle as so
from tests.test_oracle_sample import sample_cases

pytestmark = pytest.mark.gpu


def _to_i64(u: int) -> int:
    return u - (1 << 64) if u >= 1 << 63 else u


def _to_u64(i: int) -> int:
    return i + (1 << 64) if i < 0 else i


def test_sample_topk_matches_oracle():
    from vault_b200.model import sample_topk
    torch.cuda.set_device(0)
    for v, k, temp, state in sample_cases():
        logits = torch.from_numpy(np.stack([v, v[::-1].copy()])).cuda()
        states = [state, state ^ 0x5DEECE66D]
        rng = torch.tensor([_to_i64(s) for s in states], dtype=torch.int64, device="cuda")
        for call in range(2):
            tok = sample_topk(logits, k, temp, rng).cpu().tolist()
            got_states = [_to_u64(x) for x in rng.cpu().tolist()]
            for r in range(2):
                otok, states[r] = so.sample_topk(logits[r].cpu().numpy(), k, temp, states[r])
                assert tok[r] == otok, (len(v), k, temp, call, r)
                assert got_states[r] == states[r]


def test_sample_topk_skips_nan_rows():
    from vault_b200.model import sample_topk
    nan = float("nan")
    logits = torch.tensor([[nan, nan, nan, nan], [nan, 1.0, 3.0, 2.0]], dtype=torch.float32, device="cuda")
    rng = torch.tensor([5, 9], dtype=torch.int64, device="cuda")
    tok = sample_topk(logits, 4, 1.0, rng).cpu().tolist()
    assert tok[0] == 0
    otok, _ = so.sample_topk(logits[1].cpu().numpy(), 4, 1.0, 9)
    assert tok[1] == otok


def test_generate_sampled_matches_step_then_sample(case_files):
    """v3g_generate_sampled (the on-device loop) against step -> sample_topk on the host side, two sequences with
    their own xorshift states: same tokens, same final states; every draw of the host loop also matches the sampler
    oracle on that step's logits."""
    from tests.golden.cases import CASES, case_config, case_ids
    from tests.test_gpu_engine import engine
    from vault_b200.model import sample_topk
    torch.cuda.set_device(0)
    m = engine(case_files, "mini_gqa_q8_0")
    spec = CASES["mini_gqa_q8_0"]
    ids = torch.from_numpy(case_ids(spec, case_config(spec)))[:1, :40]
    ids = torch.cat([ids, ids.roll(3, dims=1)])
    k, temp, n = 20, 1.5, 24
    lg, st = m.prefill(ids)
    rng = torch.tensor([0, 0x1234567], dtype=torch.int64, device="cuda")
    first = sample_topk(lg, k, temp, rng)
    rng_a, rng_b = rng.clone(), rng.clone()
    gen = m.generate(st, first, n, top_k=k, temperature=temp, rng=rng_a).cpu()
    _, st2 = m.prefill(ids)
    states = [_to_u64(x) for x in rng_b.cpu().tolist()]
    tok, chain = first, []
    for _ in range(n):
        logits = m.step(tok, st2)
        tok = sample_topk(logits, k, temp, rng_b)
        for r in range(2):
            otok, states[r] = so.sample_topk(logits[r].cpu().numpy(), k, temp, states[r])
            assert int(tok[r]) == otok
        chain.append(tok.cpu())
    assert torch.equal(gen, torch.stack(chain, 1))
    assert torch.equal(rng_a, rng_b) and [_to_u64(x) for x in rng_a.cpu().tolist()] == states
    assert not torch.equal(rng_a, rng)
