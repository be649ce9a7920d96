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
