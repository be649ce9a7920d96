"""v3g_argmax_noalloc, the greedy-token entry point for callers that may not allocate device memory (a framework
whose allocator owns all of the GPU's memory, or a token loop that cannot take cudaMalloc's implicit device
synchronisation).  It must pick exactly the tokens v3g_step picks from the same logits, call after call: its
scratch keys live in one fixed device array that every call shares and clears first.

The file name sorts last so that a stop-at-first-failure run has executed every other test before this one."""

import ctypes as C

import numpy as np
import pytest
import torch

from tests.golden.cases import CASES, case_config, case_ids

pytestmark = pytest.mark.gpu


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _noalloc(L, logits: torch.Tensor) -> torch.Tensor:
    rows, vocab = logits.shape
    out = torch.full((rows,), -1, dtype=torch.int32, device=logits.device)
    rc = L.v3g_argmax_noalloc(C.c_void_p(logits.data_ptr()), rows, vocab, logits.stride(0),
                              C.c_void_p(out.data_ptr()), _stream())
    assert rc == 0, L.v3g_last_error()
    return out


def test_argmax_noalloc_matches_step_tokens(case_files):
    from vault_b200 import _lib
    from vault_b200.model import VAULTv3ForCausalLM
    name = "b2_swa_q8_0"   # two sequences: checks the per-row keys
    spec = CASES[name]
    cfg = case_config(spec)
    torch.cuda.set_device(0)
    m = VAULTv3ForCausalLM(case_files(name), device=0, max_sink=cfg.max_sink)
    L = _lib.lib()
    ids = torch.from_numpy(case_ids(spec, cfg)).to(device="cuda:0", dtype=torch.int32)
    B = ids.shape[0]
    st = m.new_state(B)
    results = []
    for t in range(2):   # two steps through the existing entry point: its logits and its greedy tokens
        tok = ids[:, t].contiguous()
        logits = torch.empty(B, cfg.vocab_size, dtype=torch.float32, device="cuda:0")
        nxt = torch.full((B,), -1, dtype=torch.int32, device="cuda:0")
        rc = L.v3g_step(st._h, C.c_void_p(tok.data_ptr()), C.c_void_p(logits.data_ptr()),
                        C.c_void_p(nxt.data_ptr()), _stream())
        assert rc == 0, L.v3g_last_error()
        results.append((logits, nxt))
    (l1, n1), (l2, n2) = results
    # call 1 on the first step's logits
    got1 = _noalloc(L, l1)
    # call 2 right after, on the second step's logits scaled by a power of two (order and ties unchanged) so that
    # every key is below call 1's: a key left over from call 1 would win and show up as a wrong token
    scale = 2.0 ** -10 if float(l2.max()) > 0 else 2.0 ** 10
    l2s = l2 * scale
    assert float(l2s.max()) < float(l1.max())
    got2 = _noalloc(L, l2s)
    torch.cuda.synchronize()
    assert torch.equal(got1, n1), (got1, n1)
    assert torch.equal(got2, n2), (got2, n2)
    # the step's tokens are the first maximum of its logits
    assert got1.cpu().numpy().tolist() == np.argmax(l1.cpu().numpy(), axis=1).tolist()


def test_argmax_noalloc_rejects_too_many_rows():
    from vault_b200 import _lib
    L = _lib.lib()
    torch.cuda.set_device(0)
    rows = 4097   # V3G_NOALLOC_MAX_ROWS + 1
    logits = torch.zeros(rows, 8, dtype=torch.float32, device="cuda:0")
    out = torch.zeros(rows, dtype=torch.int32, device="cuda:0")
    rc = L.v3g_argmax_noalloc(C.c_void_p(logits.data_ptr()), rows, 8, 8, C.c_void_p(out.data_ptr()), _stream())
    assert rc == -10, rc   # V3G_E_LIMIT
    assert "V3G_NOALLOC_MAX_ROWS" in L.v3g_last_error().decode()


def test_argmax_noalloc_selection_rules():
    """The key rules on synthetic rows: NaN is never selected (an all-NaN row gives token 0), a NaN before the
    maximum does not hide it, and -0.0 ties with +0.0 so the first of them wins (runtime/vault3.c:3198-3202)."""
    from vault_b200 import _lib
    L = _lib.lib()
    torch.cuda.set_device(0)
    nan = float("nan")
    rows = torch.tensor([
        [nan, nan, nan, nan, nan, nan],
        [nan, 1.0, 3.0, nan, 2.0, 3.0],
        [-1.0, -0.0, 0.0, -2.0, 0.0, -0.5],
        [-3.0, -1.0, -1.0, -2.0, -4.0, -1.5],
    ], dtype=torch.float32, device="cuda:0")
    for _ in range(2):   # two calls in a row: the shared keys are cleared each time
        got = _noalloc(L, rows)
        torch.cuda.synchronize()
        assert got.cpu().tolist() == [0, 2, 1, 1]
