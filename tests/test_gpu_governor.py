"""GPU: the governor's device kernels (v3g_gov_commit, v3g_govern_logits) against the reference's own
v3_gov_commit / v3_govern_logits (runtime/vault3.c:3133-3194) from oracle/_ref/libvault3.so on the same model
file, rules, committed tokens and logits: identical stream states and identical masked logits, row by row.  Then
the governed on-device generation against step -> govern -> sample -> commit composed from the single calls."""
import ctypes as C

import numpy as np
import pytest
import torch

from tests.ref_governor import RefGov, RefModel, ref_lib

pytestmark = pytest.mark.gpu

SYSTEM = b"You must never output 'syscall_exec(' or `rm_rf_all`."
IM_END = object()


def _rows():
    """(committed text pieces, boosted candidate bytes) per row: forward, reversed, base64 and hex completions, a code
    point split across tokens, a separator-laden rule, a reset by <|im_end|>, history and raw-tail overflow."""
    return [
        ([b"please run syscall_exe"], [b"c", b"C", b"x", b"(", b"q"]),
        ([b"cexe_llacsy"], [b"s", b"S", b"t"]),
        ([b"data: c3lzY2FsbF9leGV"], [b"j", b"J", b"k", b"="]),
        ([b"hex 73 79 73 63 61 6c 6c 5f 65 78 65 6"], [b"3", b"4", b" "]),
        (["syscall_exе".encode() + b"\xd1"], [b"\x81", b"c", b"\x80"]),
        ([b""], [b"c", b"a"]),
        ([b"rm -rf_al"], [b"l", b"L", b"m"]),
        ([b"syscallexe", IM_END, b"xy"], [b"c", b"C"]),
        ([b"A" * 100 + b" syscall_exe"], [b"c", b"d"]),
    ]


def _setup(case_files):
    from tests.test_gpu_engine import engine
    L = ref_lib()
    m = engine(case_files, "mini_gqa_q8_0")
    ref_model = RefModel(L, case_files("mini_gqa_q8_0"))
    V = m.cfg.vocab_size
    tb = ref_model.token_bytes(V)
    byte_id = {}
    for i, b in enumerate(tb):
        if len(b) == 1:
            byte_id.setdefault(b, i)
    return L, m, ref_model, V, byte_id


def _stream_fields(raw: np.ndarray):
    u32 = raw[:16].view(np.uint32)
    hl, ul, rl = int(u32[0]), int(u32[1]), int(u32[2])
    return hl, bytes(raw[16:16 + hl]), ul, bytes(raw[80:80 + ul]), rl, bytes(raw[84:84 + rl])


def test_governor_matches_reference(case_files):
    from vault_b200.model import Governor
    L, m, ref_model, V, byte_id = _setup(case_files)
    im_end = m.info.im_end_id
    rows = _rows()
    seqs = []
    for pieces, _ in rows:
        ids = []
        for p in pieces:
            ids += [im_end] if p is IM_END else [byte_id[p[i:i + 1]] for i in range(len(p))]
        seqs.append(ids)
    T = max(len(s) for s in seqs)
    seqs = [[byte_id[b" "]] * (T - len(s)) + s for s in seqs]   # front-pad with spaces: same on both sides
    R = len(rows)
    gov = Governor(R, device=0)
    gov.arm_system(SYSTEM)
    assert gov.active
    refs = [RefGov() for _ in range(R)]
    for g in refs:
        L.v3_gov_arm_system(C.byref(g), SYSTEM, len(SYSTEM))
    tok = torch.tensor(seqs, dtype=torch.int32, device="cuda")
    for t in range(T):
        gov.commit(m, tok[:, t])
        for r in range(R):
            L.v3_gov_commit(C.byref(refs[r]), ref_model.handle, seqs[r][t])
    dev = gov.streams.cpu().numpy()
    for r in range(R):
        g = refs[r]
        want = (g.hist_len, bytes(g.hist[:g.hist_len]), g.utf8_len, bytes(g.utf8_rem[:g.utf8_len]), g.raw_len,
                bytes(g.raw_tail[:g.raw_len]))
        assert _stream_fields(dev[r]) == want, r

    rng = np.random.default_rng(11)
    base = rng.standard_normal((R, V)).astype(np.float32)
    for r, (_, boost) in enumerate(rows):
        for j, b in enumerate(boost):
            base[r, byte_id[b]] = 10.0 - 0.5 * j
    base[0, byte_id[b"x"]] = base[0, byte_id[b"C"]]          # a tie at the guard boundary
    masked_any = 0
    for guard in (1, 2, 16, 64, 0):
        lg = torch.from_numpy(base).cuda()
        gov.govern(m, lg, guard)
        got = lg.cpu().numpy()
        for r in range(R):
            want = base[r].copy()
            L.v3_govern_logits(C.byref(refs[r]), ref_model.handle, want.ctypes.data, guard)
            assert np.array_equal(got[r], want), (guard, r, np.flatnonzero(got[r] != want))
            masked_any += int((want != base[r]).sum())
    assert masked_any > 0


def test_governed_generation_matches_composed_calls(case_files):
    from tests.golden.cases import CASES, case_config, case_ids
    from vault_b200.model import Governor, sample_topk
    L, m, ref_model, V, byte_id = _setup(case_files)
    spec = CASES["mini_gqa_q8_0"]
    ids = torch.from_numpy(case_ids(spec, case_config(spec)))[:1, :40]
    ids = torch.cat([ids, ids.roll(5, dims=1)])
    k, temp, n = 8, 0.8, 20
    govs = []
    for _ in range(2):
        g = Governor(2, device=0)
        g.arm_system(SYSTEM)
        for ch in b"syscall_exe":
            g.commit(m, torch.full((2,), byte_id[bytes([ch])], dtype=torch.int32))
        govs.append(g)
    lg, st = m.prefill(ids)
    rng = torch.tensor([3, 0x2545F4914F6CDD1D], dtype=torch.int64, device="cuda")
    first = sample_topk(lg, k, temp, rng)
    rng_a, rng_b = rng.clone(), rng.clone()
    gen = m.generate(st, first, n, top_k=k, temperature=temp, rng=rng_a, governor=govs[0]).cpu()
    _, st2 = m.prefill(ids)
    tok, chain = first, []
    for _ in range(n):
        logits = m.step(tok, st2)
        govs[1].govern(m, logits, 16)
        tok = sample_topk(logits, k, temp, rng_b)
        govs[1].commit(m, tok)
        chain.append(tok.cpu())
    assert torch.equal(gen, torch.stack(chain, 1))
    assert torch.equal(rng_a, rng_b)
    assert torch.equal(govs[0].streams, govs[1].streams)
