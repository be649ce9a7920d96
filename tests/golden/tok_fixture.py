"""The tokenizer test fixture: a small VLT3 file whose VTOK blob carries a merge table trained on a fixed corpus of
text fragments, and the seeded texts encoded with it.  Shared by tests/test_tokenizer.py and gen_tokenizer_golden.py
(deterministic: the same file bytes on every machine)."""
import dataclasses
import json
import os
import random

FRAGMENTS = [
    "Hello world", " I'm here", " they'll GO", " DON'T", "'s", " 12345", " 3.14159", "!!", " ...", "\n\n", "\r\n",
    "\t\tindent", "   spaces   ", "<|im_start|>system\nBe brief.<|im_end|>\n", "<|im_start|>user\n", "<|im_end|>",
    "<|im_sta", "<|endoftext|>", "café", "café", "Å", "Å", "ạ́", "ạ́",
    "ḍ̇", "q̣̇", "한국어", "각", "하", "中文字",
    "\U0001F600 ok", "क़", "क़", "Åñ", "αβγ", "Жук",
    "الع", "  nbsp", " ", "x​y", "ﬁ", "Ω", "̈́", "ཱི",
    "'ll", "'VE", "a'b", "  \n  x", "line\n", "ab;x}y&q", '",', ". ", ", ",
]
BAD_BYTES = [b"\xff", b"\x80", b"\xc0\x80", b"\xed\xa0\x80", b"\xf4\x90\x80\x80", b"\xe2\x82", b"\xcc", b"\xcc\x81"]


def _corpus_texts(rng: random.Random, n: int) -> list:
    out = []
    for _ in range(n):
        parts = []
        for _ in range(rng.randint(1, 12)):
            if rng.random() < 0.1:
                parts.append(rng.choice(BAD_BYTES))
            else:
                parts.append(rng.choice(FRAGMENTS).encode("utf-8"))
        out.append(b"".join(parts))
    return out


def _train_merges(tok_dir: str, vocab_size: int, n_merges: int) -> None:
    """Greedy BPE over the fragments (GPT-2 byte-unicode form), new tokens on free ids; one repeated merge line."""
    from vault_b200.synth import byte_to_unicode
    path = os.path.join(tok_dir, "tokenizer.json")
    tj = json.load(open(path, encoding="utf-8"))
    vocab = tj["model"]["vocab"]
    b2u = byte_to_unicode()
    taken = set(vocab.values()) | {t["id"] for t in tj["added_tokens"]}
    free = (i for i in range(vocab_size) if i not in taken)
    words = [[b2u[b] for b in f.encode("utf-8")] for f in FRAGMENTS * 3 + ["the", " the", " there", "ing"] * 5]
    merges = []
    for _ in range(n_merges):
        counts = {}
        for w in words:
            for a, b in zip(w, w[1:]):
                counts[(a, b)] = counts.get((a, b), 0) + 1
        if not counts:
            break
        (a, b), _ = max(counts.items(), key=lambda kv: (kv[1], kv[0]))
        if a + b not in vocab:
            vocab[a + b] = next(free)
        merges.append(f"{a} {b}")
        for w in words:
            i = 0
            while i + 1 < len(w):
                if w[i] == a and w[i + 1] == b:
                    w[i:i + 2] = [a + b]
                i += 1
    merges.insert(len(merges) // 2, merges[len(merges) // 3])   # a repeated pair: its first rank wins
    tj["model"]["merges"] = merges
    json.dump(tj, open(path, "w", encoding="utf-8"), ensure_ascii=False)



def build_tokenizer_file(td: str) -> str:
    """Write the fixture model (the mini GQA case's shapes with a 1,024-id vocabulary) into td; returns its path."""
    from tests.golden.cases import CASES, case_config
    from vault_b200 import synth
    spec = CASES["mini_gqa_q8_0"]
    cfg = dataclasses.replace(case_config(spec), vocab_size=1024)
    tok_dir = os.path.join(td, "tok")
    synth.make_tokenizer_dir(tok_dir, cfg.vocab_size, synth.SMALL_EXTRA_TOKENS)
    _train_merges(tok_dir, cfg.vocab_size, 400)
    path = os.path.join(td, "m.vlt3")
    synth.write_synthetic_vlt3(path, cfg, spec["fmt"], spec["seed"], tokenizer_dir=tok_dir, model_name="tok",
                               std=spec["std"])
    return path


def golden_texts() -> list:
    """(text, allow_special) pairs stored in tokenizer.npz."""
    texts = _corpus_texts(random.Random(77), 300)
    return [(t, s) for i, t in enumerate(texts) for s in ((1, 0) if i % 3 == 0 else (1,))]
