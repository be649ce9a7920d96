"""Generate the golden fixtures in tests/golden/ by running the REFERENCE implementation (run in the build
container only, where the reference checkout exists; the GPU box never runs this script).

For each case it
  1. draws a seeded synthetic state dict (vault_b200.synth) and writes it to VLT3 with the reference writer
     (tools/vlt3.py write_vlt3) and with this project's writer, asserting the two files are byte-identical and
     recording the SHA-256;
  2. rebuilds the reference model from the file's dequantized weights (as tests/test_vlt3_runtime.py:77-79 does),
     points its token-byte / tier tables at the synthetic tokenizer, and streams the case's token ids through
     VAULTv3ForCausalLM.step (src/vault_v3_model.py:2214), plus prefill(split)+step and forward(mode="block");
  3. stores the ids and fp32 logits in <case>.npz.
It also stores Q8_0/Q4_0 block-codec vectors produced by the reference quantizers/dequantizers.

Usage:  python tests/golden/gen_golden.py --ref <reference checkout>   (or VAULT_REFERENCE=<dir>)
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from tests.golden.cases import CASES, case_config, case_ids  # noqa: E402
from vault_b200 import synth  # noqa: E402
from vault_b200 import vlt3 as my_vlt3  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", nargs="*", default=None, help="regenerate these cases only (others keep their files)")
    ap.add_argument("--ref", default=os.environ.get("VAULT_REFERENCE"),
                    help="root of the reference checkout (default: $VAULT_REFERENCE)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("pass --ref or set VAULT_REFERENCE")
    sys.path.insert(0, args.ref)
    sys.path.insert(0, os.path.join(args.ref, "tools"))
    import torch
    import src.vault_v3_model as rm  # noqa: E402
    import vlt3 as ref_vlt3  # noqa: E402

    torch.set_num_threads(8)
    man_path = os.path.join(HERE, "manifest.json")
    manifest = {}
    if args.only and os.path.exists(man_path):
        with open(man_path) as f:
            manifest = json.load(f)
    with tempfile.TemporaryDirectory() as td:
        for name, spec in CASES.items():
            if args.only and name not in args.only:
                continue
            cfg = case_config(spec)
            tokdir = os.path.join(td, f"tok_{cfg.vocab_size}")
            synth.make_tokenizer_dir(tokdir, cfg.vocab_size, synth.SMALL_EXTRA_TOKENS)
            state = synth.build_state(cfg, spec["seed"], std=spec["std"], gain=spec.get("gain"),
                                      ln_bias_std=spec.get("ln_bias_std", 0.0))
            ref_cfg = rm.VAULTv3Config(**{k: v for k, v in cfg.to_dict().items()
                                          if k in rm.VAULTv3Config.__dataclass_fields__})
            ref_cfg.seg_layers = tuple(cfg.seg_layers)
            tstate = {k: torch.from_numpy(v) for k, v in state.items()}
            p_ref = os.path.join(td, f"{name}_ref.vlt3")
            p_me = os.path.join(td, f"{name}_me.vlt3")
            ref_vlt3.write_vlt3(p_ref, tstate, ref_cfg, tokdir, spec["fmt"], model_name=name)
            my_vlt3.write_vlt3(p_me, state, cfg, tokdir, spec["fmt"], model_name=name)
            b_ref = open(p_ref, "rb").read()
            b_me = open(p_me, "rb").read()
            assert b_ref == b_me, f"{name}: writer output differs from the reference writer"
            sha = hashlib.sha256(b_ref).hexdigest()

            vf = ref_vlt3.read_vlt3(p_ref)
            model = rm.VAULTv3ForCausalLM(ref_cfg).float().eval()
            model.load_state_dict(ref_vlt3.vlt3_to_state_dict(vf), strict=True)
            model._raw_bytes = rm.build_token_raw_bytes(cfg.vocab_size, tokdir)
            model._tier_lut = rm.build_token_tier_lut(cfg.vocab_size, tokdir)
            model._brk_mask = model._tier_lut == 1

            ids = case_ids(spec, cfg)                         # [B, L]
            B, L = ids.shape
            t_ids = torch.from_numpy(ids).long()
            out = {"ids": ids}
            with torch.no_grad():
                seg_b = None if B == 1 else 0
                st = model.new_state(B, seg_budget=seg_b)
                steps = [model.step(t_ids[:, t], st).numpy() for t in range(L)]
                out["step_logits"] = np.stack(steps, axis=1).astype(np.float32)          # [B, L, V]
                out["final_n_pin"] = np.int64(st.n_pin)
                out["final_mem_pos"] = st.mem_pos.numpy().astype(np.int64)
                out["final_mem_score"] = st.mem_score.numpy().astype(np.float32)
                out["final_sc_prev"] = st.sc_prev[0].numpy().astype(np.float32)
                if spec.get("forward", True):
                    fwd = model(t_ids, mode="block", seg_budget=seg_b).numpy().astype(np.float32)
                    out["forward_logits"] = fwd
                splits = spec.get("splits", [])
                for sp in splits:
                    lg, st2 = model.prefill(t_ids[:, :sp], seg_budget=seg_b)
                    tail = [lg.numpy()] + [model.step(t_ids[:, t], st2).numpy() for t in range(sp, L)]
                    out[f"prefill{sp}_logits"] = np.stack(tail, axis=1).astype(np.float32)  # [B, L-sp+1, V]
            np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
            fwd_err = float(np.abs(out["forward_logits"] - out["step_logits"]).max()) if "forward_logits" in out else 0.0
            manifest[name] = {"sha256": sha, "bytes": len(b_ref), "fmt": spec["fmt"], "B": B, "L": L,
                              "forward_vs_step_max_abs": fwd_err, "final_n_pin": int(out["final_n_pin"]),
                              "final_mem_cnt": int(len(out["final_mem_pos"]))}
            print(f"[golden] {name}: {len(b_ref)} B sha={sha[:12]} B={B} L={L} n_pin={int(out['final_n_pin'])} "
                  f"mem={len(out['final_mem_pos'])} fwd-vs-step={fwd_err:.2e}")

    # block-codec vectors from the reference quantizers / dequantizers
    if args.only:
        with open(man_path, "w") as f:
            json.dump(manifest, f, indent=1, sort_keys=True)
        return
    rng = np.random.default_rng(1234)
    w = (rng.standard_normal(32 * 96).astype(np.float32) * 0.05)
    w[:32] = 0.0                                   # all-zero block (d = 0 path)
    w[32:64] *= 1e-6                               # tiny block (fp16 subnormal scale)
    w[64] = 3.0                                    # outlier block
    q8 = ref_vlt3.quantize_q8_0(w)
    q4 = ref_vlt3.quantize_q4_0(w)
    np.savez_compressed(os.path.join(HERE, "codec.npz"), w=w,
                        q8=np.frombuffer(q8, np.uint8), q8_deq=ref_vlt3.dequantize_q8_0(q8, w.size),
                        q4=np.frombuffer(q4, np.uint8), q4_deq=ref_vlt3.dequantize_q4_0(q4, w.size))
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print("[golden] wrote", os.path.join(HERE, "manifest.json"))


if __name__ == "__main__":
    main()
