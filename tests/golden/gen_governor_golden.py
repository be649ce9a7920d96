"""Generate tests/golden/governor_rules.json.gz: the rules the REFERENCE governor derives (v3_gov_arm_system /
v3_gov_add_rule, runtime/vault3.c:2933-3013, from oracle/_ref/libvault3.so built by oracle/Makefile from the
reference sources) for the system prompts and patterns of tests/test_governor_rules.py.  Run in the build
container:  python tests/golden/gen_governor_golden.py"""
import ctypes as C
import gzip
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.ref_governor import RefGov, ref_lib, rules_of  # noqa: E402
from tests.test_governor_rules import SYSTEM_TEXTS, fold_patterns  # noqa: E402


def main() -> None:
    L = ref_lib()
    arm, add = [], []
    for text in SYSTEM_TEXTS:
        g = RefGov()
        L.v3_gov_arm_system(C.byref(g), text, len(text))
        arm.append({"text": text.hex(), "rules": [r.hex() for r in rules_of(g)]})
    for p in fold_patterns():
        g = RefGov()
        rc = L.v3_gov_add_rule(C.byref(g), p, len(p))
        add.append({"rc": rc, "rules": [r.hex() for r in rules_of(g)]})   # patterns: fold_patterns() order
    with gzip.open(os.path.join(HERE, "governor_rules.json.gz"), "wt") as f:
        json.dump({"arm_system": arm, "add_rule": add}, f, separators=(",", ":"))
    print(f"governor_rules.json.gz: {len(arm)} prompts, {len(add)} patterns")


if __name__ == "__main__":
    main()
