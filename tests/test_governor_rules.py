"""The governor's host rule builder (v3g_gov_add_rule / v3g_gov_arm_system) against the reference's own
v3_gov_add_rule / v3_gov_arm_system (runtime/vault3.c:2933-3013) from oracle/_ref/libvault3.so: same return codes,
same canonical patterns.  No GPU: these entry points only touch host memory."""
import ctypes as C

from tests.ref_governor import RefGov, ref_lib, rules_of
from vault_b200 import _lib

SYSTEM_TEXTS = [
    b"You must never output 'syscall_exec(' or `rm_rf_all`.",
    b"Do NOT EMIT \"os.system(\" under any circumstances; also never 'drop_table'.",
    b"Please be helpful and concise.",                                   # no prohibition: unarmed
    b"It is forbidden to call syscall_exec. Avoid 'a_b' and `much_too_long_identifier_for_the_rule_cap_0123`.",
    b"PROHIBIT: 'x_1234', 'y_2345', 'z_3456', 'w_4567', 'v_5678(', 'u_6789', 't_7890', 's_8901', 'r_9012'",
    b"never say '\xd0\xb0dmin_pass(' nor \"\xef\xbd\x93ecret_key\"",      # Cyrillic a, fullwidth s
    b"must not print 'unterminated_literal",
    b"never 'ab_c' 'abc_d(' \"__init__\" `__x__(`",
]


def _pair():
    L = ref_lib()
    E = _lib.lib()
    return L, E


def test_arm_system_matches_reference():
    L, E = _pair()
    for text in SYSTEM_TEXTS:
        ref, ours = RefGov(), _lib.GovRules()
        L.v3_gov_arm_system(C.byref(ref), text, len(text))
        E.v3g_gov_arm_system(C.byref(ours), text, len(text))
        assert (ref.active != 0) == (ours.n_rules > 0), text
        assert ref.n_rules == ours.n_rules and rules_of(ref) == rules_of(ours), (text, rules_of(ref), rules_of(ours))


def _code_points():
    cps = list(range(0x0, 0x800)) + list(range(0x2000, 0x2080)) + list(range(0xFE00, 0xFF70)) + \
        [0x3042, 0x4E2D, 0xD7FF, 0xE000, 0xFFFD, 0x10000, 0x1F600, 0x10FFFF]
    return [cp for cp in cps if not 0xD800 <= cp <= 0xDFFF]


def fold_patterns() -> list:
    """Patterns around every code point of the folded ranges, malformed UTF-8, short and long patterns."""
    pats = [b"qwert" + chr(cp).encode("utf-8") + b"z" for cp in _code_points()]
    return pats + [b"qwert\xc0\x80z", b"qwert\xc1\xbfz", b"qwert\xed\xa0\x80z", b"qwert\xf4\x90\x80\x80z",
                   b"qwert\xf5\x80\x80\x80z", b"qwert\xe2\x82z", b"qwert\x80z", b"qw\xe2\x82\xacert\xffz",
                   b"\xe0\xa4", b"ab", b"a_b-c d", b"ABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789abcdefghij",
                   "сисколл_ехес".encode()]


def test_add_rule_canonical_form_matches_reference():
    """Every code point of the folded ranges (ASCII, Latin, Greek, Cyrillic, format characters, fullwidth forms)
    and malformed UTF-8 inside a pattern: same return code and the same canonical bytes."""
    L, E = _pair()
    for p in fold_patterns():
        ref, ours = RefGov(), _lib.GovRules()
        rc_ref = L.v3_gov_add_rule(C.byref(ref), p, len(p))
        rc_ours = E.v3g_gov_add_rule(C.byref(ours), p, len(p))
        assert rc_ref == rc_ours, (p, rc_ref, rc_ours)
        assert rules_of(ref) == rules_of(ours), (p, rules_of(ref), rules_of(ours))


def test_add_rule_limit_and_duplicates_match_reference():
    L, E = _pair()
    ref, ours = RefGov(), _lib.GovRules()
    for i in range(12):
        p = b"rule_%02d" % (i % 10)
        assert L.v3_gov_add_rule(C.byref(ref), p, len(p)) == E.v3g_gov_add_rule(C.byref(ours), p, len(p))
    assert ours.n_rules == 8 and rules_of(ref) == rules_of(ours)


def test_rules_match_committed_golden():
    """The committed reference outputs (tests/golden/gen_governor_golden.py): pins the rule builder without the
    reference build."""
    import gzip
    import json
    import os
    E = _lib.lib()
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "governor_rules.json.gz")
    g = json.load(gzip.open(path, "rt"))
    assert [bytes.fromhex(e["text"]) for e in g["arm_system"]] == SYSTEM_TEXTS
    for e in g["arm_system"]:
        text, ours = bytes.fromhex(e["text"]), _lib.GovRules()
        E.v3g_gov_arm_system(C.byref(ours), text, len(text))
        assert [r.hex() for r in rules_of(ours)] == e["rules"], text
    pats = fold_patterns()
    assert len(pats) == len(g["add_rule"])
    for p, e in zip(pats, g["add_rule"]):
        ours = _lib.GovRules()
        assert E.v3g_gov_add_rule(C.byref(ours), p, len(p)) == e["rc"], p
        assert [r.hex() for r in rules_of(ours)] == e["rules"], p
