"""The JSON prefix oracle (oracle/json_prefix.py) against the reference's own
answers: the committed golden vectors (tests/golden/json_prefix_golden.json,
made by tests/golden/make_json_golden.py from miniserve's
JSONLogitsProcessor.is_valid_prefix, miniserve/sampler.py:139-148), and, where
the reference tree is present, a fresh fuzz against it."""
import json
import os
import random
import sys

import pytest

from oracle import json_prefix as jp
import golden_util

HERE = os.path.dirname(os.path.abspath(__file__))


def _golden():
    with open(os.path.join(HERE, "golden", "json_prefix_golden.json")) as f:
        return json.load(f)


def test_oracle_matches_golden_cases():
    g = _golden()
    bad = [(s, a) for s, a in g["cases"] if jp.is_valid_prefix(s) != a]
    assert not bad, bad[:10]
    assert len(g["cases"]) > 5000


def test_oracle_matches_golden_long_probes():
    for h, u, n, t, a in _golden()["long"]:
        assert jp.is_valid_prefix(h + u * n + t) == a, (h, u, n, t, a)


def test_known_answers():
    # the probes of the reference's behaviour that decide the mask's classes
    assert jp.is_valid_prefix("") is True
    assert jp.is_valid_prefix(" {x") is True          # leading space: parsed, "Expecting property name"
    assert jp.is_valid_prefix("{anything") is True    # raw first character '{'
    assert jp.is_valid_prefix("[1,]") is True         # "Expecting value"
    assert jp.is_valid_prefix("1.") is False          # "Extra data"
    assert jp.is_valid_prefix("01") is False
    assert jp.is_valid_prefix("true,") is False
    assert jp.is_valid_prefix("[1]]") is False
    assert jp.is_valid_prefix('"\\q') is False         # "Invalid \\escape"
    assert jp.is_valid_prefix('"\\u0041') is False     # four digits need one more character
    assert jp.is_valid_prefix('"\\u0041x') is True
    assert jp.is_valid_prefix('"\x01') is False        # "Invalid control character at"
    assert jp.is_valid_prefix("nulx") is True
    assert jp.is_valid_prefix("-Infinity") is True


def test_pack_mask_layout():
    words = jp.pack_mask([True, False, True] + [False] * 29 + [True])
    assert words.tolist() == [0b101, 1]


def test_fuzz_against_live_reference():
    ref = golden_util.reference_root()
    if not os.path.exists(os.path.join(ref, "miniserve", "sampler.py")):
        pytest.skip("reference tree not present (the golden vectors pin the oracle)")
    sys.path.insert(0, ref)
    from miniserve.sampler import JSONLogitsProcessor
    f = JSONLogitsProcessor().is_valid_prefix
    rng = random.Random(7)
    alpha = list('{}[]:,"\\ \t\n\r0123456789.-+eEtrufalsenNIyi') + [
        "\\u", "\\ud834", "true", "null", "NaN", "-Infinity", "\x01", "é"]
    for _ in range(20000):
        s = "".join(rng.choice(alpha) for _ in range(rng.randint(0, 14)))
        if rng.random() < 0.3:
            s = "[" + s
        try:
            want = f(s)
        except (RecursionError, ValueError):
            want = jp.RAISE
        assert jp.is_valid_prefix(s) == want, repr(s)


def test_length_order():
    """The mask builder's evaluation order: token ids sorted by (plain first,
    UTF-8 byte length, bytes) -- plain: 1-16 bytes, none of them '"', '\\' or
    a control byte -- a permutation of the vocabulary; unknown orders are
    refused before anything touches a device."""
    from miniserve_b200.grammar import JsonMaskBuilder, length_order
    vocab = ["bb", "a", "ab", "", "é", "{", "aa", 'a"', "\\n", "x\n", "z" * 17]
    order = length_order(vocab)
    assert sorted(order) == list(range(len(vocab)))

    def plain(b):
        return 0 < len(b) <= 16 and all(c >= 0x20 and c not in (0x22, 0x5C) for c in b)
    keys = [(not plain(vocab[t].encode()), len(vocab[t].encode()), vocab[t].encode()) for t in order]
    assert keys == sorted(keys)
    # the six plain tokens first, by (length, bytes); then the rest, the empty token first
    assert [vocab[t] for t in order[:6]] == ["a", "{", "aa", "ab", "bb", "é"]
    assert vocab[order[6]] == ""
    with pytest.raises(ValueError):
        JsonMaskBuilder(vocab, device="cpu", order="alphabetical")


def test_oracle_matches_mask_fuzz_fixture():
    """oracle/json_prefix.py against miniserve's answers for 10^6 (state,
    token) pairs (tests/golden/json_mask_fuzz.npz)."""
    from miniserve_b200 import workloads
    prefixes, tokens, allowed, raises = golden_util.load_mask_fuzz()
    vocab = workloads.json_vocab(4)
    raised = set(raises)
    bad = []
    for i, p in enumerate(prefixes):
        for j, t in enumerate(tokens[i].tolist()):
            got = jp.is_valid_prefix(p + vocab[t])
            want = jp.RAISE if (i, j) in raised else bool(allowed[i, j])
            if got != want:
                bad.append((i, vocab[t], want))
    assert tokens.size == 1_000_000
    assert not bad, bad[:10]
