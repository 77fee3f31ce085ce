"""Generate ``json_prefix_golden.json`` by running miniserve's own prefix test.

Run where the reference source tree is available (it is not on the GPU box):

    MINISERVE_REF=/path/to/miniserve python tests/golden/make_json_golden.py

It imports ``JSONLogitsProcessor`` from the reference
(miniserve/sampler.py:115-148) and records ``is_valid_prefix(s)`` -- True,
False, or "raise" where the reference raises a non-JSONDecodeError exception
-- for: hand-picked probes of every error class, config-4 strings (a prefix
of ``miniserve_b200.workloads.json_prefixes`` followed by a token of
``json_vocab``), and seeded random strings over a JSON-heavy alphabet.  The
tests pin ``oracle/json_prefix.py`` and the GPU mask builder to these answers.
"""
from __future__ import annotations

import json
import os
import random
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

import golden_util  # noqa: E402
from miniserve_b200 import workloads  # noqa: E402

PROBES = ['"\\u0041', '"\\u0041x', '"\\u004', '"\\uZZZZ', '"\\uZZZZx', '"ab\\', '"\\q', '[1.', '1.', '1.5', '1e',
          '1e+', '1e+5', '[1e+', '-', '-I', '-Infinity', '-Inf', 'NaN', 'Na', 'nulx', 'nul', 'truex', '[truex',
          'true ', ' {x', '{x', '', '   ', '1 2', '[1 2', '"\\ud834\\u12', '"\\ud834', '"\\ud834\\udd1e',
          '"\\ud834\\udd1', '"\x01', '[\x01', '\x01', '"\t"', '[1,]', '[]]', '01', '[01]', '-0', '-01', '0e',
          '0.e1', '[0.e1]', '"\\u00e9"', '1E5', '1e05', ']', "'", '[1]]', 'true,', '"\\u12', ' [1,{"a":[}]',
          '[{"a" 1}]', '[{1:2}]', '[{"a":1,}]', '[{"a":1,"b"}]', '"\\/\\b\\f\\n\\r\\t\\"\\\\"', '[-Infinity,NaN]']
# long probes, stored as (head, unit, count, tail): head + unit * count + tail
LONG = [("", "1", 4300, ""), ("", "1", 4301, ""), ("[", "1", 4301, ""), ("", "1", 4301, ".5"),
        ("", "1", 4301, "e5"), ("-", "1", 4301, ""), ("", "[", 9996, ""), ("", "[", 9997, ""),
        (" ", '[{"a":', 4998, ""), (" ", '[{"a":', 4999, "")]
MAX_CASE = 1000  # characters; longer config-4 prefixes are checked against the oracle instead


def _ref():
    ref = golden_util.reference_root()
    sys.path.insert(0, ref)
    from miniserve.sampler import JSONLogitsProcessor  # type: ignore
    return JSONLogitsProcessor().is_valid_prefix


def answer(f, s):
    try:
        return bool(f(s))
    except (RecursionError, ValueError):
        return "raise"


def main():
    f = _ref()
    rng = random.Random(20261201)
    cases = list(PROBES)
    vocab = workloads.json_vocab(4)
    prefixes = workloads.json_prefixes(4, 128)
    for p in prefixes:
        if len(p) > MAX_CASE:
            continue
        for _ in range(24):
            cases.append(p + rng.choice(vocab))
    alpha = list('{}[]:,"\\ \t\n\r0123456789.-+eEtrufalsenNIyi') + [
        '\\u', '\\ud834', 'true', 'false', 'null', 'NaN', 'Infinity', '-Infinity', '\x01', 'é', 'x']
    for _ in range(3000):
        s = "".join(rng.choice(alpha) for _ in range(rng.randint(0, 14)))
        cases.append(("[" + s) if rng.random() < 0.3 else s)
    out = {"python": sys.version.split()[0], "cases": [[s, answer(f, s)] for s in cases],
           "long": [[h, u, n, t, answer(f, h + u * n + t)] for h, u, n, t in LONG]}
    with open(os.path.join(HERE, "json_prefix_golden.json"), "w") as fh:
        json.dump(out, fh, separators=(",", ":"))
    print("wrote json_prefix_golden.json", len(cases))


if __name__ == "__main__":
    main()
