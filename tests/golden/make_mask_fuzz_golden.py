"""Generate ``json_mask_fuzz.npz``: miniserve's own answers for 10^6
(parse state, token) pairs of the config-4 kind.

Run where the reference source tree is available (it is not on the GPU box):

    MINISERVE_REF=/path/to/miniserve python tests/golden/make_mask_fuzz_golden.py

States: 40 prefixes built from ``miniserve_b200.workloads.json_prefixes(4,
2048)`` (``states()``: top-level scalars and arrays, objects behind a space,
objects inside an array).  Tokens:
for state i, ``random.Random(SEED + i).sample(range(V), N_TOKENS)`` of
``json_vocab(4)`` (V = 151936).  For every pair it records
``JSONLogitsProcessor().is_valid_prefix(prefix + token)``
(miniserve/sampler.py:139-148): True / False, or "raise" where the reference
raises a non-JSONDecodeError exception.  The fixture stores the prefixes and
the answers (True bits packed, raises as a list); the tests
rebuild the token samples from the seeds and pin both the CUDA mask builder
and ``oracle/json_prefix.py`` to it.
"""
from __future__ import annotations

import os
import random
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

import golden_util  # noqa: E402
from miniserve_b200 import workloads  # noqa: E402

N_STATES = 40
N_TOKENS = 25000
MAX_PREFIX = 400
SEED = 20261202
OUT = os.path.join(HERE, "json_mask_fuzz.npz")


def states():
    """The fixture's prefixes, from json_prefixes(4, 2048) (distinct, under
    MAX_PREFIX characters): 7 top-level scalars and 7 arrays as they are, 13
    objects behind one space (a raw first '{' makes the reference accept
    whatever follows; after a space the object is parsed), and 13 objects
    inside an array."""
    pre = [p for p in dict.fromkeys(workloads.json_prefixes(4, 2048)) if len(p) < MAX_PREFIX]
    scalars = [p for p in pre if not p.startswith(("{", "["))][:7]
    arrays = [p for p in pre if p.startswith("[")][:7]
    objs = [p for p in pre if p.startswith("{") and len(p) > 8]
    return scalars + arrays + [" " + p for p in objs[:13]] + ["[" + p for p in objs[13:26]]


def token_sample(i: int, V: int):
    return random.Random(SEED + i).sample(range(V), N_TOKENS)


def main():
    ref = golden_util.reference_root()
    sys.path.insert(0, ref)
    from miniserve.sampler import JSONLogitsProcessor  # type: ignore
    f = JSONLogitsProcessor().is_valid_prefix
    pre = states()
    assert len(pre) == N_STATES
    vocab = workloads.json_vocab(4)
    ans = np.zeros((len(pre), N_TOKENS), bool)
    raises = []
    t0 = time.time()
    for i, p in enumerate(pre):
        for j, t in enumerate(token_sample(i, len(vocab))):
            try:
                ans[i, j] = bool(f(p + vocab[t]))
            except (RecursionError, ValueError):
                raises.append((i, j))
    np.savez_compressed(OUT, prefixes=np.array(pre), true_bits=np.packbits(ans, axis=1),
                        raises=np.array(raises, np.int32).reshape(-1, 2),
                        meta=np.array([N_STATES, N_TOKENS, MAX_PREFIX, SEED, len(vocab)], np.int64),
                        python=np.array(sys.version.split()[0]))
    print(f"wrote {OUT}: {ans.size} pairs, {ans.mean():.3f} allowed, {len(raises)} raises, "
          f"{time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
