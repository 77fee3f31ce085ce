"""Loads the committed golden fixtures and rebuilds their inputs."""
from __future__ import annotations

import json
import os

import numpy as np

from miniserve_b200 import workloads

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sampler_golden.json")


def load():
    with open(GOLDEN) as f:
        return json.load(f)


def expected_token(t):
    """Reference token, or -1 where the reference raised ZeroDivisionError."""
    return -1 if t == "ZeroDivisionError" else int(t)


def config_batch(entry):
    g = dict(entry["gen"])
    fn = getattr(workloads, g.pop("fn"))
    return fn(**g)


def reference_root() -> str:
    """The reference source tree: $MINISERVE_REF, else BASELINE.json's
    reference_path (present only where the fixtures are generated)."""
    import json
    import os
    env = os.environ.get("MINISERVE_REF")
    if env:
        return env
    base = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "BASELINE.json")
    try:
        with open(base) as f:
            return json.load(f).get("reference_path", "")
    except (OSError, ValueError):
        return ""


def load_mask_fuzz():
    """The 10^6-pair JSON mask fixture (tests/golden/make_mask_fuzz_golden.py):
    (prefixes, tokens [S, N] vocabulary ids of json_vocab(4), allowed [S, N]
    bool, raises [(state, column)])."""
    import random
    d = np.load(os.path.join(os.path.dirname(GOLDEN), "json_mask_fuzz.npz"))
    n_states, n_tokens, _, seed, V = (int(v) for v in d["meta"])
    prefixes = [str(p) for p in d["prefixes"]]
    assert len(prefixes) == n_states
    tokens = np.array([random.Random(seed + i).sample(range(V), n_tokens) for i in range(n_states)], np.int64)
    allowed = np.unpackbits(d["true_bits"], axis=1)[:, :n_tokens].astype(bool)
    return prefixes, tokens, allowed, [tuple(r) for r in d["raises"].tolist()]
