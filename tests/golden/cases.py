"""Seeded small parity cases shared by the golden-fixture script and the tests.

Each group is a [B, V] float32 batch with per-row (temperature, top_k, top_p,
uniform).  The groups cover what the sampler's branches turn on: ties (values
on a coarse grid), masked entries (-inf), vocabularies that are not a multiple
of any tile (1, 7, 129, 4097, 33001), top_k at and beyond V, tiny and near-one
top_p, greedy rows, and uniforms at the ends of [0, 1).
"""
from __future__ import annotations

import random

import numpy as np

SMALL_VOCABS = (1, 2, 7, 33, 129, 1000, 4097, 33001)


def _params(rng: np.random.Generator, B: int, V: int):
    T = rng.choice(np.array([0.0, 0.05, 0.3, 0.7, 1.0, 1.7, 4.0]), B)
    k_choices = np.array([0, 0, 1, 2, 5, 20, 50, max(V - 1, 1), V, V + 3], np.int64)
    k = rng.choice(k_choices, B).astype(np.int32)
    p = rng.choice(np.array([1.0, 1.0, 0.95, 0.9, 0.5, 0.1, 1e-9, 0.999999, 1.5]), B)
    seeds = [int(s) for s in rng.integers(0, 2**31, B)]
    u = np.array([random.Random(s).random() for s in seeds])
    return T, k, p, u, seeds


def group(V: int, seed: int, B: int = 24):
    """One [B, V] group.  Row kinds rotate: gaussian, ties, masked, spiky."""
    rng = np.random.default_rng(seed * 7919 + V)
    x = np.empty((B, V), np.float32)
    for b in range(B):
        kind = b % 4
        if kind == 0:
            row = rng.normal(0.0, 2.0, V)
        elif kind == 1:   # heavy ties: values on a 0.5 grid
            row = np.round(rng.normal(0.0, 1.5, V) * 2.0) / 2.0
        elif kind == 2:   # masked entries (-inf), at least one finite value
            row = rng.normal(0.0, 1.0, V)
            drop = rng.random(V) < 0.6
            drop[rng.integers(0, V)] = False
            row[drop] = -np.inf
        else:             # a few dominant spikes
            row = rng.normal(-3.0, 1.0, V)
            row[rng.integers(0, V, 3)] += 9.0
        x[b] = row.astype(np.float32)
    T, k, p, u, seeds = _params(rng, B, V)
    return x, T, k, p, u, seeds


def edge_uniforms(u: np.ndarray) -> np.ndarray:
    """Same rows with uniforms at the ends of [0, 1): r = 0 returns index 0
    whatever its probability; r just below 1 can run past the last kept
    token and return V-1 (miniserve/sampler.py:62-68).  The reference cannot
    be seeded into these draws, so they are checked against the oracle only."""
    u = u.copy()
    u[0::3] = 0.0
    u[1::3] = 1.0 - 2.0**-53
    return u


def kat_cases():
    """Known answers.  The first is the reference's own test
    (tests/test_server.py:302-305); the second is a tie probe: first maximal
    index wins (miniserve/sampler.py:34)."""
    return [
        dict(logits=[0.1, 0.5, 0.9, 0.2], temperature=0.0, top_k=0, top_p=1.0, u=0.5, token=2),
        dict(logits=[1.0, 3.0, 3.0, 2.0], temperature=0.0, top_k=0, top_p=1.0, u=0.5, token=1),
    ]
