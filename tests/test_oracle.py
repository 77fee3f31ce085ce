"""The oracles against the reference's recorded answers (CPU only)."""
import math
import random

import numpy as np
import pytest

import cases
import golden_util
import oracle
from oracle import sampler_oracle as so


def test_py_sum_matches_interpreter():
    rng = np.random.default_rng(0)
    for n in (0, 1, 2, 17, 1000, 50000):
        for scale in ("uniform", "mixed", "exp"):
            if scale == "uniform":
                x = rng.random(n)
            elif scale == "mixed":
                x = rng.normal(0, 1, n) * 10.0 ** rng.integers(-12, 12, n)
            else:
                x = np.exp(-rng.random(n) * 40)
            xs = [float(v) for v in x]
            want = sum(xs)
            assert so.py_sum(xs) == want
            assert oracle.c_py_sum(x) == want


def test_kat():
    for c in cases.kat_cases():
        r = so.sample_row(c["logits"], c["temperature"], c["top_k"], c["top_p"], c["u"])
        assert r.token == c["token"]
        tok, *_ = oracle.c_sample(np.array([c["logits"]], np.float32), [c["temperature"]],
                                  [c["top_k"]], [c["top_p"]], [c["u"]])
        assert tok[0] == c["token"]


def test_python_oracle_matches_reference_small():
    g = golden_util.load()
    for entry in g["small"]:
        V = entry["V"]
        x, T, k, p, u, _ = cases.group(V, entry["case_seed"])
        assert np.array_equal(u, np.array(entry["uniforms"]))
        for b in range(x.shape[0]):
            r = so.sample_row(x[b].tolist(), T[b], k[b], p[b], u[b])
            assert r.token == golden_util.expected_token(entry["ref_tokens"][b]), (V, b)


def test_c_oracle_matches_python_oracle_small():
    g = golden_util.load()
    for entry in g["small"]:
        V = entry["V"]
        x, T, k, p, u, _ = cases.group(V, entry["case_seed"])
        for uu in (u, cases.edge_uniforms(u)):
            tok, prob, st, mp, mu = oracle.c_sample(x, T, k, p, uu, nthreads=2)
            for b in range(x.shape[0]):
                r = so.sample_row(x[b].tolist(), T[b], k[b], p[b], uu[b])
                assert tok[b] == r.token and prob[b] == r.prob, (V, b)
                assert st[b] == r.status
                assert (mp[b] == r.margin_p) or (math.isinf(mp[b]) and math.isinf(r.margin_p))
                assert (mu[b] == r.margin_u) or (math.isinf(mu[b]) and math.isinf(r.margin_u))


def test_c_oracle_matches_reference_configs():
    g = golden_util.load()
    for entry in g["configs"]:
        batch = golden_util.config_batch(entry)
        rows = entry["rows"]
        tok, prob, st, mp, mu = oracle.c_sample(batch.logits[rows], batch.temperature[rows],
                                                batch.top_k[rows], batch.top_p[rows],
                                                batch.uniforms[rows], bf16_bits=batch.bf16)
        want = [golden_util.expected_token(t) for t in entry["ref_tokens"]]
        assert tok.tolist() == want, entry["name"]
        assert np.all(prob[np.array(want) >= 0] > 0)


def test_token_only_restatement_matches_reference():
    """sample_token (the host-timed form) gives the reference's tokens."""
    for c in cases.kat_cases():
        assert so.sample_token(c["logits"], c["temperature"], c["top_k"], c["top_p"], c["u"]) == c["token"]
    g = golden_util.load()
    for entry in g["small"]:
        x, T, k, p, u, _ = cases.group(entry["V"], entry["case_seed"])
        for b in range(x.shape[0]):
            want = golden_util.expected_token(entry["ref_tokens"][b])
            got = so.sample_token(x[b].tolist(), T[b], k[b], p[b], u[b])
            assert got == (want if want >= 0 else -1), (entry["V"], b)
