"""Parity of the CUDA sampler (through the C ABI) with the oracle and the
reference's recorded tokens.  Needs a B200."""
import numpy as np
import pytest

import cases
import golden_util
from parity import compare, gpu_sample

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=["fast", "generic"])
def sampler(request):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from miniserve_b200 import Sampler
    return Sampler(request.param)


def test_kat(sampler):
    for c in cases.kat_cases():
        tok, prob, st = gpu_sample(sampler, np.array([c["logits"]], np.float32), [c["temperature"]],
                                   [c["top_k"]], [c["top_p"]], [c["u"]])
        assert tok[0] == c["token"]
        assert sampler.sample(c["logits"], temperature=c["temperature"]) == c["token"]


@pytest.mark.parametrize("V", cases.SMALL_VOCABS)
def test_small_groups_vs_reference_and_oracle(sampler, V):
    g = golden_util.load()
    entry = next(e for e in g["small"] if e["V"] == V)
    x, T, K, P, U, _ = cases.group(V, entry["case_seed"])
    tok, prob, st = gpu_sample(sampler, x, T, K, P, U)
    compare(tok, prob, st, x, T, K, P, U, label=f"small V={V}")
    want = np.array([golden_util.expected_token(t) for t in entry["ref_tokens"]])
    from oracle import c_sample
    _, _, _, mp, mu = c_sample(x, T, K, P, U)
    strict = (mp >= 1e-6) & (mu >= 1e-6)
    assert np.array_equal(tok[strict], want[strict])


@pytest.mark.parametrize("V", cases.SMALL_VOCABS)
def test_small_groups_edge_uniforms(sampler, V):
    x, T, K, P, U, _ = cases.group(V, 11)
    U = cases.edge_uniforms(U)
    tok, prob, st = gpu_sample(sampler, x, T, K, P, U)
    compare(tok, prob, st, x, T, K, P, U, label=f"edge-u V={V}")


@pytest.mark.parametrize("name", ["config1", "config1_greedy", "config2_fp32", "config2_bf16",
                                  "config3", "config5"])
def test_config_rows_vs_reference(sampler, name):
    g = golden_util.load()
    entry = next(e for e in g["configs"] if e["name"] == name)
    batch = golden_util.config_batch(entry)
    rows = entry["rows"]
    x = batch.logits[rows]
    tok, prob, st = gpu_sample(sampler, x, batch.temperature[rows], batch.top_k[rows],
                               batch.top_p[rows], batch.uniforms[rows], bf16=batch.bf16)
    compare(tok, prob, st, x, batch.temperature[rows], batch.top_k[rows], batch.top_p[rows],
            batch.uniforms[rows], bf16=batch.bf16, label=name)
    want = np.array([golden_util.expected_token(t) for t in entry["ref_tokens"]])
    from oracle import c_sample
    _, _, _, mp, mu = c_sample(x, batch.temperature[rows], batch.top_k[rows], batch.top_p[rows],
                               batch.uniforms[rows], bf16_bits=batch.bf16)
    strict = (mp >= 1e-6) & (mu >= 1e-6)
    assert np.array_equal(tok[strict], want[strict]), (tok, want)


@pytest.mark.parametrize("bf16", [False, True])
def test_pair_mode_batches(sampler, bf16):
    """Batches of at most one row per SM run the streaming kernel as clusters
    of two CTAs: top-p rows are shared by both CTAs (each streams half the
    row), the other rows go two to a cluster.  A mixed batch, and a batch of
    top-p-only rows at high temperature (large brackets), against the oracle."""
    from miniserve_b200 import workloads
    b = workloads.config3(3)
    x = b.logits[:140]
    if bf16:
        x = (x.view(np.uint32) >> 16).astype(np.uint16)  # truncated to bf16 bits
    tok, prob, st = gpu_sample(sampler, x, b.temperature[:140], b.top_k[:140], b.top_p[:140],
                               b.uniforms[:140], bf16=bf16)
    compare(tok, prob, st, x, b.temperature[:140], b.top_k[:140], b.top_p[:140], b.uniforms[:140],
            bf16=bf16, label="pair mode mixed B=140")
    rng = np.random.default_rng(9)
    T = 1.0 + 0.5 * rng.random(96)
    K = np.zeros(96, np.int32)
    P = 0.6 + 0.39 * rng.random(96)
    xr = b.logits[200:296]
    if bf16:
        xr = (xr.view(np.uint32) >> 16).astype(np.uint16)
    tok, prob, st = gpu_sample(sampler, xr, T, K, P, b.uniforms[200:296], bf16=bf16)
    compare(tok, prob, st, xr, T, K, P, b.uniforms[200:296], bf16=bf16, label="pair mode top-p B=96")


def test_config3_full_batch(sampler):
    from miniserve_b200 import workloads
    b = workloads.config3(3)
    tok, prob, st = gpu_sample(sampler, b.logits, b.temperature, b.top_k, b.top_p, b.uniforms)
    compare(tok, prob, st, b.logits, b.temperature, b.top_k, b.top_p, b.uniforms, label="config3 B=512")


def test_config2_full_batch_bf16(sampler):
    from miniserve_b200 import workloads
    b = workloads.config2(2, bf16=True)
    tok, prob, st = gpu_sample(sampler, b.logits, b.temperature, b.top_k, b.top_p, b.uniforms, bf16=True)
    compare(tok, prob, st, b.logits, b.temperature, b.top_k, b.top_p, b.uniforms, bf16=True,
            label="config2 bf16 B=256")


def test_masked_rows(sampler):
    rng = np.random.default_rng(7)
    B, V = 48, 5000
    x = rng.normal(0, 2, (B, V)).astype(np.float32)
    W = (V + 31) // 32
    mask = rng.integers(0, 2**32, (B, W), dtype=np.uint64).astype(np.uint32)
    mask[0] = 0                      # everything masked: ZeroDivisionError row
    mask[1] = 0
    mask[1, 3] = 1 << 5              # exactly one allowed token
    T = rng.choice([0.0, 0.5, 1.0], B)
    T[0] = 1.0
    K = rng.choice([0, 3, 40], B).astype(np.int32)
    P = rng.choice([1.0, 0.9, 0.3], B)
    U = rng.random(B)
    tok, prob, st = gpu_sample(sampler, x, T, K, P, U, mask=mask)
    compare(tok, prob, st, x, T, K, P, U, mask=mask, label="masked")
    assert tok[0] == -1 and st[0] == 1
    assert tok[1] == 3 * 32 + 5


def test_nonfinite_and_bad_temperature_status(sampler):
    x = np.zeros((4, 64), np.float32)
    x[0, 5] = np.nan
    x[1, 7] = np.inf
    T = np.array([1.0, 0.0, -1.0, np.nan])
    tok, prob, st = gpu_sample(sampler, x, T, np.zeros(4, np.int32), np.ones(4), np.full(4, 0.5))
    assert st[0] & 4 and st[1] & 4
    assert tok[1] == 7
    assert st[2] & 2 and st[3] & 2 and tok[2] == -1 and tok[3] == -1


def test_argument_errors(sampler):
    import torch
    from miniserve_b200 import _lib
    L = _lib.lib()
    x = torch.zeros(2, 8, device="cuda")
    bad = L.ms_sample(x.data_ptr(), 7, 2, 8, 8, None, None, None, None, None, 0, None, None, None, None)
    assert bad == -2
    bad = L.ms_sample(x.data_ptr(), 0, 2, 8, 4, None, None, None, None, None, 0, None, None, None, None)
    assert bad == -1
    with pytest.raises(ZeroDivisionError):
        sampler.sample([float("-inf")] * 4, temperature=1.0)
