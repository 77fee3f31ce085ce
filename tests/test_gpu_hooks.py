"""The logits-processor hook adapter (miniserve/model_runner.py:166-168,
214-216) on the GPU: the packed mask against the hook's -inf convention, the
greedy drop-in against torch.argmax of the hook's output, and sampling under
the hook against the oracle."""
import numpy as np
import pytest

from parity import compare

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _hook(seed):
    """A hook in miniserve's form: bans a seeded random set of tokens (-inf)
    that depends on the generated tokens."""
    def fn(logits, generated):
        g = torch.Generator().manual_seed(seed + len(generated) + (generated[-1] if generated else 0))
        banned = torch.rand(logits.shape[0], generator=g) < 0.3
        out = logits.clone()
        out[banned.to(logits.device)] = float("-inf")
        return out
    return fn


def _pack(allowed):
    """Bit j of word w = allowed[32 w + j] (the sampler's mask layout)."""
    B, V = allowed.shape
    W = (V + 31) // 32
    padded = np.zeros((B, W * 32), np.uint64)
    padded[:, :V] = allowed
    return (padded.reshape(B, W, 32) << np.arange(32, dtype=np.uint64)).sum(-1).astype(np.uint32)


@pytest.mark.parametrize("V", [1, 31, 32, 33, 5000, 151936])
@pytest.mark.parametrize("bf16", [False, True])
def test_allowed_mask_matches_hook_convention(V, bf16):
    from miniserve_b200.hooks import allowed_mask
    rng = np.random.default_rng(V)
    B = 5
    x = rng.normal(0, 2, (B, V)).astype(np.float32)
    x[rng.random((B, V)) < 0.4] = -np.inf
    x[0, : min(V, 3)] = np.nan  # allowed (flagged by the sampler, not masked)
    t = torch.from_numpy(x).cuda()
    if bf16:
        t = t.to(torch.bfloat16)
    buf = torch.zeros((B, V + 7), dtype=t.dtype, device="cuda")  # row stride > V
    buf[:, :V] = t
    got = allowed_mask(buf[:, :V]).cpu().numpy().view(np.uint32)
    want = _pack(~np.isneginf(x))
    assert got.shape == want.shape and np.array_equal(got, want)


def test_greedy_dropin_equals_argmax_of_hook_output():
    from miniserve_b200.hooks import HookAdapter
    rng = np.random.default_rng(3)
    fn = _hook(11)
    ad = HookAdapter(fn)
    for i in range(6):
        V = [151936, 4096, 777][i % 3]
        x = rng.normal(0, 2, V).astype(np.float32)
        if i % 2:
            x[rng.choice(V, 4, replace=False)] = x.max()  # ties: the first index wins
        logits = torch.from_numpy(x).cuda()
        generated = [int(t) for t in rng.integers(0, V, i)]  # miniserve's List[int]
        assert ad.greedy(logits, generated) == int(fn(logits, generated).argmax())


def test_sampling_under_hook_matches_oracle():
    from miniserve_b200.hooks import HookAdapter
    rng = np.random.default_rng(5)
    B, V = 12, 151936
    x = rng.normal(0, 2, (B, V)).astype(np.float32)
    T = rng.choice([0.0, 0.7, 1.0], B)
    K = rng.choice([0, 20, 50], B).astype(np.int32)
    P = rng.choice([1.0, 0.9], B)
    U = rng.random(B)
    generated = [[int(t) for t in rng.integers(0, V, b % 4)] for b in range(B)]
    ad = HookAdapter(_hook(21))
    logits = torch.from_numpy(x).cuda()
    mask = ad.mask(logits, generated)
    tok, prob, st = ad.sample_batch(logits, generated, temperature=T, top_k=K, top_p=P, uniforms=U)
    torch.cuda.synchronize()
    m = mask.cpu().numpy().view(np.uint32)
    compare(tok.cpu().numpy(), prob.cpu().numpy().astype(np.float64), st.cpu().numpy(), x, T, K, P, U, mask=m,
            label="sampling under a hook")
    processed = ad.processed(logits, generated).cpu().numpy()
    allowed = ~np.isneginf(processed)
    assert all(allowed[b, tok[b]] for b in range(B) if st[b] == 0)
