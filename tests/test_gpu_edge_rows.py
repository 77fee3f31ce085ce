"""Full-vocabulary rows that drive every branch of the streaming kernel:
top-k buffer compaction and tie overflow, the top-p high list and its
fallback histogram pass, masked first chunk, extreme top_p / temperature /
uniforms, top_k at and past the streaming limit, unaligned rows (no TMA), and
bf16.  Each batch is checked against the C oracle (float64 restatement of
miniserve/sampler.py:23-68) row by row.  Needs a B200."""
import numpy as np
import pytest

from parity import compare, gpu_sample

pytestmark = pytest.mark.gpu

V = 151936


@pytest.fixture(scope="module", params=["fast", "generic"])
def sampler(request):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from miniserve_b200 import Sampler
    return Sampler(request.param)


def _zipf(rng, n=V):
    base = -1.1 * np.log(np.arange(1, n + 1, dtype=np.float64))
    return (base[rng.permutation(n)] + rng.normal(0.0, 0.5, n)).astype(np.float32)


def edge_batch(seed=11):
    """(logits [B, V] f32, T, K, P, U, mask [B, W] u32, labels)."""
    rng = np.random.default_rng(seed)
    rows, T, K, P, U, labels = [], [], [], [], [], []
    W = (V + 31) // 32
    masks = []

    def add(x, t, k, p, u, label, mask=None):
        rows.append(x.astype(np.float32))
        T.append(t), K.append(k), P.append(p), U.append(u), labels.append(label)
        masks.append(np.full(W, 0xFFFFFFFF, np.uint32) if mask is None else mask)

    asc = np.linspace(-5.0, 5.0, V, dtype=np.float32)
    add(asc, 1.0, 50, 1.0, 0.37, "ascending top-k 50 (buffer compaction every chunk)")
    add(asc, 0.5, 0, 0.9, 0.61, "ascending top-p (high list overflows -> fallback pass)")
    add(asc[::-1].copy(), 1.0, 200, 0.8, 0.52, "descending top-k 200 + top-p")
    add(asc[::-1].copy(), 0.3, 0, 0.9, 0.44, "descending top-p")
    const = np.ones(V, np.float32)
    add(const, 1.0, 50, 1.0, 0.5071, "constant row top-k (tie block past the buffer)")
    add(const, 1.0, 0, 0.5013, 0.5137, "constant row top-p (one crowded bin)")
    add(const, 1.0, 0, 1.0, 0.2513, "constant row full softmax")
    m = np.full(W, 0xFFFFFFFF, np.uint32)
    m[: 4096 // 32] = 0
    add(_zipf(rng), 0.8, 0, 0.9, 0.3, "first chunk masked (no anchor) top-p", m)
    add(_zipf(rng), 0.8, 0, 1e-12, 0.7, "top_p ~ 0: only the maximum")
    add(_zipf(rng), 1.5, 0, 0.9999999, 0.9, "top_p ~ 1")
    add(_zipf(rng), 1e-3, 0, 0.9, 0.5, "temperature 1e-3 top-p")
    add(_zipf(rng), 1e-31, 0, 0.9, 0.5, "temperature below the fp32 weight range")
    add(_zipf(rng), 1e4, 0, 0.5, 0.4761, "temperature 1e4 top-p")
    add(_zipf(rng), 0.9, 256, 1.0, 0.81, "top_k 256 (streaming limit)")
    add(_zipf(rng), 0.9, 300, 0.95, 0.33, "top_k 300")
    add(_zipf(rng), 1.1, 512, 0.9, 0.66, "top_k 512 (streaming limit)")
    add(_zipf(rng), 1.1, 513, 0.9, 0.66, "top_k 513 (generic kernel)")
    add(_zipf(rng), 0.9, 257, 0.95, 0.19, "top_k 257 (generic kernel)")
    add(_zipf(rng), 0.9, V - 1, 0.9, 0.33, "top_k V-1")
    q = np.round(_zipf(rng) * 20.0) / 20.0
    add(q, 0.7, 0, 0.9, 0.66, "quantised values (many exact ties) top-p")
    add(q, 0.7, 20, 0.9, 0.14, "quantised values top-k 20")
    add(_zipf(rng), 0.7, 0, 1.0, 0.999999, "full softmax, uniform near 1")
    add(_zipf(rng), 0.7, 0, 0.9, 0.0, "top-p, uniform 0")
    add(_zipf(rng), 0.7, 50, 0.9, 0.0, "top-k, uniform 0")
    spike = _zipf(rng)
    spike[V - 1] = 25.0
    add(spike, 1.0, 0, 0.9, 0.5, "top-p, dominant token in the last chunk (high list)")
    many = _zipf(rng)
    many[rng.choice(np.arange(8192, V), 400, replace=False)] = 12.0
    add(many, 1.0, 0, 0.911, 0.5, "top-p, 400 far-above values after chunk 0 (fallback)")
    add(_zipf(rng), 0.6, 0, 0.75, 0.5, "plain top-p")
    add(_zipf(rng), 0.6, 0, 0.75, 0.5, "plain top-p (second row)")
    x = np.stack(rows)
    return (x, np.array(T), np.array(K, np.int32), np.array(P), np.array(U), np.stack(masks), labels)


def test_edge_rows_fp32(sampler):
    x, T, K, P, U, mask, labels = edge_batch()
    tok, prob, st = gpu_sample(sampler, x, T, K, P, U, mask=mask)
    compare(tok, prob, st, x, T, K, P, U, mask=mask, label="edge rows fp32")
    # rows whose margins are zero by construction, checked on their own terms
    for i, lab in enumerate(labels):
        if "uniform 0" in lab:  # r == 0 stops at index 0 (miniserve/sampler.py:66)
            assert tok[i] == 0, lab
        if lab.startswith("top_p ~ 0"):  # the first sorted element alone reaches top_p
            assert tok[i] == int(np.argmax(x[i])) and abs(prob[i] - 1.0) < 1e-6, lab


def test_edge_rows_bf16(sampler):
    x, T, K, P, U, mask, labels = edge_batch(seed=12)
    bits = (x.view(np.uint32) >> 16).astype(np.uint16)
    xb = (bits.astype(np.uint32) << 16).view(np.float32)  # the exact bf16 values
    tok, prob, st = gpu_sample(sampler, xb, T, K, P, U, mask=mask)
    compare(tok, prob, st, xb, T, K, P, U, mask=mask, label="edge rows (bf16 values, fp32 storage)")
    import torch
    xt = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    mt = torch.from_numpy(mask.view(np.int32)).cuda()
    t2, p2, s2 = sampler.sample_batch(xt, T, K, P, uniforms=U, mask=mt)
    torch.cuda.synchronize()
    compare(t2.cpu().numpy(), p2.cpu().numpy().astype(np.float64), s2.cpu().numpy(), xb, T, K, P, U,
            mask=mask, label="edge rows bf16")


def test_unaligned_rows(sampler):
    """Row stride V+1 floats: rows after the first start off the 16-byte grid,
    so the kernel reads them without TMA."""
    import torch
    x, T, K, P, U, mask, labels = edge_batch(seed=13)
    B = x.shape[0]
    buf = torch.zeros(B, V + 1, dtype=torch.float32, device="cuda")
    buf[:, :V] = torch.from_numpy(x).cuda()
    view = buf[:, :V]
    assert view.stride(0) == V + 1
    mt = torch.from_numpy(mask.view(np.int32)).cuda()
    tok, prob, st = sampler.sample_batch(view, T, K, P, uniforms=U, mask=mt)
    torch.cuda.synchronize()
    compare(tok.cpu().numpy(), prob.cpu().numpy().astype(np.float64), st.cpu().numpy(), x, T, K, P, U,
            mask=mask, label="unaligned rows")
