"""Sampling as the last launches of a captured decode graph, reading the
graph's static logits buffer in place (the ``_out`` of miniserve's
GraphedDecodeRunner, miniserve/model_runner.py:224-321, without the clone at
:321).  The decode step here has the runner's buffer structure -- bucketed
graphs, two alternating input sets, one static [max_batch, V] fp32 output --
with an embedding and an fp32 LM head standing in for the model.  Needs a
B200."""
import numpy as np
import pytest

from parity import compare

pytestmark = pytest.mark.gpu

BUCKETS = (1, 2, 4, 8, 16, 32)


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    if not t.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return t


class _Decode:
    """Static-buffer decode step: ids -> embedding -> fp32 LM head -> _out."""

    def __init__(self, torch, V=151936, d=64, vin=1000, max_batch=32, seed=0):
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.torch = torch
        self.emb = torch.randn(vin, d, generator=g).cuda()
        self.head = (torch.randn(V, d, generator=g) * 0.6).cuda()
        self.ids = [torch.zeros(max_batch, dtype=torch.long, device="cuda") for _ in range(2)]
        self._out = torch.zeros(max_batch, V, dtype=torch.float32, device="cuda")
        self.max_batch = max_batch

    def run_static(self, s, bucket):
        self._out[:bucket] = self.emb[self.ids[s][:bucket]] @ self.head.T


def _capture(torch, dec, gs, bucket, s):
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):  # warm the step's kernels outside the capture
        dec.run_static(s, bucket)
    torch.cuda.current_stream().wait_stream(st)
    with torch.cuda.graph(g):
        dec.run_static(s, bucket)
        gs.enqueue(bucket)
    return g


def _params(B, seed):
    rng = np.random.default_rng(seed)
    T = rng.uniform(0.2, 1.5, B)
    T[rng.random(B) < 0.2] = 0.0
    K = rng.choice([0, 1, 20, 50, 200], B).astype(np.int32)
    P = rng.uniform(0.5, 1.0, B)
    P[rng.random(B) < 0.3] = 1.0
    U = rng.random(B)
    return T, K, P, U


def test_graph_samples_static_buffer_in_place(torch):
    from miniserve_b200 import Sampler
    from miniserve_b200.graphed import GraphedSampler
    dec = _Decode(torch)
    gs = GraphedSampler(dec._out)
    assert gs.logits.data_ptr() == dec._out.data_ptr()
    graphs = {}
    rng = np.random.default_rng(5)
    step = 0
    for B in (3, 8, 17, 32, 1, 32, 9):
        bucket = next(b for b in BUCKETS if b >= B)
        s = step % 2
        step += 1
        if (bucket, s) not in graphs:
            graphs[(bucket, s)] = _capture(torch, dec, gs, bucket, s)
        ids = rng.integers(0, 1000, dec.max_batch)
        dec.ids[s].copy_(torch.from_numpy(ids))
        T, K, P, U = _params(B, 100 + step)
        gs.set_params(B, temperature=T.tolist(), top_k=K.tolist(), top_p=P.tolist(), uniforms=U.tolist())
        graphs[(bucket, s)].replay()
        torch.cuda.synchronize()
        tok, prob, st = (t.cpu().numpy() for t in gs.result(B))
        logits = dec._out[:B].cpu().numpy()
        compare(tok, prob.astype(np.float64), st, logits, T, K, P, U, label=f"graphed B={B}")
        # the same tokens as the eager call on a copy of the logits
        t2, p2, s2 = Sampler().sample_batch(dec._out[:B].clone(), T, K, P, uniforms=U)
        assert np.array_equal(tok, t2.cpu().numpy())
        assert np.array_equal(st, s2.cpu().numpy())
        assert gs.tokens(B) == tok.tolist()


def test_graph_with_mask_and_seeds(torch):
    from miniserve_b200.graphed import GraphedSampler
    from miniserve_b200.sampler import uniform_for_seed
    dec = _Decode(torch, V=50000, seed=3)
    gs = GraphedSampler(dec._out, with_mask=True)
    g = _capture(torch, dec, gs, 8, 0)
    B = 6
    rng = np.random.default_rng(11)
    dec.ids[0].copy_(torch.from_numpy(rng.integers(0, 1000, dec.max_batch)))
    W = (50000 + 31) // 32
    bits = rng.integers(0, 2**32, (B, W), dtype=np.uint64).astype(np.uint32)
    bits[2] &= np.uint32(0x01010101)  # a sparse row
    gs.set_mask(torch.from_numpy(bits.view(np.int32)).cuda())
    seeds = [7, 8, 9, 10, 11, 12]
    gs.set_params(B, temperature=0.8, top_k=[0, 50, 0, 20, 0, 1], top_p=[0.9, 1.0, 0.95, 0.8, 1.0, 1.0],
                  seeds=seeds)
    g.replay()
    torch.cuda.synchronize()
    tok, prob, st = (t.cpu().numpy() for t in gs.result(B))
    U = np.array([uniform_for_seed(s) for s in seeds])
    compare(tok, prob.astype(np.float64), st, dec._out[:B].cpu().numpy(), np.full(B, 0.8),
            np.array([0, 50, 0, 20, 0, 1], np.int32), np.array([0.9, 1.0, 0.95, 0.8, 1.0, 1.0]), U,
            mask=bits, label="graphed mask")


def test_eager_enqueue_and_argument_checks(torch):
    from miniserve_b200.graphed import GraphedSampler
    dec = _Decode(torch, V=4096, seed=4)
    gs = GraphedSampler(dec._out)
    dec.ids[0].copy_(torch.arange(dec.max_batch, device="cuda"))
    dec.run_static(0, 4)
    gs.set_params(3, temperature=0.0)
    gs.enqueue(4)
    torch.cuda.synchronize()
    want = dec._out[:3].argmax(dim=1).cpu().tolist()
    assert gs.tokens(3) == want
    with pytest.raises(ValueError):
        gs.set_params(33)
    with pytest.raises(ValueError):
        gs.enqueue(0)
    with pytest.raises(ValueError):
        gs.set_params(2, top_k=[1, 2, 3])
    with pytest.raises(RuntimeError):
        gs.set_mask(torch.zeros(1, 128, dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError):
        GraphedSampler(dec._out.t())
