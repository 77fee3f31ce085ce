"""Vocab-sharded sampling on the GPU, checked against the oracle on the full
rows.  On one GPU the ranks are emulated: each slice's candidate records come
from ms_shard_candidates, are stacked rank-major (what the all-gather
produces) and merged with ms_shard_merge.  With two or more GPUs the NCCL
path runs under torchrun (tests/mp_sharded.py).  Needs a B200."""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle
from parity import compare

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    if not t.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return t


def emulate(torch, x, T, K, P, U, world, bf16=False, mask=None):
    """Tokens of the sharded path with `world` ranks emulated on one GPU."""
    from miniserve_b200 import _lib, sharded
    L = _lib.lib()
    B, V = x.shape
    kmax = sharded.choose_kmax(list(K), list(T), list(P), V)
    W = sharded.record_words(kmax)
    xt = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    if bf16:
        xt = xt.to(torch.bfloat16)
    dev = xt.device
    Tt = torch.tensor(T, dtype=torch.float64, device=dev)
    Kt = torch.tensor(K, dtype=torch.int32, device=dev)
    Pt = torch.tensor(P, dtype=torch.float64, device=dev)
    Ut = torch.tensor(U, dtype=torch.float64, device=dev)
    recs = torch.empty((world, B, W), dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    for r in range(world):
        v0, v1 = sharded.shard_bounds(V, world, r)
        part = xt[:, v0:v1]
        mptr, mld = None, 0
        if mask is not None:
            assert v0 % 32 == 0
            mt = torch.from_numpy(np.ascontiguousarray(mask[:, v0 // 32:(v1 + 31) // 32]).view(np.int32)).cuda()
            mptr, mld = mt.data_ptr(), mt.stride(0)
        rc = L.ms_shard_candidates(part.data_ptr(), 1 if bf16 else 0, B, v1 - v0, part.stride(0), v0, V,
                                   Tt.data_ptr(), Kt.data_ptr(), mptr, mld, kmax, recs[r].data_ptr(), s)
        assert rc == 0
        torch.cuda.synchronize()
    tok = torch.empty(B, dtype=torch.int64, device=dev)
    prob = torch.empty(B, dtype=torch.float32, device=dev)
    st = torch.empty(B, dtype=torch.int32, device=dev)
    rc = L.ms_shard_merge(recs.data_ptr(), world, B, kmax, V, Tt.data_ptr(), Kt.data_ptr(), Pt.data_ptr(),
                          Ut.data_ptr(), tok.data_ptr(), prob.data_ptr(), st.data_ptr(), s)
    assert rc == 0
    torch.cuda.synchronize()
    return tok.cpu().numpy(), prob.cpu().numpy().astype(np.float64), st.cpu().numpy()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config5_rows_emulated(torch, world):
    from miniserve_b200 import workloads
    b = workloads.config5(5, B=64)
    tok, prob, st = emulate(torch, b.logits, b.temperature, b.top_k, b.top_p, b.uniforms, world)
    compare(tok, prob, st, b.logits, b.temperature, b.top_k, b.top_p, b.uniforms, label=f"config5 x{world}")


def _mixed(seed=9, B=48, V=65536):
    rng = np.random.default_rng(seed)
    base = -1.1 * np.log(np.arange(1, V + 1, dtype=np.float64))
    x = np.stack([(base[rng.permutation(V)] + rng.normal(0, 0.5, V)).astype(np.float32) for _ in range(B)])
    x[5, 40000:40100] = x[5].max() + 1.0   # a tie block of maxima across a slice edge
    x[6, :] = -np.inf                        # every logit masked
    T = rng.choice([0.0, 0.8, 1.2], B)
    K = rng.choice([1, 2, 20, 50, 200], B).astype(np.int32)
    P = rng.choice([0.95, 0.6, 1.0], B)
    U = rng.random(B)
    T[6] = 0.0
    U[7] = 0.0
    return x, T, K, P, U


@pytest.mark.parametrize("world", [2, 8])
def test_mixed_rows_emulated(torch, world):
    x, T, K, P, U = _mixed()
    tok, prob, st = emulate(torch, x, T, K, P, U, world)
    compare(tok, prob, st, x, T, K, P, U, label=f"mixed x{world}")


def test_bf16_and_mask_emulated(torch):
    x, T, K, P, U = _mixed(seed=10)
    xb = ((x.view(np.uint32) >> 16).astype(np.uint32) << 16).view(np.float32)
    rng = np.random.default_rng(3)
    mask = rng.integers(0, 2**32, (x.shape[0], x.shape[1] // 32), dtype=np.uint64).astype(np.uint32)
    tok, prob, st = emulate(torch, xb, T, K, P, U, 4, bf16=True, mask=mask)
    compare(tok, prob, st, xb, T, K, P, U, mask=mask, label="bf16 + mask x4")


def test_unsupported_rows_flagged_and_finished(torch):
    """top_k off with top_p 1, top_k above 256: the merge flags them;
    ShardedSampler finishes them from the full row (world 1 here: the gather is
    the identity)."""
    from miniserve_b200.sharded import ShardedSampler
    x, T, K, P, U = _mixed(seed=11, B=16)
    K[:4] = [0, 0, 300, 0]
    T[:4] = [0.9, 1.1, 0.7, 0.5]
    P[:4] = [1.0, 1.0, 0.9, 1.0]
    tok, prob, st = emulate(torch, x, T, K, P, U, 2)
    assert (st[:4] & 8).all() and (tok[:4] == -1).all()
    s = ShardedSampler(x.shape[1])
    t2, p2, s2 = s.sample(torch.from_numpy(x).cuda(), 0, T, K, P, uniforms=U)
    torch.cuda.synchronize()
    compare(t2.cpu().numpy(), p2.cpu().numpy().astype(np.float64), s2.cpu().numpy(), x, T, K, P, U,
            label="sharded sampler with fallback rows")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_nucleus_rows_from_records(torch, world):
    """Top-p rows without top-k: settled by the merge from the candidates and
    the slices' totals when the nucleus lies among the candidates (most low-
    and mid-temperature rows), flagged otherwise; every settled row matches
    the oracle on the full row, and ShardedSampler finishes the rest."""
    from miniserve_b200.sharded import ShardedSampler
    rng = np.random.default_rng(21)
    B, V = 64, 65536
    base = -1.1 * np.log(np.arange(1, V + 1, dtype=np.float64))
    x = np.stack([(base[rng.permutation(V)] + rng.normal(0, 0.5, V)).astype(np.float32) for _ in range(B)])
    T = rng.choice([0.2, 0.4, 0.7, 1.0, 1.4], B)
    K = np.zeros(B, np.int32)
    K[::9] = V + 5  # top_k at or above the vocabulary: off as well
    P = 0.5 + 0.49 * rng.random(B)
    U = rng.random(B)
    U[3] = 0.0
    tok, prob, st = emulate(torch, x, T, K, P, U, world)
    settled = st == 0
    assert settled.sum() >= B // 2, settled.sum()
    assert np.all(st[~settled] == 8) and np.all(tok[~settled] == -1)
    r = np.nonzero(settled)[0]
    compare(tok[r], prob[r], st[r], x[r], T[r], K[r], P[r], U[r], label=f"nucleus from records x{world}")
    if world == 2:
        s = ShardedSampler(V)
        t2, p2, s2 = s.sample(torch.from_numpy(x).cuda(), 0, T, K, P, uniforms=U)
        torch.cuda.synchronize()
        compare(t2.cpu().numpy(), p2.cpu().numpy().astype(np.float64), s2.cpu().numpy(), x, T, K, P, U,
                label="sharded sampler, nucleus rows")


def emulate_nucleus(torch, x, T, K, P, U, world):
    """The merge, then the distributed nucleus for the rows it flags, with
    `world` ranks emulated on one GPU: the histogram all-reduce is a sum over
    the ranks' histograms, the entries all-gather a stack, the token all-reduce
    a maximum.  Returns (tokens, probs, status, rows the nucleus finished)."""
    from miniserve_b200 import _lib, sharded
    L = _lib.lib()
    B, V = x.shape
    kmax = sharded.choose_kmax(list(K), list(T), list(P), V)
    W = sharded.record_words(kmax)
    xt = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    dev = xt.device
    Tt = torch.tensor(T, dtype=torch.float64, device=dev)
    Kt = torch.tensor(K, dtype=torch.int32, device=dev)
    Pt = torch.tensor(P, dtype=torch.float64, device=dev)
    Ut = torch.tensor(U, dtype=torch.float64, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    recs = torch.empty((world, B, W), dtype=torch.int32, device=dev)
    bnd = [sharded.shard_bounds(V, world, r) for r in range(world)]
    for r, (v0, v1) in enumerate(bnd):
        part = xt[:, v0:v1]
        assert L.ms_shard_candidates(part.data_ptr(), 0, B, v1 - v0, part.stride(0), v0, V, Tt.data_ptr(),
                                     Kt.data_ptr(), None, 0, kmax, recs[r].data_ptr(), s) == 0
    tok = torch.empty(B, dtype=torch.int64, device=dev)
    prob = torch.empty(B, dtype=torch.float32, device=dev)
    st = torch.empty(B, dtype=torch.int32, device=dev)
    assert L.ms_shard_merge(recs.data_ptr(), world, B, kmax, V, Tt.data_ptr(), Kt.data_ptr(), Pt.data_ptr(),
                            Ut.data_ptr(), tok.data_ptr(), prob.data_ptr(), st.data_ptr(), s) == 0
    nuc = ((st & 8) != 0) & ((Kt <= 0) | (Kt >= V))
    rows = nuc.nonzero().flatten().to(torch.int32).contiguous()
    F = int(rows.numel())
    if F:
        NB, RW, CW = (int(L.ms_nucleus_hist_words()), int(L.ms_nucleus_record_words()),
                      int(L.ms_nucleus_cut_words()))
        hist = torch.zeros((F, NB), dtype=torch.int32, device=dev)
        for r, (v0, v1) in enumerate(bnd):
            h = torch.empty((F, NB), dtype=torch.int32, device=dev)
            part = xt[:, v0:v1]
            assert L.ms_nucleus_hist(part.data_ptr(), 0, v1 - v0, part.stride(0), None, 0, rows.data_ptr(), F, B, V,
                                     recs.data_ptr(), world, kmax, Tt.data_ptr(), Pt.data_ptr(), h.data_ptr(),
                                     s) == 0
            hist += h
        bracket = torch.empty((F, 2), dtype=torch.int32, device=dev)
        assert L.ms_nucleus_bracket(hist.data_ptr(), rows.data_ptr(), F, V, Pt.data_ptr(), bracket.data_ptr(),
                                    s) == 0
        ent = torch.empty((world, F, RW), dtype=torch.int32, device=dev)
        segs = torch.empty((world, F, int(L.ms_nucleus_segments())), dtype=torch.float64, device=dev)
        for r, (v0, v1) in enumerate(bnd):
            part = xt[:, v0:v1]
            assert L.ms_nucleus_classify(part.data_ptr(), 0, v1 - v0, part.stride(0), v0, None, 0, rows.data_ptr(),
                                         F, B, recs.data_ptr(), world, kmax, Tt.data_ptr(), bracket.data_ptr(),
                                         ent[r].data_ptr(), segs[r].data_ptr(), s) == 0
        bounds = torch.tensor([a for a, _ in bnd] + [V], dtype=torch.int64, device=dev)
        cut = torch.empty((F, CW), dtype=torch.int32, device=dev)
        assert L.ms_nucleus_cut(ent.data_ptr(), world, bounds.data_ptr(), bracket.data_ptr(), rows.data_ptr(), F, B,
                                recs.data_ptr(), kmax, Tt.data_ptr(), Pt.data_ptr(), Ut.data_ptr(), cut.data_ptr(),
                                s) == 0
        out = torch.full((F, 2), -1, dtype=torch.int64, device=dev)
        for r, (v0, v1) in enumerate(bnd):
            o = torch.empty((F, 2), dtype=torch.int64, device=dev)
            part = xt[:, v0:v1]
            assert L.ms_nucleus_draw(part.data_ptr(), 0, v1 - v0, part.stride(0), v0, None, 0, rows.data_ptr(), F,
                                     B, recs.data_ptr(), world, kmax, Tt.data_ptr(), cut.data_ptr(), ent.data_ptr(),
                                     segs[r].data_ptr(), r, o.data_ptr(), s) == 0
            out = torch.maximum(out, o)
        done = (cut[:, 3] == 0) & (out[:, 0] >= 0)
        r = rows.long()[done]
        tok[r] = out[done, 0]
        prob[r] = out[done, 1].to(torch.int32).view(torch.float32)
        st[r] = 0
        finished = r.cpu().numpy()
    else:
        finished = np.zeros(0, np.int64)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), prob.cpu().numpy().astype(np.float64), st.cpu().numpy(), finished


def _wide_rows(seed, B, V):
    rng = np.random.default_rng(seed)
    base = -1.1 * np.log(np.arange(1, V + 1, dtype=np.float64))
    x = np.stack([(base[rng.permutation(V)] + rng.normal(0, 0.5, V)).astype(np.float32) for _ in range(B)])
    x[B // 2:] = rng.normal(0.0, 2.0, (B - B // 2, V)).astype(np.float32)  # Gaussian rows: wide nuclei
    T = rng.choice([0.4, 0.7, 1.0, 1.4], B)
    K = np.zeros(B, np.int32)
    K[::7] = V + 3
    P = 0.5 + 0.49 * rng.random(B)
    P[1::5] = 1.0   # top_p 1 without top-k: the draw over the whole vocabulary
    U = rng.random(B)
    U[2] = 0.0
    U[4] = 1.0 - 1e-12
    return x, T, K, P, U


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_distributed_nucleus_emulated(torch, world):
    """Rows without top-k that the records cannot settle (nuclei wider than
    the candidates, top_p 1) finish through the histogram all-reduce, the
    bracket exchange and the owner's draw, with no logits exchanged: every
    row matches the oracle on the full row."""
    B, V = 48, 65536
    x, T, K, P, U = _wide_rows(31, B, V)
    tok, prob, st, finished = emulate_nucleus(torch, x, T, K, P, U, world)
    flagged_by_merge = len(finished)
    assert flagged_by_merge >= B // 3, flagged_by_merge
    assert np.all(st == 0), st
    compare(tok, prob, st, x, T, K, P, U, label=f"distributed nucleus x{world}")


def test_distributed_nucleus_through_sharded_sampler(torch):
    """ShardedSampler on one process (world 1): the k=0 rows go through the
    distributed nucleus, not the full-row path; bf16 logits and a mask too."""
    from miniserve_b200.sharded import ShardedSampler
    B, V = 24, 40000
    x, T, K, P, U = _wide_rows(32, B, V)
    xb = ((x.view(np.uint32) >> 16).astype(np.uint32) << 16).view(np.float32)
    rng = np.random.default_rng(4)
    mask = rng.integers(0, 2**32, (B, V // 32), dtype=np.uint64).astype(np.uint32)  # V % 32 == 0
    s = ShardedSampler(V)
    xt = torch.from_numpy(xb).cuda().to(torch.bfloat16)
    mt = torch.from_numpy(mask.view(np.int32)).cuda()
    t2, p2, s2 = s.sample(xt, 0, T, K, P, uniforms=U, mask=mt)
    torch.cuda.synchronize()
    assert s.last_full_rows == 0 and s.last_nucleus_rows > 0, (s.last_full_rows, s.last_nucleus_rows)
    compare(t2.cpu().numpy(), p2.cpu().numpy().astype(np.float64), s2.cpu().numpy(), xb, T, K, P, U,
            bf16=False, mask=mask, label="sharded sampler bf16 + mask, nucleus rows")


def test_nccl_two_ranks(torch):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = min(n, 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", "--master-port=29531", os.path.join(HERE, "mp_sharded.py")]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "sharded ok" in r.stdout
