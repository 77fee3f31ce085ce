"""Host side of the vocab-sharded path on CPU: slice bounds, record width,
and a world_size-2 gloo run of the record all-gather and the full-row gather,
with the decomposition (union of the slices' top-k) checked against the
oracle on the full rows."""
import os
import socket

import numpy as np
import pytest

import oracle
import sharded_ref
from miniserve_b200 import sharded


def test_shard_bounds_partition():
    for V in (1, 7, 4096, 151936, 256000):
        for world in (1, 2, 3, 4, 8):
            b = [sharded.shard_bounds(V, world, r) for r in range(world)]
            assert b[0][0] == 0 and b[-1][1] == V
            assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
            assert max(e - s for s, e in b) - min(e - s for s, e in b) <= 1


def test_choose_kmax():
    assert sharded.choose_kmax([0, 1, 50, 20], [1.0, 1.0, 0.9, 0.0]) == 50
    # a row without top-k at top_p 1 needs the slice's maximum and total in its record
    assert sharded.choose_kmax([0, 300], [1.0, 1.0]) == 2
    assert sharded.choose_kmax([300, 1], [1.0, 1.0]) == 1
    assert sharded.record_words(50) == 104
    assert sharded.choose_kmax([0, 20], [1.0, 1.0], [0.9, 1.0], 1000) == sharded.KMAX_NUCLEUS
    assert sharded.choose_kmax([0, 20], [1.0, 1.0], [1.0, 1.0], 1000) == 20
    assert sharded.choose_kmax([1000, 20], [1.0, 0.0], [0.9, 1.0], 1000) == sharded.KMAX_NUCLEUS


def _batch(B=24, V=12288, seed=5):
    rng = np.random.default_rng(seed)
    base = -1.1 * np.log(np.arange(1, V + 1, dtype=np.float64))
    x = np.stack([(base[rng.permutation(V)] + rng.normal(0, 0.5, V)).astype(np.float32) for _ in range(B)])
    x[3, 100:200] = x[3].max()  # a tie block across the max
    T = rng.choice([0.0, 0.9, 1.3], B)
    K = rng.choice([1, 20, 50], B).astype(np.int32)
    P = rng.choice([0.95, 0.7, 1.0], B)
    U = rng.random(B)
    return x, T, K, P, U


def _worker(rank, world, port, out):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, T, K, P, U = _batch()
        B, V = x.shape
        v0, v1 = sharded.shard_bounds(V, world, rank)
        kmax = sharded.choose_kmax(K.tolist(), T.tolist())
        rec = sharded_ref.np_records(x[:, v0:v1], v0, V, T, K, kmax)
        allrec = sharded.exchange_records(torch.from_numpy(rec.view(np.int32)))
        rows = torch.tensor([0, 3, 7])
        full = sharded.gather_rows(torch.from_numpy(x[:, v0:v1].copy()), rows, V)
        if rank == 0:
            out.put((allrec.numpy().view(np.uint32), full.numpy()))
    finally:
        dist.destroy_process_group()


def test_gloo_exchange_and_decomposition():
    import multiprocessing as mp
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    allrec, full = q.get(timeout=120)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    x, T, K, P, U = _batch()
    B, V = x.shape
    assert allrec.shape[0] == world
    np.testing.assert_array_equal(full, x[[0, 3, 7]])
    kmax = sharded.choose_kmax(K.tolist(), T.tolist())
    rows, st = sharded_ref.sparse_rows(allrec, B, V, kmax)
    assert not st.any()
    t_sparse = oracle.c_sample(rows, T, K, P, U)[0]
    t_full = oracle.c_sample(x, T, K, P, U)[0]
    np.testing.assert_array_equal(t_sparse, t_full)


@pytest.mark.parametrize("world", [2, 4])
def test_nucleus_decomposition(world):
    """Top-p rows without top-k from the records alone (the merge's rule,
    restated in numpy): whenever the rule settles a row, its token is the
    oracle's token on the full row; low-temperature rows are settled."""
    rng = np.random.default_rng(31)
    B, V, kmax = 40, 12288, 64
    base = -1.1 * np.log(np.arange(1, V + 1, dtype=np.float64))
    x = np.stack([(base[rng.permutation(V)] + rng.normal(0, 0.5, V)).astype(np.float32) for _ in range(B)])
    T = rng.choice([0.2, 0.5, 0.9, 1.4], B)
    K = np.zeros(B, np.int32)
    P = 0.5 + 0.49 * rng.random(B)
    U = rng.random(B)
    recs = []
    for r in range(world):
        v0, v1 = sharded.shard_bounds(V, world, r)
        recs.append(sharded_ref.np_records(x[:, v0:v1], v0, V, T, K, kmax))
    allrec = np.stack(recs)
    o_tok, _, _, mp, mu = oracle.c_sample(x, T, K, P, U)
    settled = 0
    for b in range(B):
        t = sharded_ref.np_nucleus(allrec, b, V, kmax, T[b], P[b], U[b])
        if t is None:
            continue
        settled += 1
        if mp[b] >= 1e-6 and mu[b] >= 1e-6:
            assert t == o_tok[b], (b, t, o_tok[b])
    assert settled >= B // 3


@pytest.mark.parametrize("world", [1, 2, 3])
def test_distributed_nucleus_rule(world):
    """The distributed nucleus's rule (histogram bracket, exact cut on the
    bracket's values, owner of the index-order target), restated in numpy:
    its token is the oracle's token on the full row for every row outside the
    1e-6 boundary band, with nuclei far wider than any candidate record, top_p
    1 rows, r == 0 and r near 1."""
    rng = np.random.default_rng(41)
    B, V = 24, 8192
    base = -1.1 * np.log(np.arange(1, V + 1, dtype=np.float64))
    x = np.stack([(base[rng.permutation(V)] + rng.normal(0, 0.5, V)).astype(np.float32) for _ in range(B)])
    x[B // 2:] = rng.normal(0.0, 2.0, (B - B // 2, V)).astype(np.float32)
    x[5, 1000:1100] = -np.inf
    T = rng.choice([0.4, 1.0, 1.5], B)
    K = np.zeros(B, np.int32)
    P = 0.5 + 0.49 * rng.random(B)
    P[1::4] = 1.0
    U = rng.random(B)
    U[2], U[3] = 0.0, 1.0 - 1e-12
    bounds = [sharded.shard_bounds(V, world, r)[0] for r in range(world)] + [V]
    o_tok, _, _, mp, mu = oracle.c_sample(x, T, K, P, U)
    for b in range(B):
        slices = [x[b, bounds[r]:bounds[r + 1]] for r in range(world)]
        t = sharded_ref.np_distributed_nucleus(slices, bounds, T[b], P[b], U[b], V)
        assert t is not None, b
        if mp[b] >= 1e-6 and mu[b] >= 1e-6:
            assert t == o_tok[b], (b, t, o_tok[b])
