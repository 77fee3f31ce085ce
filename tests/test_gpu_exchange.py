"""The fused peer exchange of vocab-sharded sampling (ms_shard_exchange +
ms_exchange_merge) on one GPU.  The ranks are emulated: every rank's
exchange buffer is a block on this GPU, and every rank's streaming kernel
runs before any merge, every merge before any result collection (a step that
waits finds what it waits for already stored).
Tokens must equal the all-gather path (ms_shard_candidates + ms_shard_merge)
bit for bit and the oracle on the full rows.  With two GPUs the same path
runs under torchrun (tests/mp_sharded.py).  Needs a B200."""
import ctypes

import numpy as np
import pytest

from parity import compare

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    if not t.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return t


class Buffers:
    """`world` exchange buffers on this GPU, freed on close."""

    def __init__(self, torch, world, Bcap, kmax_cap):
        from miniserve_b200 import _lib
        self.L = _lib.lib()
        self.Bcap, self.kmax_cap, self.world = Bcap, kmax_cap, world
        words = self.L.ms_exchange_words(Bcap, world, kmax_cap)
        assert words > 0
        self.ptrs = []
        for _ in range(world):
            p = ctypes.c_void_p()
            assert self.L.ms_device_alloc(words * 4, ctypes.byref(p)) == 0
            self.ptrs.append(p.value)
        self.peers = torch.tensor(self.ptrs, dtype=torch.int64, device="cuda")
        self.epoch = 0

    def close(self):
        for p in self.ptrs:
            self.L.ms_device_free(p)


def _slice_mask(torch, mask, v0, v1):
    mt = torch.from_numpy(np.ascontiguousarray(mask[:, v0 // 32:(v1 + 31) // 32]).view(np.int32)).cuda()
    return mt.data_ptr(), mt.stride(0), mt


def run_exchange(torch, bufs, xt, T, K, P, U, kmax, bf16=False, mask=None, ranks=None, timeout_ns=10**9):
    """One call of every emulated rank (or of `ranks` only, the others
    missing); returns each of those ranks' (tokens, probs, status) as numpy
    arrays."""
    from miniserve_b200 import sharded
    L = bufs.L
    B, V = xt.shape
    dev = xt.device
    Tt = torch.tensor(T, dtype=torch.float64, device=dev)
    Kt = torch.tensor(K, dtype=torch.int32, device=dev)
    Pt = torch.tensor(P, dtype=torch.float64, device=dev)
    Ut = torch.tensor(U, dtype=torch.float64, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    bufs.epoch += 1
    world = bufs.world
    for r in (range(world) if ranks is None else ranks):
        v0, v1 = sharded.shard_bounds(V, world, r)
        part = xt[:, v0:v1]
        mptr, mld, keep = (None, 0, None) if mask is None else _slice_mask(torch, mask, v0, v1)
        rc = L.ms_shard_exchange(part.data_ptr(), 1 if bf16 else 0, B, v1 - v0, part.stride(0), v0, V,
                                 Tt.data_ptr(), Kt.data_ptr(), Pt.data_ptr(), Ut.data_ptr(), mptr, mld, kmax,
                                 bufs.ptrs[r], bufs.peers.data_ptr(), r, world, bufs.Bcap, bufs.kmax_cap,
                                 bufs.epoch, s)
        assert rc == 0, rc
        torch.cuda.synchronize()
    out = []
    for r in (range(world) if ranks is None else ranks):
        tok = torch.empty(B, dtype=torch.int64, device=dev)
        prob = torch.empty(B, dtype=torch.float32, device=dev)
        st = torch.empty(B, dtype=torch.int32, device=dev)
        out.append((tok, prob, st))
        rc = L.ms_exchange_merge(bufs.ptrs[r], bufs.peers.data_ptr(), r, world, B, bufs.Bcap, kmax, bufs.kmax_cap, V, Tt.data_ptr(),
                                 Kt.data_ptr(), Pt.data_ptr(), Ut.data_ptr(), bufs.epoch, timeout_ns, tok.data_ptr(),
                                 prob.data_ptr(), st.data_ptr(), s)
        assert rc == 0, rc
        torch.cuda.synchronize()
    # every rank's merges ran before any rank collects the results (a
    # collection waits for other ranks' merges)
    for r, (tok, prob, st) in zip(range(world) if ranks is None else ranks, out):
        rc = L.ms_exchange_results(bufs.ptrs[r], world, B, bufs.Bcap, bufs.kmax_cap, bufs.epoch, timeout_ns,
                                   tok.data_ptr(), prob.data_ptr(), st.data_ptr(), s)
        assert rc == 0, rc
        torch.cuda.synchronize()
    return [(tok.cpu().numpy(), prob.cpu().numpy(), st.cpu().numpy()) for tok, prob, st in out]


def gathered(torch, xt, T, K, P, U, world, kmax, bf16=False, mask=None):
    """The all-gather path on the same slices (records stacked rank-major)."""
    from miniserve_b200 import _lib, sharded
    L = _lib.lib()
    B, V = xt.shape
    dev = xt.device
    Tt = torch.tensor(T, dtype=torch.float64, device=dev)
    Kt = torch.tensor(K, dtype=torch.int32, device=dev)
    Pt = torch.tensor(P, dtype=torch.float64, device=dev)
    Ut = torch.tensor(U, dtype=torch.float64, device=dev)
    recs = torch.empty((world, B, sharded.record_words(kmax)), dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    for r in range(world):
        v0, v1 = sharded.shard_bounds(V, world, r)
        part = xt[:, v0:v1]
        mptr, mld, keep = (None, 0, None) if mask is None else _slice_mask(torch, mask, v0, v1)
        assert L.ms_shard_candidates(part.data_ptr(), 1 if bf16 else 0, B, v1 - v0, part.stride(0), v0, V,
                                     Tt.data_ptr(), Kt.data_ptr(), mptr, mld, kmax, recs[r].data_ptr(), s) == 0
        torch.cuda.synchronize()
    tok = torch.empty(B, dtype=torch.int64, device=dev)
    prob = torch.empty(B, dtype=torch.float32, device=dev)
    st = torch.empty(B, dtype=torch.int32, device=dev)
    assert L.ms_shard_merge(recs.data_ptr(), world, B, kmax, V, Tt.data_ptr(), Kt.data_ptr(), Pt.data_ptr(),
                            Ut.data_ptr(), tok.data_ptr(), prob.data_ptr(), st.data_ptr(), s) == 0
    torch.cuda.synchronize()
    return tok.cpu().numpy(), prob.cpu().numpy(), st.cpu().numpy(), recs


def _mixed(seed=9, B=48, V=65536):
    rng = np.random.default_rng(seed)
    base = -1.1 * np.log(np.arange(1, V + 1, dtype=np.float64))
    x = np.stack([(base[rng.permutation(V)] + rng.normal(0, 0.5, V)).astype(np.float32) for _ in range(B)])
    x[5, 40000:40100] = x[5].max() + 1.0   # a tie block of maxima across a slice edge
    x[6, :] = -np.inf                        # every logit masked
    x[9, 123] = np.nan                       # a NaN: flagged, left to the full-row path
    T = rng.choice([0.0, 0.8, 1.2], B)
    K = rng.choice([0, 1, 2, 20, 50, 200], B).astype(np.int32)
    P = rng.choice([0.95, 0.6, 1.0], B)
    U = rng.random(B)
    T[6] = 0.0
    U[7] = 0.0
    return x, T, K, P, U


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_exchange_equals_gather_path(torch, world):
    """Three calls in a row on the same buffers (both record areas, the flags
    of earlier calls in place): every rank's tokens equal the all-gather
    path's bit for bit, the records sit in every buffer in the all-gather
    layout, and the exact rows equal the oracle."""
    from miniserve_b200 import sharded
    x, T, K, P, U = _mixed(seed=world)
    kmax = sharded.choose_kmax(list(K), list(T), list(P), x.shape[1])
    xt = torch.from_numpy(x).cuda()
    bufs = Buffers(torch, world, 64, max(kmax, 64))
    try:
        for call in range(3):
            Uc = np.roll(U, call)
            outs = run_exchange(torch, bufs, xt, T, K, P, Uc, kmax)
            g_tok, g_prob, g_st, recs = gathered(torch, xt, T, K, P, Uc, world, kmax)
            for tok, prob, st in outs:
                assert np.array_equal(tok, g_tok)
                assert np.array_equal(prob.view(np.uint32), g_prob.view(np.uint32))
                assert np.array_equal(st, g_st)
            # the words a record defines: count, status, the count's keys and ids
            off = bufs.L.ms_exchange_records_offset(bufs.Bcap, world, bufs.kmax_cap, bufs.epoch)
            W = sharded.record_words(kmax)
            want = recs.cpu().numpy()
            m = np.minimum(want[:, :, 0], kmax)
            for p in bufs.ptrs:
                view = torch.as_tensor(sharded._RawInt32(p + 4 * off, (world, x.shape[0], W)), device="cuda")
                got = view.cpu().numpy()
                assert np.array_equal(got[:, :, :2], want[:, :, :2])
                for q in range(world):
                    for row in range(x.shape[0]):
                        n = m[q, row]
                        assert np.array_equal(got[q, row, 2:2 + n], want[q, row, 2:2 + n])
                        assert np.array_equal(got[q, row, 2 + kmax:2 + kmax + n],
                                              want[q, row, 2 + kmax:2 + kmax + n])
            r = np.nonzero(g_st == 0)[0]
            compare(g_tok[r], g_prob[r].astype(np.float64), g_st[r], x[r], T[r], K[r], P[r], Uc[r],
                    label=f"exchange x{world} call {call}")
    finally:
        bufs.close()


def test_exchange_bf16_mask_and_batch_sizes(torch):
    """bf16 slices with a mask, and calls of different batch sizes on one
    buffer (rows past a call's batch keep older flags)."""
    from miniserve_b200 import sharded
    x, T, K, P, U = _mixed(seed=10)
    xb = ((x.view(np.uint32) >> 16).astype(np.uint32) << 16).view(np.float32)
    rng = np.random.default_rng(3)
    mask = rng.integers(0, 2**32, (x.shape[0], x.shape[1] // 32), dtype=np.uint64).astype(np.uint32)
    xt = torch.from_numpy(xb).cuda().to(torch.bfloat16)
    kmax = sharded.choose_kmax(list(K), list(T), list(P), x.shape[1])
    bufs = Buffers(torch, 4, 64, kmax)
    try:
        for B in (48, 7, 48, 1):
            outs = run_exchange(torch, bufs, xt[:B], T[:B], K[:B], P[:B], U[:B], kmax, bf16=True, mask=mask[:B])
            g_tok, g_prob, g_st, _ = gathered(torch, xt[:B], T[:B], K[:B], P[:B], U[:B], 4, kmax, bf16=True,
                                              mask=mask[:B])
            for tok, prob, st in outs:
                assert np.array_equal(tok, g_tok) and np.array_equal(st, g_st)
                assert np.array_equal(prob.view(np.uint32), g_prob.view(np.uint32))
    finally:
        bufs.close()


def test_exchange_merge_times_out_without_peer(torch):
    """A rank that never runs its streaming kernel: its records never arrive,
    so rank 0's merges wait their limit (2 ms here) and its rows come back
    MS_ROW_PEER_TIMEOUT with token -1, and so do the rows rank 1 would have
    merged (their results never arrive); the device stays usable."""
    x, T, K, P, U = _mixed(seed=12, B=16)
    K[:] = 20
    xt = torch.from_numpy(x).cuda()
    bufs = Buffers(torch, 2, 16, 64)
    try:
        outs = run_exchange(torch, bufs, xt, T, K, P, U, 20, ranks=[0], timeout_ns=2_000_000)
        tok, prob, st = outs[0]
        assert np.all(st == 16) and np.all(tok == -1)
        assert float(torch.ones(4, device="cuda").sum()) == 4.0
    finally:
        bufs.close()


def test_sharded_sampler_peer_matches_nccl_path(torch):
    """ShardedSampler on one rank: the peer exchange and the all-gather path
    give the same tokens, the distributed nucleus included (its rows read the
    records from the exchange buffer)."""
    from miniserve_b200.sharded import ShardedSampler
    x, T, K, P, U = _mixed(seed=13, B=32)
    K[:6] = 0
    P[:6] = [1.0, 1.0, 0.9, 0.99, 0.5, 1.0]
    T[:6] = [0.9, 1.5, 1.4, 1.2, 0.7, 0.0]
    xt = torch.from_numpy(x).cuda()
    a = ShardedSampler(x.shape[1], exchange="peer")
    b = ShardedSampler(x.shape[1], exchange="nccl")
    try:
        for call in range(2):
            Uc = np.roll(U, call)
            t1, p1, s1 = a.sample(xt, 0, T, K, P, uniforms=Uc)
            t2, p2, s2 = b.sample(xt, 0, T, K, P, uniforms=Uc)
            torch.cuda.synchronize()
            assert a.last_exchange == "peer" and b.last_exchange == "nccl"
            assert torch.equal(t1, t2) and torch.equal(s1, s2) and torch.equal(p1, p2)
            assert a.last_nucleus_rows == b.last_nucleus_rows
            compare(t1.cpu().numpy(), p1.cpu().numpy().astype(np.float64), s1.cpu().numpy(), x, T, K, P, Uc,
                    label=f"sharded sampler peer call {call}")
    finally:
        a.close()
