"""Vocab-sharded sampling: one process per GPU, each holding a contiguous
slice of the vocabulary (as a tensor-parallel LM head produces the logits).

Step 1 runs ``ms_shard_candidates`` on the rank's slice: per row, the slice's
top-k values (value descending, index ascending) with their global token ids,
in a fixed-size record.  Step 2 all-gathers the records of every rank (NCCL
over NVLink on GPUs; the only data that crosses the interconnect is
``B * (4 + 2*kmax) * 4`` bytes per rank).  Step 3 runs ``ms_shard_merge`` on
every rank, which finishes each row exactly as miniserve's
``Sampler.sample`` (miniserve/sampler.py:23-68) does on the whole vocabulary:
the row's top-k set is contained in the union of the slices' top-k sets.

With a peer exchange (``PeerExchange``, the default) step 2 is
fused into step 1: ``ms_shard_exchange`` stores each row's record into every
other rank's exchange buffer over NVLink as the row finishes (every word
tagged with the call's epoch in one 8-byte store); ``ms_exchange_merge``
waits (bounded) until a row's words from every rank carry the epoch, and the
row's owner (row mod world) merges it and stores the result into every
rank's buffer the same way; ``ms_exchange_results`` collects them (bounded).
No collective call is made on that path.

A top-p row without top-k is settled from the records too when its nucleus
lies among the candidates (the records carry each slice's softmax total);
rows the records cannot carry exactly (top_k above kmax, top_p >= 1 without
top-k, a nucleus reaching past the candidates, a non-finite logit, a tie block
larger than the candidate buffer) come back flagged; for those rows only, every rank all-gathers the full logits and
samples them with the single-GPU kernel, so every row is exact.  All ranks see
identical statuses, so they take the same collective steps.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

from . import _lib
from .sampler import Sampler, _param, _torch, check_mask, uniform_for_seed

KMAX_LIMIT = 256


def record_words(kmax: int) -> int:
    """32-bit words in one row's candidate record."""
    return 4 + 2 * int(kmax)


def shard_bounds(V: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous slice [v0, v1) of rank `rank` (slices in rank order)."""
    return (V * rank) // world, (V * (rank + 1)) // world


KMAX_NUCLEUS = 64  # record width for top-p rows without top-k


def choose_kmax(top_k: Sequence[int], temperature: Sequence[float],
                top_p: Optional[Sequence[float]] = None, V: Optional[int] = None) -> int:
    """Smallest record width that carries every greedy / top-k row (<= 256),
    and at least KMAX_NUCLEUS when some top-p row has no top-k."""
    need = 1
    ps = top_p if top_p is not None else [1.0] * len(top_k)
    for k, t, p in zip(top_k, temperature, ps):
        if t == 0.0 or k == 1:
            continue
        if 2 <= k <= KMAX_LIMIT and (V is None or k < V):
            need = max(need, int(k))
        elif k == 0 or (V is not None and k >= V):
            # no top-k: the record carries the slice's maximum and total (and,
            # for top-p rows, the top KMAX_NUCLEUS candidates)
            need = max(need, KMAX_NUCLEUS if p < 1.0 else 2)
    return need


def _host_list(x, B: int):
    """The per-row values of a host-side parameter (scalar or sequence) as a
    list, or None for a tensor (whose values live on the device)."""
    torch = _torch()
    if isinstance(x, torch.Tensor):
        return None
    if isinstance(x, (int, float)):
        return [x] * B
    return list(x)


def exchange_records(records, group=None):
    """All-gather [B, W] int32 records of every rank -> [world, B, W], rank-major."""
    torch = _torch()
    import torch.distributed as dist
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return records.unsqueeze(0)
    world = dist.get_world_size(group)
    out = torch.empty((world * records.shape[0],) + tuple(records.shape[1:]), dtype=records.dtype,
                      device=records.device)
    dist.all_gather_into_tensor(out, records.contiguous(), group=group)
    return out.view((world,) + tuple(records.shape))


class _RawInt32:
    """A CUDA array interface over raw device memory, for a tensor view."""

    def __init__(self, ptr: int, shape: Tuple[int, ...]) -> None:
        self.__cuda_array_interface__ = {"shape": tuple(int(d) for d in shape), "typestr": "<i4",
                                         "data": (int(ptr), False), "version": 3, "strides": None}


class PeerExchangeError(RuntimeError):
    pass


class PeerExchange:
    """Exchange buffers of the fused peer exchange (``ms_shard_exchange``):
    one zeroed device block per rank, mapped into every other rank's process
    by CUDA IPC (no multicast object).  Collective: every rank of ``group``
    constructs it with the same capacities; all ranks agree on success (the
    constructor raises PeerExchangeError on every rank when any rank fails).
    ``timeout_s`` bounds each call's wait for the other ranks' results."""

    def __init__(self, Bcap: int, kmax_cap: int, group=None, device=None, timeout_s: float = 10.0) -> None:
        import ctypes
        torch = _torch()
        self.group = group
        self.world, self.rank = _world(group)
        self.Bcap, self.kmax_cap = int(Bcap), int(kmax_cap)
        self.timeout_ns = int(timeout_s * 1e9)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        L = _lib.lib()
        words = L.ms_exchange_words(self.Bcap, self.world, self.kmax_cap)
        if words < 0:
            raise ValueError("exchange capacity out of range")
        self.words = int(words)
        self.local = None
        self._opened = []
        self.epoch = 0
        self.broken = False
        err = None
        handle = b""
        with torch.cuda.device(self.device):
            ptr = ctypes.c_void_p()
            rc = L.ms_device_alloc(self.words * 4, ctypes.byref(ptr))
            if rc == _lib.MS_OK:
                self.local = ptr.value
                if self.world > 1:
                    h = ctypes.create_string_buffer(64)
                    rc = L.ms_ipc_handle(self.local, h)
                    handle = h.raw if rc == _lib.MS_OK else b""
            if rc != _lib.MS_OK:
                err = f"exchange buffer: {L.ms_error_string(rc).decode()}"
            peers = [0] * self.world
            peers[self.rank] = self.local or 0
            if self.world > 1:
                import torch.distributed as dist
                handles = [None] * self.world
                dist.all_gather_object(handles, handle, group=group)
                for q in range(self.world):
                    if q == self.rank or err is not None:
                        continue
                    if len(handles[q]) != 64:
                        err = f"rank {q} has no exchange buffer"
                        continue
                    p = ctypes.c_void_p()
                    rc = L.ms_ipc_open(handles[q], ctypes.byref(p))
                    if rc != _lib.MS_OK:
                        err = f"CUDA IPC open of rank {q}: {L.ms_error_string(rc).decode()}"
                        continue
                    self._opened.append(p.value)
                    peers[q] = p.value
                errs = [None] * self.world
                dist.all_gather_object(errs, err, group=group)
                err = next((e for e in errs if e is not None), None)
            if err is not None:
                self._release()
                raise PeerExchangeError(err)
            self.peers = torch.tensor(peers, dtype=torch.int64, device=self.device)

    def fits(self, B: int, kmax: int) -> bool:
        return B <= self.Bcap and kmax <= self.kmax_cap and not self.broken

    def records(self, B: int, kmax: int, epoch: int):
        """[world, B, 4 + 2 kmax] int32 view of call ``epoch``'s records in
        this rank's buffer (the all-gather layout)."""
        torch = _torch()
        off = _lib.lib().ms_exchange_records_offset(self.Bcap, self.world, self.kmax_cap, epoch)
        shape = (self.world, B, record_words(kmax))
        return torch.as_tensor(_RawInt32(self.local + 4 * off, shape), device=self.device)

    def _release(self) -> None:
        L = _lib.lib()
        for p in self._opened:
            L.ms_ipc_close(p)
        self._opened = []
        if self.local:
            L.ms_device_free(self.local)
            self.local = None

    def close(self) -> None:
        """Unmap and free the buffers once no call is in flight on any rank
        (device synchronize and a barrier first).  Collective."""
        torch = _torch()
        if self.local is None:
            return
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            if self.world > 1:
                import torch.distributed as dist
                dist.barrier(group=self.group)
            self._release()


def _world(group=None) -> Tuple[int, int]:
    """(world size, rank) of the group, (1, 0) without a process group."""
    import torch.distributed as dist
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _all_reduce(t, op: str, group=None):
    """In-place all-reduce ('sum' or 'max') over the group; the identity
    without a process group."""
    import torch.distributed as dist
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return t
    dist.all_reduce(t, op=dist.ReduceOp.SUM if op == "sum" else dist.ReduceOp.MAX, group=group)
    return t


def gather_rows(logits_slice, rows, V: int, group=None):
    """Full-vocabulary logits [len(rows), V] of the given rows, assembled from
    every rank's slice (slices may differ in width by one token)."""
    torch = _torch()
    import torch.distributed as dist
    part = logits_slice[rows]
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return part.contiguous()
    world = dist.get_world_size(group)
    width = max(b - a for a, b in (shard_bounds(V, world, r) for r in range(world)))
    padded = torch.zeros((part.shape[0], width), dtype=part.dtype, device=part.device)
    padded[:, : part.shape[1]] = part
    out = torch.empty((world * padded.shape[0], width), dtype=part.dtype, device=part.device)
    dist.all_gather_into_tensor(out, padded.contiguous(), group=group)
    out = out.view(world, padded.shape[0], width)
    cols = [out[r, :, : b - a] for r, (a, b) in enumerate(shard_bounds(V, world, r) for r in range(world))]
    return torch.cat(cols, dim=1).contiguous()


class ShardedSampler:
    """Sample [B, V] rows whose vocabulary is split across the ranks of `group`."""

    def __init__(self, V: int, group=None, exchange: str = "auto", peer_timeout_s: float = 10.0) -> None:
        """``exchange``: "auto" (the fused peer exchange when CUDA IPC maps
        every rank's buffer, else nccl; the choice is the same on every
        rank), "peer" (PeerExchangeError if CUDA IPC is unavailable) or
        "nccl" (all-gather of the records and a merge kernel)."""
        if exchange not in ("auto", "peer", "nccl"):
            raise ValueError("exchange must be 'auto', 'peer' or 'nccl'")
        self.V = int(V)
        self.group = group
        self.exchange = exchange
        self.peer_timeout_s = float(peer_timeout_s)
        self._x = None
        self.last_exchange = None  # "peer" or "nccl": the path the last call took
        self._single = Sampler()
        # rows of the last call finished by the distributed nucleus, and rows
        # that took the full-row path (gathered logits)
        self.last_nucleus_rows = 0
        self.last_full_rows = 0

    def _peer(self, B: int, kmax: int, dev):
        """The peer exchange for a call of B rows and record width kmax, (re)made
        when it does not fit; None on the nccl path."""
        if self.exchange == "nccl":
            return None
        if self._x is not None and self._x.fits(B, kmax):
            return self._x
        if self._x is not None:
            if self._x.broken:
                raise PeerExchangeError("the peer exchange timed out in an earlier call")
            self._x.close()
            self._x = None
        try:
            self._x = PeerExchange(max(B, 256), max(kmax, KMAX_NUCLEUS), self.group, dev, self.peer_timeout_s)
        except PeerExchangeError:
            if self.exchange == "peer":
                raise
            self.exchange = "nccl"
            return None
        return self._x

    def close(self) -> None:
        """Release the peer exchange buffers (collective)."""
        if self._x is not None:
            self._x.close()
            self._x = None

    def sample(self, logits_slice, v0: int, temperature=1.0, top_k=0, top_p=1.0,
               uniforms=None, seeds: Optional[Sequence[Optional[int]]] = None,
               mask=None, kmax: Optional[int] = None, events=None):
        """``logits_slice``: this rank's [B, Vloc] CUDA tensor (fp32/bf16) for
        tokens [v0, v0 + Vloc); ``mask``: optional [B, ceil(Vloc/32)] bitmask of
        the slice.  Per-row parameters must be the same on every rank.  Returns
        (tokens i64, probs f32, status i32), identical on every rank.

        The record width ``kmax`` is chosen from the parameters (choose_kmax)
        when they are host values; pass it when they are device tensors, or
        their values are read back once.  After the merge one device->host read
        of a count decides whether any row needs the full-row path.
        ``events``: optional four CUDA events recorded around the shard pass,
        the all-gather and the merge (for timing the phases); with the peer
        exchange: before and after the streaming kernel (which also stores the
        records into every rank's buffer) and after the merge (the last two
        events together)."""
        torch = _torch()
        if logits_slice.dim() != 2 or not logits_slice.is_cuda:
            raise ValueError("logits_slice must be a [B, Vloc] CUDA tensor")
        if kmax is None:
            B0 = logits_slice.shape[0]
            hk, ht, hp = _host_list(top_k, B0), _host_list(temperature, B0), _host_list(top_p, B0)
            if hk is not None and ht is not None and hp is not None:
                kmax = choose_kmax(hk, ht, hp, self.V)
        if logits_slice.stride(1) != 1:
            logits_slice = logits_slice.contiguous()
        dtype = {torch.float32: _lib.MS_DTYPE_F32, torch.bfloat16: _lib.MS_DTYPE_BF16}.get(logits_slice.dtype)
        if dtype is None:
            raise TypeError(f"logits dtype {logits_slice.dtype} is not float32 or bfloat16")
        B, Vloc = logits_slice.shape
        dev = logits_slice.device
        T = _param(temperature, B, torch.float64, dev)
        K = _param(top_k, B, torch.int32, dev)
        P = _param(top_p, B, torch.float64, dev)
        if uniforms is None:
            seeds = [None] * B if seeds is None else list(seeds)
            uniforms = [uniform_for_seed(s) for s in seeds]
        U = _param(uniforms, B, torch.float64, dev)
        if kmax is None:  # device-side parameters: one read of their values
            kmax = choose_kmax(K.tolist(), T.tolist(), P.tolist(), self.V)
        if not 1 <= int(kmax) <= KMAX_LIMIT:
            raise ValueError(f"kmax must be in 1..{KMAX_LIMIT}")
        kmax = int(kmax)
        W = record_words(kmax)
        L = _lib.lib()
        mask_ptr, mask_ld = None, 0
        if mask is not None:
            mask_ptr, mask_ld = check_mask(mask, B, Vloc, dev)
        tokens = torch.empty(B, dtype=torch.int64, device=dev)
        probs = torch.empty(B, dtype=torch.float32, device=dev)
        status = torch.empty(B, dtype=torch.int32, device=dev)
        x = self._peer(B, kmax, dev) if B > 0 else None
        self.last_exchange = "peer" if x is not None else "nccl"
        if x is not None:
            with torch.cuda.device(dev):
                cur = torch.cuda.current_stream(dev)
                stream = cur.cuda_stream
                x.epoch += 1
                epoch = (x.epoch - 1) % (2 ** 32 - 2) + 1  # parity alternates across the wrap
                if events is not None:
                    events[0].record(cur)
                rc = L.ms_shard_exchange(logits_slice.data_ptr(), dtype, B, Vloc, logits_slice.stride(0), int(v0),
                                         self.V, T.data_ptr(), K.data_ptr(), P.data_ptr(), U.data_ptr(), mask_ptr,
                                         mask_ld, kmax, x.local, x.peers.data_ptr(), x.rank, x.world, x.Bcap,
                                         x.kmax_cap, epoch, stream)
                _lib.check(rc, "ms_shard_exchange")
                if events is not None:
                    events[1].record(cur)
                rc = L.ms_exchange_merge(x.local, x.peers.data_ptr(), x.rank, x.world, B, x.Bcap, kmax, x.kmax_cap, self.V, T.data_ptr(),
                                         K.data_ptr(), P.data_ptr(), U.data_ptr(), epoch, x.timeout_ns,
                                         tokens.data_ptr(), probs.data_ptr(), status.data_ptr(), stream)
                _lib.check(rc, "ms_exchange_merge")
                rc = L.ms_exchange_results(x.local, x.world, B, x.Bcap, x.kmax_cap, epoch, x.timeout_ns,
                                           tokens.data_ptr(), probs.data_ptr(), status.data_ptr(), stream)
                _lib.check(rc, "ms_exchange_results")
                if events is not None:
                    events[2].record(cur)
                    events[3].record(cur)
            allrec = x.records(B, kmax, epoch)
            return self._finish(logits_slice, dtype, v0, allrec, kmax, T, K, P, U, mask, mask_ptr, mask_ld,
                                tokens, probs, status, x)
        records = torch.empty((B, W), dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            cur = torch.cuda.current_stream(dev)
            stream = cur.cuda_stream
            if events is not None:
                events[0].record(cur)
            rc = L.ms_shard_candidates(logits_slice.data_ptr(), dtype, B, Vloc, logits_slice.stride(0), int(v0),
                                       self.V, T.data_ptr(), K.data_ptr(), mask_ptr, mask_ld, kmax,
                                       records.data_ptr(), stream)
            _lib.check(rc, "ms_shard_candidates")
            if events is not None:
                events[1].record(cur)
            allrec = exchange_records(records, self.group)
            if events is not None:
                events[2].record(cur)
            nranks = allrec.shape[0]
            rc = L.ms_shard_merge(allrec.data_ptr(), nranks, B, kmax, self.V, T.data_ptr(), K.data_ptr(),
                                  P.data_ptr(), U.data_ptr(), tokens.data_ptr(), probs.data_ptr(),
                                  status.data_ptr(), stream)
            _lib.check(rc, "ms_shard_merge")
            if events is not None:
                events[3].record(cur)
        return self._finish(logits_slice, dtype, v0, allrec, kmax, T, K, P, U, mask, mask_ptr, mask_ld,
                            tokens, probs, status, None)

    def _finish(self, logits_slice, dtype, v0, allrec, kmax, T, K, P, U, mask, mask_ptr, mask_ld, tokens, probs,
                status, x):
        """The flagged rows of a merged call: the distributed nucleus, then
        the full-row path for what is left."""
        torch = _torch()
        Vloc = logits_slice.shape[1]
        flagged = (status & (_lib.MS_ROW_UNSUPPORTED | _lib.MS_ROW_NONFINITE)) != 0
        # rows without top-k the records could not settle: the distributed
        # nucleus (no logits exchanged); the statuses are identical on every
        # rank, so are these counts and branches
        nuc = flagged & ((status & _lib.MS_ROW_NONFINITE) == 0) & ((K <= 0) | (K >= self.V))
        late = (status & _lib.MS_ROW_PEER_TIMEOUT) != 0
        n_flagged, n_nuc, n_late = (int(v) for v in torch.stack([flagged.sum(), nuc.sum(), late.sum()]).tolist())
        if n_late:
            x.broken = True
            raise PeerExchangeError(f"{n_late} rows missed another rank's record within "
                                    f"{self.peer_timeout_s} s")
        self.last_nucleus_rows = 0
        if (n_nuc and kmax >= 2 and Vloc <= NUCLEUS_MAX_SLICE and self.V <= NUCLEUS_MAX_V
                and allrec.shape[0] <= NUCLEUS_MAX_RANKS):
            rows = nuc.nonzero().flatten()
            done = self._nucleus(logits_slice, dtype, v0, rows, allrec, kmax, T, P, U, mask_ptr, mask_ld,
                                 tokens, probs, status)
            flagged[rows] = ~done
            n_flagged, n_done = (int(v) for v in torch.stack([flagged.sum(), done.sum()]).tolist())
            self.last_nucleus_rows = n_done
        self.last_full_rows = n_flagged
        if n_flagged:
            rows = flagged.nonzero().flatten()
            full = gather_rows(logits_slice, rows, self.V, self.group)
            fmask = None
            if mask is not None:
                fmask = _full_mask(mask, rows, Vloc, self.V, self.group)
            t2, p2, s2 = self._single.sample_batch(full, T[rows], K[rows], P[rows], uniforms=U[rows], mask=fmask)
            tokens[rows], probs[rows], status[rows] = t2, p2, s2
        return tokens, probs, status


    def _nucleus(self, logits_slice, dtype, v0, rows, allrec, kmax, T, P, U, mask_ptr, mask_ld, tokens, probs,
                 status):
        """Rows without top-k that the candidate records could not settle:
        histogram all-reduce, bracket, classifying pass, all-gather of the
        bracket's values, exact cut, draw on the rank holding the target, max
        all-reduce of the tokens (ms_nucleus_* in include/mssample.h).  Writes
        the finished rows; returns which of ``rows`` it finished."""
        torch = _torch()
        L = _lib.lib()
        dev = logits_slice.device
        B, Vloc = logits_slice.shape
        F = int(rows.numel())
        world, rank = _world(self.group)
        nranks = int(allrec.shape[0])
        rows32 = rows.to(torch.int32).contiguous()
        hist = torch.empty((F, int(L.ms_nucleus_hist_words())), dtype=torch.int32, device=dev)
        bracket = torch.empty((F, 2), dtype=torch.int32, device=dev)
        ent = torch.empty((F, int(L.ms_nucleus_record_words())), dtype=torch.int32, device=dev)
        cut = torch.empty((F, int(L.ms_nucleus_cut_words())), dtype=torch.int32, device=dev)
        segs = torch.empty((F, int(L.ms_nucleus_segments())), dtype=torch.float64, device=dev)
        out = torch.empty((F, 2), dtype=torch.int64, device=dev)
        bounds = torch.tensor([shard_bounds(self.V, world, r)[0] for r in range(world)] + [self.V],
                              dtype=torch.int64, device=dev)
        ld = logits_slice.stride(0)
        x = logits_slice.data_ptr()
        with torch.cuda.device(dev):
            stream = torch.cuda.current_stream(dev).cuda_stream
            _lib.check(L.ms_nucleus_hist(x, dtype, Vloc, ld, mask_ptr, mask_ld, rows32.data_ptr(), F, B, self.V,
                                         allrec.data_ptr(), nranks, kmax, T.data_ptr(), P.data_ptr(),
                                         hist.data_ptr(), stream), "ms_nucleus_hist")
            _all_reduce(hist, "sum", self.group)
            _lib.check(L.ms_nucleus_bracket(hist.data_ptr(), rows32.data_ptr(), F, self.V, P.data_ptr(),
                                            bracket.data_ptr(), stream), "ms_nucleus_bracket")
            _lib.check(L.ms_nucleus_classify(x, dtype, Vloc, ld, int(v0), mask_ptr, mask_ld, rows32.data_ptr(), F,
                                             B, allrec.data_ptr(), nranks, kmax, T.data_ptr(), bracket.data_ptr(),
                                             ent.data_ptr(), segs.data_ptr(), stream), "ms_nucleus_classify")
            allent = exchange_records(ent, self.group)
            _lib.check(L.ms_nucleus_cut(allent.data_ptr(), nranks, bounds.data_ptr(), bracket.data_ptr(),
                                        rows32.data_ptr(), F, B, allrec.data_ptr(), kmax, T.data_ptr(),
                                        P.data_ptr(), U.data_ptr(), cut.data_ptr(), stream), "ms_nucleus_cut")
            _lib.check(L.ms_nucleus_draw(x, dtype, Vloc, ld, int(v0), mask_ptr, mask_ld, rows32.data_ptr(), F, B,
                                         allrec.data_ptr(), nranks, kmax, T.data_ptr(), cut.data_ptr(),
                                         allent.data_ptr(), segs.data_ptr(), rank, out.data_ptr(), stream),
                       "ms_nucleus_draw")
            _all_reduce(out, "max", self.group)
        # written on the device, without reading `done` back
        done = (cut[:, 3] == 0) & (out[:, 0] >= 0)
        tokens[rows] = torch.where(done, out[:, 0], tokens[rows])
        probs[rows] = torch.where(done, out[:, 1].to(torch.int32).view(torch.float32), probs[rows])
        status[rows] = torch.where(done, torch.zeros_like(status[rows]), status[rows])
        return done


NUCLEUS_MAX_SLICE = 1 << 20  # longest slice the distributed nucleus takes
NUCLEUS_MAX_V = (2**31 - 1) // 16  # largest vocabulary (histogram scale >= 16)
NUCLEUS_MAX_RANKS = 256


def _full_mask(mask, rows, Vloc: int, V: int, group):
    """Full-vocabulary bitmask of `rows` from every rank's slice mask."""
    torch = _torch()
    import torch.distributed as dist
    bits = _unpack_bits(mask[rows], Vloc)
    if group is not None or (dist.is_available() and dist.is_initialized()):
        bits = gather_rows(bits, torch.arange(bits.shape[0], device=bits.device), V, group)
    return _pack_bits(bits)


def _unpack_bits(words, n: int):
    torch = _torch()
    w = words.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(32, device=w.device, dtype=torch.int64)
    bits = ((w.unsqueeze(-1) >> shifts) & 1).reshape(w.shape[0], -1)[:, :n]
    return bits.to(torch.uint8)


def _pack_bits(bits):
    torch = _torch()
    B, n = bits.shape
    W = (n + 31) // 32
    padded = torch.zeros((B, W * 32), dtype=torch.int64, device=bits.device)
    padded[:, :n] = bits.to(torch.int64)
    shifts = torch.arange(32, device=bits.device, dtype=torch.int64)
    words = (padded.reshape(B, W, 32) << shifts).sum(-1)
    return ((words + 2**31) % 2**32 - 2**31).to(torch.int32)  # the same 32 bits as int32
