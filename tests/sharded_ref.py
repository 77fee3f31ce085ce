"""Test-side numpy restatement of the vocab-sharded record (the layout
documented at ms_shard_candidates in include/mssample.h), used to check the
host protocol and the decomposition on CPU."""
from __future__ import annotations

import numpy as np

ROW_BAD_TEMPERATURE = 2
ROW_UNSUPPORTED = 8


def fkey(v: np.ndarray) -> np.ndarray:
    """Order key of fp32 values (-0 shares +0's key)."""
    bits = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32).copy()
    bits[bits == 0x80000000] = 0
    return np.where(bits & 0x80000000, ~bits, bits | 0x80000000).astype(np.uint32)


def key_to_f32(k: np.ndarray) -> np.ndarray:
    k = k.astype(np.uint32)
    bits = np.where(k & 0x80000000, k & 0x7FFFFFFF, ~k).astype(np.uint32)
    return bits.view(np.float32)


def np_records(x_slice, v0, V, T, K, kmax):
    """Candidate records [B, 2 + 2*kmax] (uint32) of one rank's slice."""
    B, Vloc = x_slice.shape
    rec = np.zeros((B, 2 + 2 * kmax), np.uint32)
    for b in range(B):
        t, k = float(T[b]), int(K[b])
        if not (t >= 0.0) or np.isinf(t):
            rec[b, 1] = ROW_BAD_TEMPERATURE
            continue
        if t == 0.0 or k == 1:
            kk = 1
        elif 2 <= k < V and k <= kmax and k < Vloc:
            kk = k
        else:
            rec[b, 1] = ROW_UNSUPPORTED
            continue
        vals = x_slice[b].astype(np.float32)
        order = np.lexsort((np.arange(Vloc), -vals.astype(np.float64)))
        order = [i for i in order if vals[i] > -np.inf][:kk]
        m = len(order)
        rec[b, 0] = m
        rec[b, 2:2 + m] = fkey(vals[order])
        rec[b, 2 + kmax:2 + kmax + m] = (v0 + np.array(order, np.int64)).astype(np.uint32)
    return rec


def sparse_rows(allrec, B, V, kmax):
    """Full-vocabulary rows holding only the gathered candidates (-inf
    elsewhere), and the OR of the ranks' statuses."""
    rows = np.full((B, V), -np.inf, np.float32)
    st = np.zeros(B, np.uint32)
    for r in range(allrec.shape[0]):
        for b in range(B):
            m = int(allrec[r, b, 0])
            st[b] |= allrec[r, b, 1]
            ids = allrec[r, b, 2 + kmax:2 + kmax + m].astype(np.int64)
            rows[b, ids] = key_to_f32(allrec[r, b, 2:2 + m])
    return rows, st
