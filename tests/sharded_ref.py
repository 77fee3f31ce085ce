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
    """Candidate records [B, 4 + 2*kmax] (uint32) of one rank's slice."""
    B, Vloc = x_slice.shape
    rec = np.zeros((B, 4 + 2 * kmax), np.uint32)
    for b in range(B):
        t, k = float(T[b]), int(K[b])
        if not (t >= 0.0) or np.isinf(t):
            rec[b, 1] = ROW_BAD_TEMPERATURE
            continue
        total = False
        if t == 0.0 or k == 1:
            kk = 1
        elif 2 <= k < V:
            if not (k <= kmax and k < Vloc):
                rec[b, 1] = ROW_UNSUPPORTED
                continue
            kk = k
        elif 2 <= kmax < Vloc and t >= 1e-30:  # no top-k: top kmax and the slice total
            kk, total = kmax, True
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
        if total and m:
            fin = vals[vals > -np.inf].astype(np.float64)
            z = np.exp((fin - fin.max()) / t).sum()
            rec[b, 2 + 2 * kmax:4 + 2 * kmax] = np.array([z], np.float64).view(np.uint32)
    return rec


def np_nucleus(allrec, b, V, kmax, t, p, u):
    """Restatement of the merge for a top-p row without top-k: the token, or
    None when the nucleus may reach past the candidates."""
    vals, ids, zs, ms, cut = [], [], [], [], -np.inf
    for r in range(allrec.shape[0]):
        m = int(allrec[r, b, 0])
        if m == 0:
            continue
        v = key_to_f32(allrec[r, b, 2:2 + m]).astype(np.float64)
        vals.append(v)
        ids.append(allrec[r, b, 2 + kmax:2 + kmax + m].astype(np.int64))
        zs.append(allrec[r, b, 2 + 2 * kmax:4 + 2 * kmax].copy().view(np.float64)[0])
        ms.append(v[0])
        if m == kmax:
            cut = max(cut, v[-1])
    v = np.concatenate(vals)
    i = np.concatenate(ids)
    order = np.lexsort((i, -v))
    v, i = v[order], i[order]
    M = v[0]
    Z = sum(z * np.exp((m - M) / t) for z, m in zip(zs, ms))
    w = np.exp(v / t - M / t)
    j = int(np.searchsorted(np.cumsum(w), p * Z))  # first cumsum >= p*Z
    if j >= len(v) or not v[j] > cut:
        return None
    keep = np.argsort(i[:j + 1], kind="stable")
    ki, kw = i[:j + 1][keep], w[:j + 1][keep]
    if not u > 0.0:
        return 0
    c = np.cumsum(kw)
    hit = np.nonzero(c >= u * c[-1])[0]
    return int(ki[hit[0]]) if hit.size else V - 1


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
