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


NU_BINS, NU_RANGE = 16384, 20.0


def np_distributed_nucleus(slices, bounds, t, p, u, V):
    """Restatement of the distributed nucleus (ms_nucleus_* in
    include/mssample.h) for one row without top-k, in float64: the ranks'
    fixed-point histograms over (M - v) / T summed, the bracket of bins that
    must hold the top-p crossing, each slice's mass above the bracket and the
    bracket's values, the exact cut on the ranked bracket values, each rank's
    kept mass, the owner of the index-order target and its draw.  `slices`:
    each rank's fp32 values of the row.  Returns the token, or None when the
    bracket cannot place the crossing (the full-row path)."""
    M = max(float(s[s > -np.inf].max()) for s in slices if np.any(s > -np.inf))
    xs = NU_BINS / (NU_RANGE * t)

    def weights_bins(s):
        v = s.astype(np.float64)
        fin = v > -np.inf
        w = np.where(fin, np.exp((np.where(fin, v, M) - M) / t), 0.0)
        z = (M - np.where(fin, v, -1e300)) * xs
        b = np.where(z < NU_BINS, np.floor(np.minimum(z, NU_BINS)), NU_BINS).astype(np.int64)
        return fin, w, b

    if p < 1.0:
        # each value adds round(scale * its weight relative to its bin's upper
        # edge); bin b then carries e^-(b dz) * hist[b] / scale
        scale = float(min(65535, (2**31 - 1) // V))
        dz = NU_RANGE / NU_BINS
        hist = np.zeros(NU_BINS, np.float64)
        for s in slices:
            fin, w, b = weights_bins(s)
            sel = fin & (b < NU_BINS)
            z = (M - s.astype(np.float64)[sel]) / t
            q = np.rint(scale * np.exp(-(z / dz - b[sel]) * dz))
            np.add.at(hist, b[sel], q)
        c = np.cumsum(hist * np.exp(-np.arange(NU_BINS) * dz))
        Z = c[-1]
        tol = 2.0 * (0.51 / scale + 1e-5) * Z
        lo = np.nonzero(c > p * Z - tol)[0]
        hi = np.nonzero(c >= p * Z + tol)[0]
        b_lo = int(lo[0]) if lo.size else NU_BINS
        b_hi = int(hi[0]) if hi.size else NU_BINS
    else:
        b_lo = b_hi = NU_BINS + 1
    above, total, ents = [], [], []
    for r, s in enumerate(slices):
        fin, w, b = weights_bins(s)
        above.append(w[fin & (b < b_lo)].sum())
        total.append(w[fin].sum())
        sel = np.nonzero(fin & (b >= b_lo) & (b <= b_hi))[0]
        ents += [(float(s[i]), bounds[r] + int(i), w[i]) for i in sel]
    A, Z = sum(above), sum(total)
    ents.sort(key=lambda e: (-e[0], e[1]))
    kept_ids = None  # None: every value kept
    if p < 1.0:
        need = p * Z
        run = A + np.cumsum([e[2] for e in ents]) if ents else np.zeros(0)
        j = np.nonzero(run >= need)[0]
        if A >= need or (not j.size and b_hi < NU_BINS):
            return None
        if j.size:
            kept_ids = {e[1]: e[2] for e in ents[: int(j[0]) + 1]}
    kr = []
    for r in range(len(slices)):
        if kept_ids is None:
            kr.append(total[r])
        else:
            kr.append(above[r] + sum(w for i, w in kept_ids.items() if bounds[r] <= i < bounds[r + 1]))
    K = sum(kr)
    target = u * K
    pre, owner = 0.0, None
    for r, k in enumerate(kr):
        if pre + k >= target and (k > 0 or not u > 0.0):
            owner = r
            break
        pre += k
    if owner is None:
        return V - 1
    s = slices[owner]
    fin, w, b = weights_bins(s)
    if kept_ids is not None:
        ids = bounds[owner] + np.arange(len(s))
        cutv, cuti = min(((e[0], e[1]) for e in ents if e[1] in kept_ids), key=lambda e: (e[0], -e[1]))
        keep = fin & ((s.astype(np.float64) > cutv) | ((s.astype(np.float64) == cutv) & (ids <= cuti)))
        w = np.where(keep, w, 0.0)
    c = np.cumsum(w)
    hit = np.nonzero(c >= target - pre)[0]
    return int(bounds[owner] + hit[0]) if hit.size else int(bounds[owner] + len(s) - 1)
