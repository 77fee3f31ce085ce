"""CPU oracle for the token-sampling path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg and the
``--impl reference`` arm) may import it.  The shipped sampler runs on the GPU
through ``libmssample.so`` and fails loudly when that library is missing.

It restates miniserve's ``Sampler.sample`` (miniserve/sampler.py:23-68) step
by step in float64 Python, and additionally reports what the reference keeps
internal:

* ``prob``     -- the final (post top-k, post top-p, renormalised) probability
                  of the returned token (miniserve/sampler.py:60);
* ``margin_p`` -- distance of the top-p running sum to ``top_p`` on both sides
                  of the cut (miniserve/sampler.py:53-57);
* ``margin_u`` -- distance of the index-order CDF to the uniform ``r`` on both
                  sides of the chosen token (miniserve/sampler.py:62-67).

The uniform ``r`` is passed in; ``uniform_for_seed(seed)`` returns exactly the
``random.Random(seed).random()`` the reference draws (miniserve/sampler.py:32,62).

Parity pin: ``tests/golden/make_golden.py`` imports the reference sampler in a
container that has it, runs it on seeded rows and commits the tokens; the
tests check this restatement (and the C restatement in ``ms_oracle.c``)
against those tokens.
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass
from typing import List, Optional, Sequence

# Row status codes shared with the CUDA library (include/mssample.h).
ROW_OK = 0
ROW_ALL_MASKED = 1        # reference raises ZeroDivisionError (sampler.py:46-47)
ROW_BAD_TEMPERATURE = 2   # temperature < 0, NaN or infinite: outside the supported domain
ROW_NONFINITE = 4         # NaN or +inf logit present (reference result is arbitrary)

BOUNDARY_EPS = 1e-6


def uniform_for_seed(seed: Optional[int]) -> float:
    """The reference's draw: ``random.Random(seed).random()`` (sampler.py:32,62)."""
    return random.Random(seed).random()


def py_sum(values: Sequence[float]) -> float:
    """CPython >= 3.12 ``sum()`` of floats: Neumaier-compensated summation.

    Restates builtins.sum's float loop (Python/bltinmodule.c, 3.12): a running
    sum ``s`` and compensation ``c``; the compensation is added at the end when
    it is non-zero and finite.  ``tests/test_oracle.py`` checks this against
    the interpreter's own ``sum``.
    """
    s = 0.0
    c = 0.0
    for x in values:
        t = s + x
        if abs(s) >= abs(x):
            c += (s - t) + x
        else:
            c += (x - t) + s
        s = t
    if c and math.isfinite(c):
        s += c
    return s


@dataclass
class RowResult:
    token: int
    prob: float
    status: int
    margin_p: float = math.inf
    margin_u: float = math.inf
    n_kept: int = 0

    @property
    def boundary(self) -> bool:
        return self.margin_p < BOUNDARY_EPS or self.margin_u < BOUNDARY_EPS


def sample_row(logits: Sequence[float], temperature: float, top_k: int, top_p: float,
               u: float) -> RowResult:
    """One row, the reference's float64 steps (miniserve/sampler.py:33-68)."""
    n = len(logits)
    logits = [float(v) for v in logits]
    # greedy: first maximal index (sampler.py:33-34)
    if temperature == 0.0:
        best = 0
        for i in range(1, n):
            if logits[i] > logits[best]:
                best = i
        return RowResult(best, 1.0, ROW_OK)
    if not (temperature > 0.0) or math.isinf(temperature):
        return RowResult(-1, 0.0, ROW_BAD_TEMPERATURE)
    # temperature scale (sampler.py:35)
    scaled = [l / temperature for l in logits]
    # top-k: stable descending sort, first k kept (sampler.py:37-42)
    if top_k > 0:
        order = sorted(range(n), key=lambda i: scaled[i], reverse=True)[:top_k]
        filtered = [-math.inf] * n
        for i in order:
            filtered[i] = scaled[i]
        scaled = filtered
    # softmax (sampler.py:44-47)
    max_v = max(scaled)
    exps = [math.exp(v - max_v) if v != -math.inf else 0.0 for v in scaled]
    total = py_sum(exps)
    if total == 0.0:
        return RowResult(-1, 0.0, ROW_ALL_MASKED)
    probs = [e / total for e in exps]
    margin_p = math.inf
    # top-p nucleus (sampler.py:49-60)
    if top_p < 1.0:
        sorted_idx = sorted(range(n), key=lambda i: probs[i], reverse=True)
        cumsum = 0.0
        keep = set()
        prev = 0.0
        for i in sorted_idx:
            prev = cumsum
            cumsum += probs[i]
            keep.add(i)
            if cumsum >= top_p:
                margin_p = min(cumsum - top_p, top_p - prev)
                break
        else:
            margin_p = top_p - cumsum
        probs = [p if i in keep else 0.0 for i, p in enumerate(probs)]
        total = py_sum(probs)
        probs = [p / total for p in probs]
    # index-order inverse CDF draw (sampler.py:62-68)
    cumulative = 0.0
    for i, p in enumerate(probs):
        prev = cumulative
        cumulative += p
        if u <= cumulative:
            return RowResult(i, p, ROW_OK, margin_p, min(cumulative - u, u - prev if p > 0 else math.inf),
                             sum(1 for q in probs if q > 0.0))
    return RowResult(n - 1, probs[n - 1], ROW_OK, margin_p, u - cumulative,
                     sum(1 for q in probs if q > 0.0))


def sample_token(logits: Sequence[float], temperature: float, top_k: int, top_p: float, u: float) -> int:
    """The token alone, in the reference's own steps and calls
    (miniserve/sampler.py:33-68): builtins ``sum`` (which ``py_sum``
    restates and the tests pin), no margins.  Used to time the reference
    algorithm on the host (bench.py), where sample_row's bookkeeping would
    make the CPU baseline slower than the reference itself."""
    n = len(logits)
    if temperature == 0.0:
        return max(range(n), key=lambda i: logits[i])
    if not (temperature > 0.0) or math.isinf(temperature):
        return -1
    scaled = [l / temperature for l in logits]
    if top_k > 0:
        order = sorted(range(n), key=lambda i: scaled[i], reverse=True)[:top_k]
        filtered = [-math.inf] * n
        for i in order:
            filtered[i] = scaled[i]
        scaled = filtered
    max_v = max(scaled)
    exps = [math.exp(v - max_v) if v != -math.inf else 0.0 for v in scaled]
    total = sum(exps)
    if total == 0.0:
        return -1
    probs = [e / total for e in exps]
    if top_p < 1.0:
        sorted_idx = sorted(range(n), key=lambda i: probs[i], reverse=True)
        cumsum = 0.0
        keep = set()
        for i in sorted_idx:
            cumsum += probs[i]
            keep.add(i)
            if cumsum >= top_p:
                break
        probs = [p if i in keep else 0.0 for i, p in enumerate(probs)]
        total = sum(probs)
        probs = [p / total for p in probs]
    cumulative = 0.0
    for i, p in enumerate(probs):
        cumulative += p
        if u <= cumulative:
            return i
    return n - 1


def sample_rows(rows, temperature, top_k, top_p, uniforms) -> List[RowResult]:
    """Row loop over a 2-D array-like (one reference call per row)."""
    out = []
    for b in range(len(rows)):
        out.append(sample_row(list(map(float, rows[b])), float(temperature[b]), int(top_k[b]),
                              float(top_p[b]), float(uniforms[b])))
    return out
