"""Shared comparison: GPU sampler vs the C oracle (and the reference's tokens)."""
from __future__ import annotations

import numpy as np

import oracle

BOUNDARY = 1e-6      # rows whose top-p or CDF margin is below this are reported, not failed
PROB_RTOL = 1e-5     # relative tolerance on the returned probability


def gpu_sample(sampler, batch_logits, T, K, P, U, *, bf16=False, mask=None):
    import torch
    arr = np.ascontiguousarray(batch_logits)
    if bf16:
        x = torch.from_numpy(arr.view(np.int16)).cuda().view(torch.bfloat16)
    else:
        x = torch.from_numpy(arr).cuda()
    m = None if mask is None else torch.from_numpy(mask.view(np.int32)).cuda()
    tok, prob, st = sampler.sample_batch(x, T, K, P, uniforms=U, mask=m)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), prob.cpu().numpy().astype(np.float64), st.cpu().numpy()


def compare(tok, prob, st, logits, T, K, P, U, *, bf16=False, mask=None, label=""):
    """Assert parity; return the number of boundary rows (reported, not failed)."""
    o_tok, o_prob, o_st, mp, mu = oracle.c_sample(logits, T, K, P, U, mask, bf16_bits=bf16)
    boundary = (mp < BOUNDARY) | (mu < BOUNDARY)
    strict = ~boundary
    assert np.array_equal(st, o_st), f"{label}: status {st} vs {o_st}"
    bad = np.nonzero(strict & (tok != o_tok))[0]
    assert bad.size == 0, (f"{label}: token mismatch rows {bad[:10].tolist()} gpu={tok[bad[:10]].tolist()} "
                           f"oracle={o_tok[bad[:10]].tolist()}")
    ok = strict & (o_tok >= 0)
    err = np.abs(prob[ok] - o_prob[ok])
    tol = PROB_RTOL * np.abs(o_prob[ok]) + 1e-30
    badp = np.nonzero(err > tol)[0]
    assert badp.size == 0, f"{label}: prob mismatch {prob[ok][badp[:5]]} vs {o_prob[ok][badp[:5]]}"
    nb = int(boundary.sum())
    if nb:
        print(f"{label}: {nb} boundary rows (margins < {BOUNDARY}), tokens gpu/oracle: "
              f"{list(zip(tok[boundary].tolist(), o_tok[boundary].tolist()))[:8]}")
    return nb
